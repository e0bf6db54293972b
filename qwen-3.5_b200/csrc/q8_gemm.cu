// q8_gemm.cu -- Q8F projections of a prompt (prefill) on the tcgen05 tensor
// cores, with the weights dequantised tile by tile on load.
//
// Replaces Linear::forward of the Q8F weights at seq_len > 1 (inventwithdean/
// Qwen-3.5 src/text_modules.rs:499-506 in_proj_qkv / in_proj_z, :663
// out_proj, :858-888 q/k/v_proj, :941 o_proj, :1003-1009 up/gate/down):
//   Y[T, N] = X[T, K] W[K, N],  W[k, n] = fl(q[k, n] * s[k, n / 64])
// with q int8 stored 4 per u32 word (byte j of word c = column 4c + j) and f32
// scales [K, N/64] -- the dense f32 weight the reference multiplies with.  No
// dense copy of W is ever made: each CTA turns the int8 tile it streams into
// bf16 operand tiles in shared memory.
//
// Arithmetic: x = x_hi + x_lo and w = w_hi + w_lo, each term bf16 (round to
// nearest); Y = x_hi w_hi + x_hi w_lo + x_lo w_hi on kind::f16 MMAs with f32
// accumulation in TMEM.  The dropped x_lo w_lo term and the rounding of the lo
// terms leave a relative error near 2^-16 per product, far inside the 1e-3
// parity bar of the attention path.  q is converted exactly (int8 values are
// integers below 2^8) and w = q * s is rounded once to f32, as the reference's
// dequantisation does.
//
// CTA tile: 128 tokens x BN (128 or 256) columns, K in stages of 32.
//   warp 0 (one thread)  2-D TMA loads of the raw x tile (128-byte swizzle),
//                        the int8 words and the scales into a 3-stage ring;
//   warp 1 (one thread)  the MMAs: per stage 2 K-steps x 3 products, then a
//                        commit that frees the operand buffers;
//   warps 2-9            convert raw tiles into the bf16 hi/lo operands (two
//                        operand buffers), then the epilogue (TMEM -> Y).
// The operands use the no-swizzle K-major layout (8 x 16-byte core matrices);
// B's 8-row groups are 528 bytes apart instead of 512 so the converters'
// 16-byte stores hit 32 distinct banks per quarter warp.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace q35 {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 32;
constexpr int kRS = 3;
constexpr int kOS = 2;
constexpr int kGemmThreads = 320;
constexpr int kConvWarps = 8;
constexpr uint32_t kSboA = 512;
constexpr uint32_t kSboB = 528;

template <int BN>
struct GemmSmem {
  float rawX[kRS][kBM * kBK];          // [128 t][32 k], 128-byte rows, swizzled (1024-byte aligned)
  uint32_t rawQ[kRS][kBK * BN / 4];    // [32 k][BN/4 words]
  float rawS[kRS][kBK * 4];            // [32 k][4 column blocks]
  uint8_t opA[kOS][2][kBM / 8 * kSboA];  // x [hi, lo]
  uint8_t opB[kOS][2][BN / 8 * kSboB];   // w [hi, lo]
  uint64_t raw_full[kRS], raw_empty[kRS], op_full[kOS], op_empty[kOS], acc_full;
  uint32_t tbase;
};
static_assert(sizeof(GemmSmem<256>) + 1024 <= 227 * 1024, "GEMM shared memory");

struct GemmParams {
  CUtensorMap xmap, qmap, smap;
  float *y;
  uint32_t *status;
  uint64_t wait_ns;
  int T, K, N;
};

// kind::f16 instruction descriptor: bf16 A and B (K-major), f32 accumulator.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo_elem, float hi_elem) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi_elem), "f"(lo_elem));
  return r;
}

// Eight consecutive-k values -> one 16-byte core-matrix row of the hi term and
// one of the lo term.
__device__ __forceinline__ void split_store(const float (&v)[8], uint8_t *hi, uint8_t *lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    h[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
    const float h0 = __uint_as_float(h[i] << 16), h1 = __uint_as_float(h[i] & 0xFFFF0000u);
    l[i] = pack_bf16x2(v[2 * i] - h0, v[2 * i + 1] - h1);
  }
  *reinterpret_cast<uint4 *>(hi) = make_uint4(h[0], h[1], h[2], h[3]);
  *reinterpret_cast<uint4 *>(lo) = make_uint4(l[0], l[1], l[2], l[3]);
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1) q8_gemm_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ unsigned char smem_raw[];
  GemmSmem<BN> &sm = *reinterpret_cast<GemmSmem<BN> *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                      ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n0 = blockIdx.x * BN, t0 = blockIdx.y * kBM;
  const int nk = p.K / kBK;
  const uint64_t wns = p.wait_ns;
  constexpr uint32_t kStageBytes = kBM * kBK * 4 + kBK * BN + kBK * 16;

  if (warp == 1) {
    umma::tmem_alloc(&sm.tbase, BN);
    umma::tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < kRS; ++i) {
      mbar_init(&sm.raw_full[i], 1);
      mbar_init(&sm.raw_empty[i], kConvWarps);
    }
    for (int i = 0; i < kOS; ++i) {
      mbar_init(&sm.op_full[i], kConvWarps);
      mbar_init(&sm.op_empty[i], 1);
    }
    mbar_init(&sm.acc_full, 1);
    fence_mbar_init();
    prefetch_tmap(&p.xmap);
    prefetch_tmap(&p.qmap);
    prefetch_tmap(&p.smap);
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tb = sm.tbase;
  pdl_entry();  // x is the previous kernel's output
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {  // ---- producer
      int issued = 0;
      for (int s = 0; s < nk; ++s) {
        const int slot = s % kRS;
        if (s >= kRS && !mbar_wait_ns(&sm.raw_empty[slot], ((s / kRS) - 1) & 1, wns)) ok = false;
        if (!ok) break;
        mbar_arrive_expect_tx(&sm.raw_full[slot], kStageBytes);
        tma_load_2d(sm.rawX[slot], &p.xmap, s * kBK, t0, &sm.raw_full[slot]);
        tma_load_2d(sm.rawQ[slot], &p.qmap, n0 / 4, s * kBK, &sm.raw_full[slot]);
        // the scale box starts on a 4-block (16-byte) boundary; a 128-column
        // tile uses 2 of its 4 blocks, from block (n0 / 64) % 4
        tma_load_2d(sm.rawS[slot], &p.smap, (n0 / 256) * 4, s * kBK, &sm.raw_full[slot]);
        issued = s + 1;
      }
      // every copy this thread started has landed before the CTA retires
      for (int s = max(0, issued - kRS); s < issued; ++s)
        (void)mbar_wait_ns(&sm.raw_full[s % kRS], (s / kRS) & 1, wns);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issue
      constexpr uint32_t id = idesc_bf16(kBM, BN);
      for (int s = 0; s < nk; ++s) {
        const int os = s % kOS;
        if (!mbar_wait_ns(&sm.op_full[os], (s / kOS) & 1, wns)) ok = false;
        if (!ok) break;
        umma::fence_after_sync();
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const uint64_t ah = umma::smem_desc(sm.opA[os][0] + 256 * kk, 128, kSboA);
          const uint64_t al = umma::smem_desc(sm.opA[os][1] + 256 * kk, 128, kSboA);
          const uint64_t bh = umma::smem_desc(sm.opB[os][0] + 256 * kk, 128, kSboB);
          const uint64_t bl = umma::smem_desc(sm.opB[os][1] + 256 * kk, 128, kSboB);
          mma_bf16(tb, ah, bh, id, (s > 0 || kk > 0) ? 1u : 0u);
          mma_bf16(tb, ah, bl, id, 1u);
          mma_bf16(tb, al, bh, id, 1u);
        }
        umma::commit(&sm.op_empty[os]);
      }
      umma::commit(&sm.acc_full);  // arrives once every MMA issued above is complete
      if (!mbar_wait_ns(&sm.acc_full, 0, wns)) ok = false;
    }
  } else {
    // ---- converters (warps 2-9), then the epilogue
    const int cw = warp - 2;
    for (int s = 0; s < nk; ++s) {
      const int rs = s % kRS, os = s % kOS;
      if (ok && !mbar_wait_ns(&sm.raw_full[rs], (s / kRS) & 1, wns)) ok = false;
      if (ok && s >= kOS && !mbar_wait_ns(&sm.op_empty[os], ((s / kOS) - 1) & 1, wns)) ok = false;
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      // x: lane -> row 8 g + (lane & 7), k group lane >> 3 (8 values)
      const float *rx = sm.rawX[rs];
#pragma unroll
      for (int gi = 0; gi < 2; ++gi) {
        const int r = 8 * (cw + 8 * gi) + (lane & 7), kg = lane >> 3;
        const float4 *row = reinterpret_cast<const float4 *>(rx + r * kBK);
        const float4 a = row[(2 * kg) ^ (r & 7)], b = row[(2 * kg + 1) ^ (r & 7)];
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        const uint32_t off = (uint32_t)(r >> 3) * kSboA + kg * 128 + (r & 7) * 16;
        split_store(v, sm.opA[os][0] + off, sm.opA[os][1] + off);
      }
      // w: a task is 8 k rows x 32 words (128 columns); lane = word
      constexpr int kSegs = BN / 128, kTasks = 4 * kSegs;
      const uint32_t *rq = sm.rawQ[rs];
      const float *rsc = sm.rawS[rs] + ((n0 / 64) & 3);
      for (int tk = cw; tk < kTasks; tk += kConvWarps) {
        const int kg = tk / kSegs, n4 = 32 * (tk % kSegs) + lane;
        uint32_t u[8];
        float sc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          u[j] = rq[(8 * kg + j) * (BN / 4) + n4] ^ 0x80808080u;  // bytes v + 128
          sc[j] = rsc[(8 * kg + j) * 4 + (n4 >> 4)];
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float v[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            // 2^23 + (v + 128) as a float, then the exact integer v
            const float m = __uint_as_float(__byte_perm(u[j], 0x4B000000u, 0x7540u | c));
            v[j] = (m - 8388736.0f) * sc[j];
          }
          const int n = 4 * n4 + c;
          const uint32_t off = (uint32_t)(n >> 3) * kSboB + kg * 128 + (n & 7) * 16;
          split_store(v, sm.opB[os][0] + off, sm.opB[os][1] + off);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.op_full[os]);
        mbar_arrive(&sm.raw_empty[rs]);
      }
    }
    // epilogue: TMEM lane = token row, column = output column
    if (ok && !mbar_wait_ns(&sm.acc_full, 0, wns)) ok = false;
    ok = __all_sync(0xffffffffu, ok);
    umma::fence_after_sync();
    const int quad = warp & 3, half = cw >> 2;
    const int t = t0 + 32 * quad + lane;
    float *yrow = p.y + (size_t)t * p.N + n0 + half * (BN / 2);
#pragma unroll 1
    for (int cc = 0; cc < BN / 32; ++cc) {
      float v[16];
      umma::ld_32x32b_x16(tb + ((uint32_t)(32 * quad) << 16) + half * (BN / 2) + 16 * cc, v);
      umma::wait_ld();
      if (ok && t < p.T) {
        float4 *dst = reinterpret_cast<float4 *>(yrow + 16 * cc);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      }
    }
  }

  umma::fence_before_sync();
  const int failed = __syncthreads_or(ok ? 0 : 1);
  if (failed && tid == 0) {  // a bounded wait gave up: flag it and poison the tile
    atomicOr(p.status, Q35_STATUS_WAIT_TIMEOUT);
    if (t0 < p.T) p.y[(size_t)t0 * p.N + n0] = __int_as_float(0x7fc00000);
  }
  if (warp == 1) umma::tmem_dealloc(tb, BN);
}

template <int BN>
int launch_bn(const GemmParams &p, cudaStream_t st) {
  const size_t smem = sizeof(GemmSmem<BN>) + 1024;
  auto kern = q8_gemm_kernel<BN>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "q8_gemm attributes");
  note_launch();
  (void)launch_kernel(kern, dim3(p.N / BN, (p.T + kBM - 1) / kBM), dim3(kGemmThreads), smem, st, 1, 1, p);
  return check_cuda(cudaGetLastError(), "q8_gemm launch");
}

}  // namespace

int q8_gemm_launch(int T, int K, int N, const float *x, const uint32_t *w, const float *scales, float *y,
                   cudaStream_t st) {
  Q35_REQUIRE(K % kBK == 0 && N % 256 == 0, Q35_ERR_UNSUPPORTED,
              "q8_gemm: in_dim must be a multiple of 32 and out_dim a multiple of 256");
  const EncodeTiledFn encode = encode_tiled_fn();
  Q35_REQUIRE(encode != nullptr, Q35_ERR_DEVICE, "q8_gemm: cuTensorMapEncodeTiled unavailable");
  uint32_t *status = device_status_word();
  Q35_REQUIRE(status != nullptr, Q35_ERR_CUDA, "q8_gemm: device status word unavailable");
  GemmParams p;
  p.y = y;
  p.status = status;
  p.wait_ns = kWaitLimitNs;
  p.T = T; p.K = K; p.N = N;
  const cuuint32_t es[2] = {1, 1};
  {
    const cuuint64_t d[2] = {(cuuint64_t)K, (cuuint64_t)T};
    const cuuint64_t str[1] = {(cuuint64_t)K * sizeof(float)};
    const cuuint32_t box[2] = {kBK, kBM};
    Q35_REQUIRE(encode(&p.xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(x), d, str, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS,
                Q35_ERR_INVALID_ARG, "q8_gemm: x tensor map rejected");
  }
  const int sms = device_sm_count();
  const int mt = (T + kBM - 1) / kBM;
  // 256-column tiles when they still give about a wave, else 128 (twice the CTAs)
  const int BN = (long long)mt * (N / 256) * 4 >= 3LL * sms ? 256 : 128;
  {
    const cuuint64_t d[2] = {(cuuint64_t)(N / 4), (cuuint64_t)K};
    const cuuint64_t str[1] = {(cuuint64_t)N};
    const cuuint32_t box[2] = {(cuuint32_t)(BN / 4), kBK};
    Q35_REQUIRE(encode(&p.qmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t *>(w), d, str, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS,
                Q35_ERR_INVALID_ARG, "q8_gemm: weight tensor map rejected");
  }
  {
    const cuuint64_t d[2] = {(cuuint64_t)(N / 64), (cuuint64_t)K};
    const cuuint64_t str[1] = {(cuuint64_t)(N / 64) * sizeof(float)};
    const cuuint32_t box[2] = {4, kBK};
    Q35_REQUIRE(encode(&p.smap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(scales), d, str, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS,
                Q35_ERR_INVALID_ARG, "q8_gemm: scale tensor map rejected");
  }
  return BN == 256 ? launch_bn<256>(p, st) : launch_bn<128>(p, st);
}

}  // namespace q35
