// q8_gemm.cu -- Q8F projections of a prompt (prefill) on the tcgen05 tensor
// cores, with the weights dequantised tile by tile on load.
//
// Replaces Linear::forward of the Q8F weights at seq_len > 1 (inventwithdean/
// Qwen-3.5 src/text_modules.rs:499-506 in_proj_qkv / in_proj_z, :663
// out_proj, :858-888 q/k/v_proj, :941 o_proj, :1003-1009 up/gate/down):
//   Y[T, N] = X[T, K] W[K, N],  W[k, n] = fl(q[k, n] * s[k, n / 64])
// with q int8 stored 4 per u32 word (byte j of word c = column 4c + j) and f32
// scales [K, N/64] -- the dense f32 weight the reference multiplies with.  No
// dense copy of W is made: each CTA turns the int8 tile it streams into bf16
// operand tiles in shared memory.
//
// Arithmetic: x = x_hi + x_lo and w = w_hi + w_lo with bf16 terms;
// Y = x_hi w_hi + x_hi w_lo + x_lo w_hi on kind::f16 MMAs with f32
// accumulation in TMEM (relative error near 2^-16 per product, far inside the
// attention path's 1e-3 parity bar).  q is converted exactly (int8 values are
// integers below 2^8) and w = q * s is rounded once to f32, as the reference's
// dequantisation does.
//
// Two launches per call:
//  (1) q8_gemm_split_x: x once into bf16 hi / lo (round to nearest), written
//      as [128-row tile][32-k slab][term] blocks already in the MMA's K-major
//      core-matrix layout, so the GEMM fetches each as one bulk copy;
//  (2) q8_gemm_kernel: CTA tile = 128 tokens x NH halves of 128 output
//      columns.  Each half is (segment, first column), so one launch serves up
//      to four projections of the same input (a tile never straddles two), and
//      in SwiGLU mode a tile pairs up-projection and gate-projection columns
//      n0 .. n0+127 in one N=256 accumulator whose epilogue writes
//      up * silu(gate).
//        warp 0 (one thread)  2-D TMA loads of the int8 words and scales
//                             (4-stage ring, freed by the converters);
//        warp 2 (one thread)  bulk copies of the x blocks (3-stage ring, freed
//                             by the MMA commit);
//        warp 1 (one thread)  per 32-k stage 2 K-steps x 3 products, N = 128 NH;
//        warps 3-18           four groups of four warps: group g dequantises
//                             and splits the weight tiles of stages g, g+4, ...
//                             into bf16 hi / lo in operand buffer g; then all
//                             sixteen run the epilogue.
//      The weight split avoids the bf16 conversion instructions (they issue on
//      a quarter-rate pipe; a profile of that form showed them as the limit):
//      the int8 -> float conversion is a byte permute into the mantissa of
//      2^23 and an exact subtraction (packed f32x2), hi is w rounded to its
//      leading 8 bits by an integer add of half an ulp and a mask, and
//      lo = w - hi is exact and keeps its leading 8 bits.
// The operands use the no-swizzle K-major layout (8 x 16-byte core matrices,
// 128-byte aligned, 8-row groups 512 bytes apart).
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace q35 {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 32;
constexpr int kAS = 3;             // x-block stages (released by the MMA commit)
constexpr int kConvWarps = 16;
constexpr int kConvWarp0 = 3;      // warps 0 (weight loads), 1 (MMA), 2 (x loads), then the converters
constexpr int kGemmThreads = 32 * (kConvWarp0 + kConvWarps);
constexpr uint32_t kSboA = 512;
constexpr uint32_t kSboB = 512;
constexpr uint32_t kTermBytes = kBM * kBK * 2;  // one bf16 term of a [128 x 32] x block
constexpr int kMaxSeg = 4;

// A CTA tile is MS row blocks of 128 tokens x NH halves of 128 columns.
// Stage s is converted by converter group s % G (16 / G warps each), into the
// group's own weight-tile and operand buffers.
template <int NH, int MS>
struct GemmSmem {
  static constexpr int G = (NH == 2 && MS == 2) ? 2 : 4;
  uint8_t rawA[kAS][MS][2][kTermBytes];  // x [hi, lo] per row block, MMA layout, from the split kernel
  uint32_t rawQ[G][NH][kBK * 32];        // per half [32 k][32 words]
  float rawS[G][NH][kBK * 4];            // per half [32 k][4 column blocks]
  uint8_t opB[G][2][NH * 16 * kSboB];    // w [hi, lo], 128 NH rows
  uint64_t a_full[kAS], a_empty[kAS], q_full[G], q_empty[G], op_full[G], op_empty[G], acc_full;
  uint32_t tbase;
};
static_assert(sizeof(GemmSmem<2, 1>) + 128 <= 227 * 1024, "GEMM shared memory");
static_assert(sizeof(GemmSmem<2, 2>) + 128 <= 227 * 1024, "GEMM shared memory");
static_assert(sizeof(GemmSmem<1, 2>) + 128 <= 227 * 1024, "GEMM shared memory");

struct GemmParams {
  CUtensorMap qmap[kMaxSeg], smap[kMaxSeg];
  const uint8_t *xs;       // split x blocks
  float *y[kMaxSeg];
  int n_out[kMaxSeg];      // out_dim per segment
  int tile_end[kMaxSeg];   // running count of tiles up to and including each segment (plain mode)
  int n_seg, swiglu;
  uint32_t *status;
  uint64_t wait_ns;
  int T, K;
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

__device__ __forceinline__ uint32_t pack_bf16x2_rn(float lo_elem, float hi_elem) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi_elem), "f"(lo_elem));
  return r;
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// ---------------------------------------------------------------------------
// (1) x [T, K] f32 -> blocks [ceil(T/128)][K/32][hi, lo] of [128 rows x 32 k]
// bf16 in the K-major core-matrix layout (row r, k-group g at
// (r / 8) * 512 + g * 128 + (r % 8) * 16 bytes).  Rows >= T are zero.
// One thread = one (row, 8-k group); a block = one [128 x 32] tile.
__global__ void __launch_bounds__(512) q8_gemm_split_x(const float *__restrict__ x, uint8_t *__restrict__ xs,
                                                     int T, int K) {
  pdl_entry();
  const int ks = blockIdx.x, mt = blockIdx.y, nks = gridDim.x;
  const int r = threadIdx.x >> 2, g = threadIdx.x & 3;
  const int t = mt * kBM + r;
  float v[8];
  if (t < T) {
    const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)t * K + ks * kBK + 8 * g);
    const float4 a = __ldg(src), b = __ldg(src + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.0f;
  }
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    h[i] = pack_bf16x2_rn(v[2 * i], v[2 * i + 1]);
    const float h0 = __uint_as_float(h[i] << 16), h1 = __uint_as_float(h[i] & 0xFFFF0000u);
    l[i] = pack_bf16x2_rn(v[2 * i] - h0, v[2 * i + 1] - h1);
  }
  uint8_t *blk = xs + ((size_t)mt * nks + ks) * 2 * kTermBytes;
  const uint32_t off = (uint32_t)(r >> 3) * kSboA + g * 128 + (r & 7) * 16;
  *reinterpret_cast<uint4 *>(blk + off) = make_uint4(h[0], h[1], h[2], h[3]);
  *reinterpret_cast<uint4 *>(blk + kTermBytes + off) = make_uint4(l[0], l[1], l[2], l[3]);
}

// Packed pairs of f32 (low word = first element) and the sm_100 f32x2 ops,
// round to nearest, no contraction.
__device__ __forceinline__ uint64_t pack2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}


// ---------------------------------------------------------------------------
// (2) the GEMM
template <int NH, int MS>
__global__ void __launch_bounds__(kGemmThreads, 1) q8_gemm_kernel(const __grid_constant__ GemmParams p) {
  using Smem = GemmSmem<NH, MS>;
  constexpr int G = Smem::G, GW = kConvWarps / G;  // groups, warps per group
  extern __shared__ unsigned char smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~static_cast<uintptr_t>(127));
  constexpr int BN = 128 * NH;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tile = blockIdx.x, mb = blockIdx.y * MS, t0 = mb * kBM;  // first row block, first row
  const int nk = p.K / kBK;
  const uint64_t wns = p.wait_ns;
  // the tile's halves: (seg0, col0) and, when NH = 2, (seg1, col0 + dcol)
  int seg0, seg1, col0, dcol;
  if (p.swiglu) {
    seg0 = 0; seg1 = 1; col0 = 128 * tile; dcol = 0;
  } else {
    int s = 0;
    while (s + 1 < p.n_seg && tile >= p.tile_end[s]) ++s;
    seg0 = seg1 = s;
    col0 = BN * (tile - (s == 0 ? 0 : p.tile_end[s - 1]));
    dcol = 128;
  }
  constexpr uint32_t kQBytes = NH * (kBK * 128 + kBK * 16);

  if (warp == 1) {
    umma::tmem_alloc(&sm.tbase, MS * BN);
    umma::tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < kAS; ++i) {
      mbar_init(&sm.a_full[i], 1);
      mbar_init(&sm.a_empty[i], 1);
    }
    for (int i = 0; i < G; ++i) {
      mbar_init(&sm.q_full[i], 1);
      mbar_init(&sm.q_empty[i], GW);
      mbar_init(&sm.op_full[i], GW);
      mbar_init(&sm.op_empty[i], 1);
    }
    mbar_init(&sm.acc_full, 1);
    fence_mbar_init();
    prefetch_tmap(&p.qmap[seg0]);
    prefetch_tmap(&p.smap[seg0]);
    if (NH == 2) {
      prefetch_tmap(&p.qmap[seg1]);
      prefetch_tmap(&p.smap[seg1]);
    }
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tb = sm.tbase;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {  // ---- weight tiles: 2-D TMA of the int8 words and the scales
      int issued = 0;
      for (int s = 0; s < nk; ++s) {
        const int slot = s % G;
        if (s >= G && !mbar_wait_ns(&sm.q_empty[slot], ((s / G) - 1) & 1, wns)) ok = false;
        if (!ok) break;
        mbar_arrive_expect_tx(&sm.q_full[slot], kQBytes);
#pragma unroll
        for (int h = 0; h < NH; ++h) {
          const int sg = h == 0 ? seg0 : seg1, cl = col0 + h * dcol;
          tma_load_2d(sm.rawQ[slot][h], &p.qmap[sg], cl / 4, s * kBK, &sm.q_full[slot]);
          // the scale box starts on a 4-block (16-byte) boundary; the half uses
          // 2 of its 4 blocks, from block (col / 64) % 4
          tma_load_2d(sm.rawS[slot][h], &p.smap[sg], (cl / 256) * 4, s * kBK, &sm.q_full[slot]);
        }
        issued = s + 1;
      }
      for (int s = max(0, issued - G); s < issued; ++s)  // nothing of ours is in flight at exit
        (void)mbar_wait_ns(&sm.q_full[s % G], (s / G) & 1, wns);
    }
  } else if (warp == 2) {
    if (lane == 0) {  // ---- x blocks (written by the split kernel: wait for it here only)
      pdl_entry();
      int issued = 0;
      for (int s = 0; s < nk; ++s) {
        const int slot = s % kAS;
        if (s >= kAS && !mbar_wait_ns(&sm.a_empty[slot], ((s / kAS) - 1) & 1, wns)) ok = false;
        if (!ok) break;
        mbar_arrive_expect_tx(&sm.a_full[slot], MS * 2 * kTermBytes);
#pragma unroll
        for (int ms = 0; ms < MS; ++ms)
          bulk_g2s_nohint(sm.rawA[slot][ms][0], p.xs + ((size_t)(mb + ms) * nk + s) * 2 * kTermBytes,
                          2 * kTermBytes, &sm.a_full[slot]);
        issued = s + 1;
      }
      for (int s = max(0, issued - kAS); s < issued; ++s)
        (void)mbar_wait_ns(&sm.a_full[s % kAS], (s / kAS) & 1, wns);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issue: per stage and row block 2 K-steps x 3 products
      constexpr uint32_t id = idesc_bf16(kBM, BN);
      for (int s = 0; s < nk; ++s) {
        const int os = s % G, as = s % kAS;
        if (!mbar_wait_ns(&sm.a_full[as], (s / kAS) & 1, wns)) ok = false;
        if (ok && !mbar_wait_ns(&sm.op_full[os], (s / G) & 1, wns)) ok = false;
        if (!ok) break;
        umma::fence_after_sync();
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const uint64_t bh = umma::smem_desc(sm.opB[os][0] + 256 * kk, 128, kSboB);
          const uint64_t bl = umma::smem_desc(sm.opB[os][1] + 256 * kk, 128, kSboB);
#pragma unroll
          for (int ms = 0; ms < MS; ++ms) {
            const uint64_t ah = umma::smem_desc(sm.rawA[as][ms][0] + 256 * kk, 128, kSboA);
            const uint64_t al = umma::smem_desc(sm.rawA[as][ms][1] + 256 * kk, 128, kSboA);
            const uint32_t d = tb + ms * BN;
            mma_bf16(d, ah, bh, id, (s > 0 || kk > 0) ? 1u : 0u);
            mma_bf16(d, ah, bl, id, 1u);
            mma_bf16(d, al, bh, id, 1u);
          }
        }
        umma::commit(&sm.op_empty[os]);
        umma::commit(&sm.a_empty[as]);
      }
      umma::commit(&sm.acc_full);  // arrives once every MMA issued above is complete
      if (!mbar_wait_ns(&sm.acc_full, 0, wns)) ok = false;
    }
  } else {
    // ---- converters: G groups; group g converts stages g, g + G, ... into its
    // own operand buffer, so G stages are in conversion at once and the fixed
    // latency of each (waits, proxy fence, arrivals) overlaps.  A warp takes
    // one k group (8 k rows) of the stage for PW passes of 32 columns: lane =
    // one column n, its 8 int8 weights are byte n % 4 of word n / 4 in 8 rows
    // (four lanes share each word load), and its hi / lo terms are one 16-byte
    // core-matrix row each.  A quarter warp stores 8 consecutive columns, i.e.
    // 8 distinct 16-byte slots of one 128-byte core matrix: no bank conflicts.
    const int cw = warp - kConvWarp0, grp = cw / GW, wi = cw % GW;
    const int kg = wi & 3;
    constexpr int PW = 16 * NH / GW;  // passes per warp
    const int gp0 = (wi >> 2) * PW;   // first global pass (h = pass / 4, 32-column chunk = pass % 4)
    const uint64_t kMagic2 = pack2(8388736.0f, 8388736.0f);
    const uint32_t sel = 0x7540u | (uint32_t)(lane & 3);  // byte n % 4 into the mantissa of 2^23
    for (int s = grp; s < nk; s += G) {
      const int slot = grp;  // = s % G
      const uint32_t ph = (uint32_t)(s / G) & 1u;
      if (ok && !mbar_wait_ns(&sm.q_full[slot], ph, wns)) ok = false;
      if (ok && s >= G && !mbar_wait_ns(&sm.op_empty[slot], ph ^ 1u, wns)) ok = false;
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      uint8_t *bh = sm.opB[slot][0], *bl = sm.opB[slot][1];
#pragma unroll 1
      for (int pp = 0; pp < PW; ++pp) {
        const int gp = gp0 + pp;
        const int h = gp >> 2, nl = 32 * (gp & 3) + lane;  // half, column within the half
        const int hc = col0 + h * dcol;
        const uint32_t *rq = sm.rawQ[slot][h] + (8 * kg) * 32 + (nl >> 2);
        const float *rsc = sm.rawS[slot][h] + (8 * kg) * 4 + ((hc / 64) & 3) + (nl >> 6);
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          // rows 2i, 2i+1: 2^23 + (v + 128) as floats, then the exact v, then fl(v s)
          const float m0 = __uint_as_float(__byte_perm(rq[(2 * i) * 32] ^ 0x80808080u, 0x4B000000u, sel));
          const float m1 = __uint_as_float(__byte_perm(rq[(2 * i + 1) * 32] ^ 0x80808080u, 0x4B000000u, sel));
          const uint64_t w2 = mul2(sub2(pack2(m0, m1), kMagic2), pack2(rsc[(2 * i) * 4], rsc[(2 * i + 1) * 4]));
          // hi = w rounded to its leading 8 bits (add half an ulp of bit 16, cut
          // the low 16 bits), lo = w - hi exactly
          const uint32_t w0 = (uint32_t)w2, w1 = (uint32_t)(w2 >> 32);
          const uint32_t r0 = w0 + 0x8000u, r1 = w1 + 0x8000u;
          const uint64_t lo2 = sub2(w2, pack2(__uint_as_float(r0 & 0xFFFF0000u), __uint_as_float(r1 & 0xFFFF0000u)));
          // bf16 = the upper 16 bits (hi has 8 significant bits; lo keeps its leading 8)
          hw[i] = __byte_perm(r0, r1, 0x7632u);
          lw[i] = __byte_perm((uint32_t)lo2, (uint32_t)(lo2 >> 32), 0x7632u);
        }
        const int n = 128 * h + nl;
        const uint32_t off = (uint32_t)(n >> 3) * kSboB + kg * 128 + (n & 7) * 16;
        *reinterpret_cast<uint4 *>(bh + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4 *>(bl + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.op_full[slot]);
        mbar_arrive(&sm.q_empty[slot]);
      }
    }
    // ---- epilogue: TMEM lane = token row of a row block, column = ms * BN +
    // output column; four warps per lane quadrant split MS * BN columns
    if (ok && !mbar_wait_ns(&sm.acc_full, 0, wns)) ok = false;
    ok = __all_sync(0xffffffffu, ok);
    umma::fence_after_sync();
    const int quad = warp & 3, wq = cw >> 2;
    const int ms = MS == 2 ? wq >> 1 : 0, part = MS == 2 ? wq & 1 : wq;  // row block, column part
    constexpr int kParts = 4 / MS;
    const int t = t0 + 128 * ms + 32 * quad + lane;
    const uint32_t lrow = ((uint32_t)(32 * quad) << 16) + ms * BN;
    if (NH == 2 && p.swiglu) {
      // columns 0-127 up, 128-255 gate: y0 = up * silu(gate)
      constexpr int kCols = 128 / kParts;
      float *yr = p.y[0] + (size_t)t * p.n_out[0] + col0 + kCols * part;
#pragma unroll 1
      for (int cc = 0; cc < kCols / 16; ++cc) {
        float a[16], g[16];
        umma::ld_32x32b_x16(tb + lrow + kCols * part + 16 * cc, a);
        umma::ld_32x32b_x16(tb + lrow + 128 + kCols * part + 16 * cc, g);
        umma::wait_ld();
        if (ok && t < p.T) {
          float4 *dst = reinterpret_cast<float4 *>(yr + 16 * cc);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[i] = make_float4(a[4 * i] * siluf_dev(g[4 * i]), a[4 * i + 1] * siluf_dev(g[4 * i + 1]),
                                 a[4 * i + 2] * siluf_dev(g[4 * i + 2]), a[4 * i + 3] * siluf_dev(g[4 * i + 3]));
        }
      }
    } else {
      // plain: the tile's columns are col0 .. col0 + BN - 1 of segment seg0
      constexpr int kCols = BN / kParts;
      float *yr = p.y[seg0] + (size_t)t * p.n_out[seg0] + col0 + kCols * part;
#pragma unroll 1
      for (int cc = 0; cc < kCols / 16; ++cc) {
        float v[16];
        umma::ld_32x32b_x16(tb + lrow + kCols * part + 16 * cc, v);
        umma::wait_ld();
        if (ok && t < p.T) {
          float4 *dst = reinterpret_cast<float4 *>(yr + 16 * cc);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
      }
    }
  }

  umma::fence_before_sync();
  const int failed = __syncthreads_or(ok ? 0 : 1);
  if (failed && tid == 0) {  // a bounded wait gave up: flag it and poison the tile
    atomicOr(p.status, Q35_STATUS_WAIT_TIMEOUT);
    if (t0 < p.T) p.y[seg0][(size_t)t0 * p.n_out[seg0] + col0] = __int_as_float(0x7fc00000);
  }
  if (warp == 1) umma::tmem_dealloc(tb, MS * BN);
}

template <int NH, int MS>
int launch_cfg(const GemmParams &p, int tiles, int mt, cudaStream_t st) {
  const size_t smem = sizeof(GemmSmem<NH, MS>) + 128;
  auto kern = q8_gemm_kernel<NH, MS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "q8_gemm attributes");
  note_launch();
  (void)launch_kernel(kern, dim3(tiles, (mt + MS - 1) / MS), dim3(kGemmThreads), smem, st, 1, 1, p);
  return check_cuda(cudaGetLastError(), "q8_gemm launch");
}

}  // namespace

// Row blocks of the split x, padded to an even count (a two-block CTA reads a
// zero block past the last one).
static int padded_row_blocks(int T) { return ((T + kBM - 1) / kBM + 1) & ~1; }

size_t q8_gemm_workspace_bytes(int T, int K) {
  return (size_t)padded_row_blocks(T) * (size_t)(K / kBK) * 2 * kTermBytes;
}

int q8_gemm_launch(int T, int K, int n_seg, const q35_q8_segment *segs, const float *x, int swiglu, void *ws,
                   size_t ws_bytes, cudaStream_t st) {
  Q35_REQUIRE(n_seg >= 1 && n_seg <= kMaxSeg, Q35_ERR_INVALID_ARG, "q8_gemm: 1 to 4 segments");
  Q35_REQUIRE(K % kBK == 0, Q35_ERR_UNSUPPORTED, "q8_gemm: in_dim must be a multiple of 32");
  Q35_REQUIRE(!swiglu || (n_seg == 2 && segs[0].out_dim == segs[1].out_dim), Q35_ERR_INVALID_ARG,
              "q8_gemm: swiglu needs exactly two segments (up, gate) of equal out_dim");
  for (int i = 0; i < n_seg; ++i)
    Q35_REQUIRE(segs[i].out_dim > 0 && segs[i].out_dim % 256 == 0, Q35_ERR_UNSUPPORTED,
                "q8_gemm: every out_dim must be a positive multiple of 256");
  const size_t need = q8_gemm_workspace_bytes(T, K);
  Q35_REQUIRE(ws != nullptr && ws_bytes >= need && (reinterpret_cast<uintptr_t>(ws) & 15u) == 0, Q35_ERR_WORKSPACE,
              "q8_gemm: workspace missing, unaligned or too small (need " + std::to_string(need) + " bytes)");
  const EncodeTiledFn encode = encode_tiled_fn();
  Q35_REQUIRE(encode != nullptr, Q35_ERR_DEVICE, "q8_gemm: cuTensorMapEncodeTiled unavailable");
  uint32_t *status = device_status_word();
  Q35_REQUIRE(status != nullptr, Q35_ERR_CUDA, "q8_gemm: device status word unavailable");

  GemmParams p = {};
  p.xs = static_cast<const uint8_t *>(ws);
  p.n_seg = n_seg;
  p.swiglu = swiglu ? 1 : 0;
  p.status = status;
  p.wait_ns = kWaitLimitNs;
  p.T = T;
  p.K = K;
  const int sms = device_sm_count();
  const int mt = (T + kBM - 1) / kBM;
  int halves = 0;
  for (int i = 0; i < n_seg; ++i) halves += segs[i].out_dim / 128;
  // Tile shape (NH halves of 128 columns, MS row blocks of 128): the waves
  // each needs times the tile's time, modelled as MMA work MS * NH (units of a
  // 128 x 128 tile stage) against weight conversion 1.2 NH (independent of MS,
  // the two overlap) plus 0.3 fixed.  SwiGLU needs NH = 2.
  auto cost = [&](int nh, int msub) {
    const long long ctas = (long long)((mt + msub - 1) / msub) * (halves / nh);
    const double per = std::max((double)(msub * nh), 1.2 * nh);
    return (double)((ctas + sms - 1) / sms) * (per + 0.3);
  };
  int NH = 2, MS = 1;
  double best = 1e30;
  for (int nh = swiglu ? 2 : 1; nh <= 2; ++nh)
    for (int msub = 1; msub <= 2; ++msub)
      if (cost(nh, msub) < best - 1e-9) {
        best = cost(nh, msub);
        NH = nh;
        MS = msub;
      }
  int tiles = 0;
  const cuuint32_t es[2] = {1, 1};
  for (int i = 0; i < n_seg; ++i) {
    const int N = segs[i].out_dim;
    Q35_REQUIRE(segs[i].w != nullptr && segs[i].scales != nullptr && segs[i].y != nullptr &&
                    (reinterpret_cast<uintptr_t>(segs[i].w) & 15u) == 0 &&
                    (reinterpret_cast<uintptr_t>(segs[i].scales) & 15u) == 0 &&
                    (reinterpret_cast<uintptr_t>(segs[i].y) & 15u) == 0,
                Q35_ERR_INVALID_ARG, "q8_gemm: segment pointers must be non-NULL and 16-byte aligned");
    p.y[i] = segs[i].y;
    p.n_out[i] = N;
    tiles += swiglu ? 0 : N / (128 * NH);
    p.tile_end[i] = tiles;
    const cuuint64_t qd[2] = {(cuuint64_t)(N / 4), (cuuint64_t)K};
    const cuuint64_t qs[1] = {(cuuint64_t)N};
    const cuuint32_t qb[2] = {32, kBK};
    Q35_REQUIRE(encode(&p.qmap[i], CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t *>(segs[i].w), qd, qs, qb,
                       es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS,
                Q35_ERR_INVALID_ARG, "q8_gemm: weight tensor map rejected");
    const cuuint64_t sd[2] = {(cuuint64_t)(N / 64), (cuuint64_t)K};
    const cuuint64_t ss[1] = {(cuuint64_t)(N / 64) * sizeof(float)};
    const cuuint32_t sb[2] = {4, kBK};
    Q35_REQUIRE(encode(&p.smap[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(segs[i].scales), sd, ss,
                       sb, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS,
                Q35_ERR_INVALID_ARG, "q8_gemm: scale tensor map rejected");
  }
  if (swiglu) tiles = segs[0].out_dim / 128;
  Q35_REQUIRE(tiles <= 65535 && mt <= 65535, Q35_ERR_UNSUPPORTED, "q8_gemm: problem too large for the grid");

  note_launch();
  (void)launch_kernel(q8_gemm_split_x, dim3(K / kBK, padded_row_blocks(T)), dim3(512), 0, st, 1, 1, x,
                      static_cast<uint8_t *>(ws), T, K);
  if (cudaError_t e = cudaGetLastError(); e != cudaSuccess) return check_cuda(e, "q8_gemm split launch");
  if (NH == 2) return MS == 2 ? launch_cfg<2, 2>(p, tiles, mt, st) : launch_cfg<2, 1>(p, tiles, mt, st);
  return MS == 2 ? launch_cfg<1, 2>(p, tiles, mt, st) : launch_cfg<1, 1>(p, tiles, mt, st);
}

}  // namespace q35
