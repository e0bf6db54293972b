// q8_gemv.cu -- Q8F split-K GEMV y = x^T W for the decode projections.
//
// Replaces q8_gemv_partial_sum_kernel + q8_gemv_sum_reduction_kernel
// (inventwithdean/Qwen-3.5 src/kernels.rs:103-165, host side :495-537).
// Weight format (burn QFloat, kernels.rs:104-110): W [in, out] int8 stored as
// [in, out/4] u32 words, byte j of word c (little-endian) = column 4c + j;
// f32 scales [in, out/64], one per (input row, 64-column block).  Each term is
// int8 * x[i] * scale[i][col/64].
//
// B200 layout: at batch 1 these GEMVs move 1-13 MB (lm_head 541 MB), i.e.
// 0.2-2 us at HBM rate, so the design goal is one DRAM round trip per call
// and no cross-CTA reduction (each one costs a further round trip or a
// barrier).  A CTA owns a slab of 32 or 64 output columns over all input
// rows; every thread has 16 rows of 16-byte weight loads (plus their x and
// scale values) in flight, and the row sums are reduced inside the CTA with
// warp shuffles and one shared-memory pass.  A warp request covers 16 or 8
// consecutive rows x 32 or 64 bytes, i.e. whole 32-byte sectors.
//
// Mode 1 reproduces the reference's row coverage: its split-K kernel
// (kernels.rs:119-131) floors chunk = in/splits and then walks only
// (chunk/8)*8 rows of each split, splits = clamp(25000/out, 1, max(in/80, 1))
// (kernels.rs:504).  Mode 0 uses every row.
#include <cuda.h>

#include <algorithm>
#include <cstdlib>

#include "common.cuh"

namespace q35 {
namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kBatch = 16;  // rows in flight per thread

struct GemvParams {
  const float *x;
  const uint4 *w;  // 16 int8 weights per uint4; a row is out_dim / 16 of them
  const float *scales;
  float *y;
  int in_dim, out_dim;
  int rows;              // active rows
  int chunk, per_split;  // active row a -> (a / per_split) * chunk + a % per_split
};

__device__ __forceinline__ float s8(uint32_t v, int j) { return (float)((int32_t)(v << (24 - 8 * j)) >> 24); }

__device__ __forceinline__ void fma16(float (&acc)[16], uint4 q, float xs) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    acc[j] = fmaf(s8(q.x, j), xs, acc[j]);
    acc[4 + j] = fmaf(s8(q.y, j), xs, acc[4 + j]);
    acc[8 + j] = fmaf(s8(q.z, j), xs, acc[8 + j]);
    acc[12 + j] = fmaf(s8(q.w, j), xs, acc[12 + j]);
  }
}

template <bool kCompat>
__device__ __forceinline__ int active_row(const GemvParams &p, int a) {
  return kCompat ? (a / p.per_split) * p.chunk + a % p.per_split : a;
}

// One CTA = a slab of 16 NQ output columns over every active row.  Lane l of
// a warp takes column quad l % NQ (16 columns, one 16-byte load per row) of
// row group l / NQ, so a warp reads 32/NQ consecutive rows x 16 NQ bytes per
// request; thread rows are rg, rg + RG, ... (RG = 256 / NQ row groups), 16 of
// them in flight with their x and scale values.  Reduction: warp shuffles over
// the row groups of a warp, then one shared-memory pass over the 8 warps.
template <bool kCompat, int NQ>
__global__ void __launch_bounds__(kGemvThreads, 2) q8_gemv_kernel(const GemvParams p) {
  pdl_entry();
  constexpr int CW = 16 * NQ;        // columns per CTA
  constexpr int LPQ = 32 / NQ;       // lanes (row groups) per column quad in a warp
  constexpr int RG = kGemvThreads / NQ;
  constexpr int VPL = 16 / LPQ;  // column sums a lane holds after the warp reduction
  static_assert(NQ == 2 || NQ == 4, "32- or 64-column slabs");
  __shared__ float red[kGemvWarps][CW];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int q = lane % NQ, rg = warp * LPQ + lane / NQ;
  const int c0 = blockIdx.x * CW;
  const int col = c0 + 16 * q;
  const size_t wpr = (size_t)p.out_dim / 16;
  const size_t spr = (size_t)p.out_dim / 64;
  const uint4 *wc = p.w + col / 16;
  const float *sc = p.scales + col / 64;

  float acc[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) acc[e] = 0.0f;
  for (int a = rg; a < p.rows; a += RG * kBatch) {
    uint4 w[kBatch];
    float xv[kBatch], sv[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int aa = a + u * RG;
      if (aa < p.rows) {
        const int row = active_row<kCompat>(p, aa);
        w[u] = __ldg(wc + (size_t)row * wpr);
        xv[u] = __ldg(p.x + row);
        sv[u] = __ldg(sc + (size_t)row * spr);
      } else {
        w[u] = make_uint4(0u, 0u, 0u, 0u);
        xv[u] = sv[u] = 0.0f;
      }
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) fma16(acc, w[u], xv[u] * sv[u]);
  }
  // reduce-scatter over the LPQ lanes of this quad (lane bits above log2(NQ)),
  // halving the held columns per step: afterwards lane group g = lane / NQ
  // holds columns VPL g .. VPL g + VPL - 1 of quad q
#pragma unroll
  for (int off = 16, n = 16; off >= NQ; off >>= 1) {
    const bool upper = (lane & off) != 0;
    n >>= 1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j < n) {
        const float send = upper ? acc[j] : acc[j + n];
        const float keep = upper ? acc[j + n] : acc[j];
        acc[j] = keep + __shfl_xor_sync(0xffffffffu, send, off);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < VPL; ++j) red[warp][16 * q + VPL * (lane / NQ) + j] = acc[j];
  __syncthreads();
  if (tid < CW && c0 + tid < p.out_dim) {
    float v = red[0][tid];
#pragma unroll
    for (int w = 1; w < kGemvWarps; ++w) v += red[w][tid];
    p.y[c0 + tid] = v;
  }
}

struct GemvPlan {
  int rows, chunk, per_split, nq;
};

GemvPlan gemv_plan(int in_dim, int out_dim, int mode, int sms) {
  GemvPlan g;
  if (mode == 1) {
    const int ref_splits = std::max(1, std::min(25000 / out_dim, std::max(in_dim / 80, 1)));  // kernels.rs:504
    g.chunk = in_dim / ref_splits;                                                            // kernels.rs:119
    g.per_split = (g.chunk / 8) * 8;                                                          // kernels.rs:130
    g.rows = ref_splits * g.per_split;
  } else {
    g.chunk = g.per_split = std::max(in_dim, 1);
    g.rows = in_dim;
  }
  // 64-column slabs when that still gives every SM a CTA, else 32 (full 32-byte sectors either way)
  g.nq = out_dim / 64 >= sms ? 4 : 2;
  return g;
}

template <bool kCompat, int NQ>
int launch_nq(const GemvParams &p, cudaStream_t st) {
  const int ctas = (p.out_dim + 16 * NQ - 1) / (16 * NQ);
  note_launch();
  (void)launch_kernel(q8_gemv_kernel<kCompat, NQ>, dim3(ctas), dim3(kGemvThreads), 0, st, 1, 1, p);
  return check_cuda(cudaGetLastError(), "q8_gemv launch");
}

// ---------------------------------------------------------------------------
// TMA path (out_dim % 256 == 0, x 16-byte aligned): a CTA owns 64 output
// columns (one scale per row) over every row.  A producer thread streams
// 128-row boxes of the weights ([128 x 64] bytes) and of the scales ([128 x 4]
// floats: the 16-byte TMA minimum, of which one column is used) from 2-D tensor
// maps over the reference layout into a 6-stage ring -- one instruction per
// box, so the stream is not capped by the SM's outstanding-load limit that
// bounds the per-thread LDG kernel above.  Eight consumer warps take 8 rows x
// 64 bytes per step (lane = row * 4 + 16-byte quarter) and reduce with warp
// shuffles and one shared-memory pass.  When the column blocks alone give few
// CTAs, the row boxes are split over a cluster of KS CTAs (grid.y) and rank 0
// adds the ranks' 64 column sums through distributed shared memory in rank
// order (deterministic).
constexpr int kTC = 64;
constexpr int kTR = 128;
constexpr int kTNS = 6;
constexpr int kTWarps = 8;
constexpr int kTThreads = (kTWarps + 1) * 32;

struct alignas(64) GemvTmaParams {
  CUtensorMap wmap;  // uint8 [in][out], box {64, 128}
  CUtensorMap smap;  // f32 [in][out / 64], box {4, 128}
  const float *x;
  float *y;
  int in_dim, out_dim;
  int chunk, per_split, ref_splits;  // mode 1 row set
  int ks;                            // row-box split = cluster size
};

struct GemvTmaSmem {
  unsigned char w[kTNS][kTR][kTC];
  float sc[kTNS][kTR][4];
  float red[kTWarps][kTC];
  float mine[kTC];  // this CTA's column sums (read by rank 0 of the cluster)
  uint64_t full[kTNS], empty[kTNS], xbar;
  alignas(16) float x[4];  // in_dim floats (dynamic tail; 16-byte aligned for the bulk copy)
};

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

template <bool kCompat>
__global__ void __launch_bounds__(kTThreads) q8_gemv_tma_kernel(const __grid_constant__ GemvTmaParams p) {
  pdl_entry();
  extern __shared__ __align__(128) unsigned char smem_raw[];
  GemvTmaSmem &sm = *reinterpret_cast<GemvTmaSmem *>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c0 = blockIdx.x * kTC;
  const int sb0 = (c0 / 64) & ~3, sj = (c0 / 64) & 3;  // scale box start (16-byte aligned) and our column in it
  const int nst_all = (p.in_dim + kTR - 1) / kTR;
  const int rk = blockIdx.y;  // row-box range of this CTA within the cluster
  const int sbeg = (int)((long long)nst_all * rk / p.ks), send = (int)((long long)nst_all * (rk + 1) / p.ks);
  const int nst = send - sbeg;
  if (tid == 0) {
    for (int i = 0; i < kTNS; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], kTWarps);
    }
    mbar_init(&sm.xbar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  bool ok = true;
  if (warp == kTWarps) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&sm.xbar, (uint32_t)p.in_dim * sizeof(float));
      bulk_g2s_nohint(sm.x, p.x, (uint32_t)p.in_dim * sizeof(float), &sm.xbar);
      for (int st = 0; st < nst && ok; ++st) {
        const int slot = st % kTNS;
        if (st >= kTNS && !mbar_wait(&sm.empty[slot], ((st / kTNS) - 1) & 1)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&sm.full[slot], kTR * kTC + kTR * 4 * sizeof(float));
        tma_load_2d(&sm.w[slot][0][0], &p.wmap, c0, (sbeg + st) * kTR, &sm.full[slot]);
        tma_load_2d(&sm.sc[slot][0][0], &p.smap, sb0, (sbeg + st) * kTR, &sm.full[slot]);
      }
    }
  } else {
    float acc[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) acc[e] = 0.0f;
    if (!mbar_wait(&sm.xbar, 0)) ok = false;
    const int q = lane & 3;
    for (int st = 0; st < nst && ok; ++st) {
      const int slot = st % kTNS;
      if (!mbar_wait(&sm.full[slot], (st / kTNS) & 1)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int step = 0; step < kTR / (8 * kTWarps); ++step) {
        const int rr = warp * (kTR / kTWarps) + step * 8 + (lane >> 2);
        const int row = (sbeg + st) * kTR + rr;
        bool live = row < p.in_dim;
        if (kCompat && live) {
          const int s = row / p.chunk;
          live = s < p.ref_splits && row - s * p.chunk < p.per_split;
        }
        if (live) {
          const uint4 w = *reinterpret_cast<const uint4 *>(&sm.w[slot][rr][16 * q]);
          fma16(acc, w, sm.x[row] * sm.sc[slot][rr][sj]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[slot]);
    }
    // reduce over the 8 rows of a step (lane bits 2-4): lane holds columns 16 q + 2 g, + 1 (g = lane / 4)
#pragma unroll
    for (int off = 16, n = 16; off >= 4; off >>= 1) {
      const bool upper = (lane & off) != 0;
      n >>= 1;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j < n) {
          const float send = upper ? acc[j] : acc[j + n];
          const float keep = upper ? acc[j + n] : acc[j];
          acc[j] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
    }
    sm.red[warp][16 * q + 2 * (lane >> 2)] = acc[0];
    sm.red[warp][16 * q + 2 * (lane >> 2) + 1] = acc[1];
  }
  __syncthreads();
  const float poison = __int_as_float(0x7fc00000);  // a bounded wait gave up
  if (tid < kTC) {
    float v = sm.red[0][tid];
#pragma unroll
    for (int w = 1; w < kTWarps; ++w) v += sm.red[w][tid];
    if (!ok) v = poison;
    if (p.ks == 1) p.y[c0 + tid] = v;
    else sm.mine[tid] = v;
  }
  if (p.ks > 1) {
    cluster_sync_all();
    if (cluster_ctarank() == 0 && tid < kTC) {
      float t = 0.0f;
      for (int r = 0; r < p.ks; ++r) t += ld_dsmem_f32(&sm.mine[tid], (uint32_t)r);
      p.y[c0 + tid] = t;
    }
    cluster_sync_all();  // no CTA leaves while rank 0 still reads its sums
  }
}

bool gemv_tma_enabled() {
  static const bool on = [] {
    const char *v = std::getenv("Q35_GEMV_TMA");
    return !(v && v[0] == '0');
  }();
  return on;
}

// Encodes the two tensor maps; false when the driver rejects them.
bool encode_gemv_maps(GemvTmaParams &p, const uint32_t *w, const float *scales, int in_dim, int out_dim) {
  const cuuint64_t wd[2] = {(cuuint64_t)out_dim, (cuuint64_t)in_dim};
  const cuuint64_t ws[1] = {(cuuint64_t)out_dim};
  const cuuint32_t wb[2] = {kTC, kTR};
  const cuuint64_t sd[2] = {(cuuint64_t)(out_dim / 64), (cuuint64_t)in_dim};
  const cuuint64_t ss[1] = {(cuuint64_t)(out_dim / 64) * sizeof(float)};
  const cuuint32_t sbx[2] = {4, kTR};
  const cuuint32_t es[2] = {1, 1};
  if (cuTensorMapEncodeTiled(&p.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint32_t *>(w), wd, ws, wb, es,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  return cuTensorMapEncodeTiled(&p.smap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(scales), sd, ss, sbx,
                                es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int launch_tma(const GemvTmaParams &p, bool compat, cudaStream_t st) {
  const size_t smem = sizeof(GemvTmaSmem) + (size_t)p.in_dim * sizeof(float);  // x tail (over-sized by 16 B)
  auto kern = compat ? q8_gemv_tma_kernel<true> : q8_gemv_tma_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "q8_gemv attributes");
  note_launch();
  (void)launch_kernel(kern, dim3(p.out_dim / kTC, p.ks), dim3(kTThreads), smem, st, 1, (unsigned)p.ks, p);
  return check_cuda(cudaGetLastError(), "q8_gemv launch");
}

}  // namespace

int q8_gemv_launch(int in_dim, int out_dim, const float *x, const uint32_t *w, const float *scales, float *y,
                   int mode, cudaStream_t st) {
  const GemvPlan g = gemv_plan(in_dim, out_dim, mode, device_sm_count());
  GemvParams p;
  p.x = x;
  p.w = reinterpret_cast<const uint4 *>(w);
  p.scales = scales;
  p.y = y;
  p.in_dim = in_dim;
  p.out_dim = out_dim;
  p.rows = g.rows;
  p.chunk = g.chunk;
  p.per_split = std::max(g.per_split, 1);
  if (gemv_tma_enabled() && out_dim % 256 == 0 && in_dim % 4 == 0 && in_dim <= 16384 &&
      (reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
    GemvTmaParams t;
    if (encode_gemv_maps(t, w, scales, in_dim, out_dim)) {
      t.x = x;
      t.y = y;
      t.in_dim = in_dim;
      t.out_dim = out_dim;
      t.chunk = std::max(g.chunk, 1);
      t.per_split = g.per_split;
      t.ref_splits = g.per_split > 0 ? g.rows / g.per_split : 0;
      // row-box split: the largest of 8 / 4 / 2 that keeps the grid within two CTAs per SM
      const int ncb = out_dim / kTC, nst = (in_dim + kTR - 1) / kTR;
      t.ks = 1;
      for (int k : {8, 4, 2})
        if (ncb * k <= 2 * device_sm_count() && k <= nst) {
          t.ks = k;
          break;
        }
      return launch_tma(t, mode == 1, st);
    }
  }
  if (mode == 1) return g.nq == 4 ? launch_nq<true, 4>(p, st) : launch_nq<true, 2>(p, st);
  return g.nq == 4 ? launch_nq<false, 4>(p, st) : launch_nq<false, 2>(p, st);
}

}  // namespace q35
