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
#include <algorithm>

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
  if (mode == 1) return g.nq == 4 ? launch_nq<true, 4>(p, st) : launch_nq<true, 2>(p, st);
  return g.nq == 4 ? launch_nq<false, 4>(p, st) : launch_nq<false, 2>(p, st);
}

}  // namespace q35
