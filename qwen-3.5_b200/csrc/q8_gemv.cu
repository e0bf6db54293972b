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
#include "tma.cuh"

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

// acc[c] += int8(byte c of q) * xs for the 16 columns of one 16-byte load,
// through the conversion instruction (the LDG kernel's form: its lower
// register need keeps 16 rows of loads in flight per thread without spills).
__device__ __forceinline__ void fma16_cvt(float (&acc)[16], uint4 q, float xs) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    acc[j] = fmaf(s8(q.x, j), xs, acc[j]);
    acc[4 + j] = fmaf(s8(q.y, j), xs, acc[4 + j]);
    acc[8 + j] = fmaf(s8(q.z, j), xs, acc[8 + j]);
    acc[12 + j] = fmaf(s8(q.w, j), xs, acc[12 + j]);
  }
}

// The TMA kernel's form of fma16_cvt: each lane of a packed f32x2 FMA is one
// round-to-nearest FMA, so every column sum is bit-identical to fmaf((float)q,
// xs, acc), at one integer and one FMA-pipe instruction per weight instead of
// the quarter-rate conversion (2B decode step 1.9 % faster with 256-row boxes,
// same tokens; with 128-row boxes, two steps per ring wait, it was slower).
__device__ __forceinline__ void fma16(float (&acc)[16], uint4 q, float xs) {
  const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
  const uint64_t x2 = f2_pack(xs, xs);
#pragma unroll
  for (int k = 0; k < 4; ++k)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int e = 4 * k + 2 * h;
      f2_unpack(f2_fma(s8_pair(wd[k], h), x2, f2_pack(acc[e], acc[e + 1])), acc[e], acc[e + 1]);
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
    for (int u = 0; u < kBatch; ++u) fma16_cvt(acc, w[u], xv[u] * sv[u]);
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
// TMA path (every out_dim % 256 == 0, x 16-byte aligned): a CTA owns 64
// output columns (one scale per row) over every row.  A producer thread
// streams 256-row boxes of the weights ([256 x 64] bytes) and of the scales
// ([256 x 4] floats: the 16-byte TMA minimum, of which one column is used) from
// 2-D tensor maps over the reference layout into a shared-memory ring -- one
// instruction per box, so the stream is not capped by the SM's
// outstanding-load limit that bounds the per-thread LDG kernel above.  Eight
// consumer warps take 8 rows x 64 bytes per step (lane = row * 4 + 16-byte
// quarter), four steps per box between two ring waits (256-row boxes in a
// 3-stage ring measured 1-2 % faster on the 2B decode step than 128-row boxes
// in a 6-stage ring of the same 60 KB; deeper or shallower rings were slower),
// and reduce with warp shuffles and one shared-memory pass.  In mode 1
// the rows the reference skips get x = 0 in the CTA's shared copy of x (adding
// exact zeros leaves every f32 sum unchanged), so the inner loop has no row
// test.  When the column blocks alone give few CTAs, the row boxes are split
// over a cluster of KS CTAs (grid.y): ranks 1 .. KS-1 push their column sums
// into rank 0's shared memory with st.async (complete_tx on rank 0's
// mbarrier) and exit; rank 0 adds them in rank order (deterministic).  One
// split cluster barrier (arrive at entry, wait before the push) makes rank 0's
// mbarrier initialisation visible; no barrier holds the ranks at the end.
//
// One launch serves up to 4 projections of the same input (segments, laid out
// one after the other along grid.x), optionally with the decoder's input
// RMSNorm fused in front (h = x + residual, the input is
// h / sqrt(mean(h^2) + eps) * (1 + norm_w); text_modules.rs:800-809, residual of
// :1053-1085) and optionally with the MLP's SwiGLU behind (two segments up and
// gate streamed by the same CTA, y = up * silu(gate); :999-1011).
constexpr int kTC = 64;
constexpr int kTR = 256;
constexpr int kTWarps = 8;
constexpr int kTThreads = (kTWarps + 1) * 32;
constexpr int kMaxSeg = 4;

struct alignas(64) GemvSeg {
  CUtensorMap wmap;  // uint8 [in][out], box {64, 256}
  CUtensorMap smap;  // f32 [in][out / 64], box {4, 256}
  float *y;
  int out_dim, ncb;                  // ncb = out_dim / 64 column blocks
  int chunk, per_split, ref_splits;  // mode 1 row set of this projection
};

struct alignas(64) GemvTmaParams {
  GemvSeg seg[kMaxSeg];
  const float *x, *residual, *norm_w;
  float *sum_out, *x_out;
  uint32_t *status;  // device status word: Q35_STATUS_WAIT_TIMEOUT when a bounded wait gave up
  float eps;
  int in_dim, nseg, ks;
};

template <int NW, int NS>  // NW weight streams per CTA (2: SwiGLU), NS ring stages
struct GemvTmaSmem {
  unsigned char w[NS][NW][kTR][kTC];
  float sc[NS][NW][kTR][4];
  float red[NW][kTWarps][kTC];
  float part[kTWarps];
  static_assert(kTR % (8 * kTWarps) == 0, "whole 8-row steps per consumer warp and box");
  uint64_t full[NS], empty[NS], xbar, redbar;
  // dynamic tail: x, then residual and norm_w when the norm is fused, then (on
  // rank 0 of a cluster) the other ranks' column sums [KS - 1][NW][64]
  alignas(16) float x[4];
};


template <bool kCompat, bool kNorm, int NW, int NS>
__global__ void __launch_bounds__(kTThreads) q8_gemv_tma_kernel(const __grid_constant__ GemvTmaParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  using Smem = GemvTmaSmem<NW, NS>;
  Smem &sm = *reinterpret_cast<Smem *>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // segment and column block of this CTA (SwiGLU: segments 0 and 1 together)
  int sg = 0, cb = blockIdx.x;
  if (NW == 1)
    while (sg + 1 < p.nseg && cb >= p.seg[sg].ncb) {
      cb -= p.seg[sg].ncb;
      ++sg;
    }
  const GemvSeg *S[NW];
#pragma unroll
  for (int k = 0; k < NW; ++k) S[k] = &p.seg[sg + k];
  const int c0 = cb * kTC;
  const int sb0 = (c0 / 64) & ~3, sj = (c0 / 64) & 3;  // scale box start (16-byte aligned) and our column in it
  const int nst_all = (p.in_dim + kTR - 1) / kTR;
  const int rk = blockIdx.y;  // row-box range of this CTA within the cluster
  const int sbeg = (int)((long long)nst_all * rk / p.ks), send = (int)((long long)nst_all * (rk + 1) / p.ks);
  const int nst = send - sbeg;
  float *xs = sm.x, *rs = sm.x + p.in_dim, *ws = sm.x + 2 * p.in_dim;
  float *recv = sm.x + (kNorm ? 3 : 1) * p.in_dim;  // [KS - 1][NW][kTC]
  const bool producer = tid == kTWarps * 32;
  auto issue = [&](int st) {  // one ring stage: NW weight boxes and their scale boxes
    const int slot = st % NS;
    mbar_arrive_expect_tx(&sm.full[slot], NW * (kTR * kTC + kTR * 4 * sizeof(float)));
#pragma unroll
    for (int k = 0; k < NW; ++k) {
      tma_load_2d(&sm.w[slot][k][0][0], &S[k]->wmap, c0, (sbeg + st) * kTR, &sm.full[slot]);
      tma_load_2d(&sm.sc[slot][k][0][0], &S[k]->smap, sb0, (sbeg + st) * kTR, &sm.full[slot]);
    }
  };
  if (producer) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], kTWarps);
    }
    mbar_init(&sm.xbar, 1);
    if (p.ks > 1) {  // rank 0 expects the other ranks' sums
      mbar_init(&sm.redbar, 1);
      if (blockIdx.y == 0) mbar_arrive_expect_tx(&sm.redbar, (uint32_t)((p.ks - 1) * NW * kTC * sizeof(float)));
    }
    fence_mbar_init();
    // The weights and scales are never written by an earlier kernel: fill the
    // ring before the grid-dependency wait, so the first DRAM round trips
    // overlap the previous kernel's tail.
    for (int st = 0; st < NS && st < nst; ++st) issue(st);
  }
  __syncthreads();
  if (p.ks > 1) cluster_arrive_relaxed();  // this CTA's barriers are initialised (waited on before the push)
  pdl_entry();  // x, residual and the outputs belong to the kernel stream order from here
  bool ok = true;
  if (warp == kTWarps) {
    if (lane == 0) {
      const uint32_t xb = (uint32_t)p.in_dim * sizeof(float);
      const bool res = kNorm && p.residual != nullptr;
      mbar_arrive_expect_tx(&sm.xbar, xb * (kNorm ? (res ? 3 : 2) : 1));
      bulk_g2s_nohint(xs, p.x, xb, &sm.xbar);
      if (kNorm) {
        bulk_g2s_nohint(ws, p.norm_w, xb, &sm.xbar);
        if (res) bulk_g2s_nohint(rs, p.residual, xb, &sm.xbar);
      }
      int issued = min(NS, nst);
      for (int st = NS; st < nst && ok; ++st) {
        if (!mbar_wait(&sm.empty[st % NS], ((st / NS) - 1) & 1)) {
          ok = false;
          break;
        }
        issue(st);
        issued = st + 1;
      }
      // every box this thread requested has landed before the CTA retires
      for (int st = max(0, issued - NS); st < issued; ++st) (void)mbar_wait(&sm.full[st % NS], (st / NS) & 1);
    }
  } else {
    ok = __all_sync(0xffffffffu, mbar_wait(&sm.xbar, 0));
    const int nthr = kTWarps * 32;
    if (kNorm) {  // input RMSNorm over the whole row, by the consumer threads
      const bool res = p.residual != nullptr;
      float ss = 0.0f;
      for (int i = tid; i < p.in_dim; i += nthr) {
        float h = xs[i];
        if (res) h = h + rs[i];
        xs[i] = h;
        ss = fmaf(h, h, ss);
      }
      ss = warp_sum(ss);
      if (lane == 0) sm.part[warp] = ss;
      named_bar_sync(1, nthr);
      float tot = 0.0f;
#pragma unroll
      for (int w = 0; w < kTWarps; ++w) tot += sm.part[w];
      const float inv = 1.0f / sqrtf(tot / (float)p.in_dim + p.eps);
      const bool first = blockIdx.x == 0 && blockIdx.y == 0;
      for (int i = tid; i < p.in_dim; i += nthr) {
        const float h = xs[i];
        const float v = (h * inv) * (1.0f + ws[i]);
        if (first && p.sum_out) p.sum_out[i] = h;
        if (first && p.x_out) p.x_out[i] = v;
        xs[i] = v;
      }
    }
    if (kCompat) {  // rows outside the reference's split coverage read x = 0 (one plan per CTA)
      const int chunk = S[0]->chunk, per = S[0]->per_split, nsp = S[0]->ref_splits;
      for (int i = tid; i < p.in_dim; i += nthr) {
        const int sp = i / chunk;
        if (sp >= nsp || i - sp * chunk >= per) xs[i] = 0.0f;
      }
    }
    if (kNorm || kCompat) named_bar_sync(1, nthr);
    float acc[NW][16];
#pragma unroll
    for (int k = 0; k < NW; ++k)
#pragma unroll
      for (int e = 0; e < 16; ++e) acc[k][e] = 0.0f;
    const int q = lane & 3;
    for (int st = 0; st < nst && ok; ++st) {
      const int slot = st % NS;
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.full[slot], (st / NS) & 1))) {
        ok = false;
        break;
      }
#pragma unroll
      for (int step = 0; step < kTR / (8 * kTWarps); ++step) {
        const int rr = (step * kTWarps + warp) * 8 + (lane >> 2);  // this lane's row within the box
        const int row = (sbeg + st) * kTR + rr;
        const float xv = row < p.in_dim ? xs[row] : 0.0f;  // rows past the end are TMA zero fill
#pragma unroll
        for (int k = 0; k < NW; ++k) {
          const uint4 w = *reinterpret_cast<const uint4 *>(&sm.w[slot][k][rr][16 * q]);
          fma16(acc[k], w, xv * sm.sc[slot][k][rr][sj]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[slot]);
    }
    // reduce over the 8 rows of a step (lane bits 2-4): lane holds columns 16 q + 2 g, + 1 (g = lane / 4)
#pragma unroll
    for (int k = 0; k < NW; ++k) {
#pragma unroll
      for (int off = 16, n = 16; off >= 4; off >>= 1) {
        const bool upper = (lane & off) != 0;
        n >>= 1;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (j < n) {
            const float send = upper ? acc[k][j] : acc[k][j + n];
            const float keep = upper ? acc[k][j + n] : acc[k][j];
            acc[k][j] = keep + __shfl_xor_sync(0xffffffffu, send, off);
          }
        }
      }
      sm.red[k][warp][16 * q + 2 * (lane >> 2)] = acc[k][0];
      sm.red[k][warp][16 * q + 2 * (lane >> 2) + 1] = acc[k][1];
    }
  }
  const int failed = __syncthreads_or(ok ? 0 : 1);
  const float poison = __int_as_float(0x7fc00000);  // a bounded wait gave up
  if (failed && tid == 0 && p.status != nullptr) atomicOr(p.status, Q35_STATUS_WAIT_TIMEOUT);
  float v[NW];
  if (tid < kTC) {
#pragma unroll
    for (int k = 0; k < NW; ++k) {
      float t = sm.red[k][0][tid];
#pragma unroll
      for (int w = 1; w < kTWarps; ++w) t += sm.red[k][w][tid];
      v[k] = failed ? poison : t;
    }
  }
  if (p.ks > 1) {
    cluster_wait();  // every CTA of the cluster has initialised its barriers
    if (blockIdx.y != 0) {  // push this rank's sums to rank 0 and leave
      if (tid < kTC) {
        const uint32_t rbar = dsmem_addr(&sm.redbar, 0);
#pragma unroll
        for (int k = 0; k < NW; ++k)
          st_async_f32(dsmem_addr(&recv[((blockIdx.y - 1) * NW + k) * kTC + tid], 0), v[k], rbar);
      }
      return;
    }
    if (tid < kTC) {  // rank 0: add the ranks' sums in rank order
      const bool got = mbar_wait(&sm.redbar, 0);
      if (!got && p.status != nullptr) atomicOr(p.status, Q35_STATUS_WAIT_TIMEOUT);
#pragma unroll
      for (int k = 0; k < NW; ++k) {
        float t = v[k];
        for (int r = 1; r < p.ks; ++r) t += recv[((r - 1) * NW + k) * kTC + tid];
        v[k] = got ? t : poison;
      }
    }
  }
  if (tid < kTC) {
    if (NW == 2)
      S[0]->y[c0 + tid] = v[0] * siluf_dev(v[NW - 1]);  // up * silu(gate)
    else
      S[0]->y[c0 + tid] = v[0];
  }
}

bool gemv_tma_enabled() {
  static const bool on = [] {
    const char *v = std::getenv("Q35_GEMV_TMA");
    return !(v && v[0] == '0');
  }();
  return on;
}


// Encodes the two tensor maps of one projection; false when the driver rejects them.
bool encode_gemv_maps(GemvSeg &g, const uint32_t *w, const float *scales, int in_dim, int out_dim) {
  const EncodeTiledFn cuTensorMapEncodeTiled = encode_tiled_fn();
  if (!cuTensorMapEncodeTiled) return false;
  const cuuint64_t wd[2] = {(cuuint64_t)out_dim, (cuuint64_t)in_dim};
  const cuuint64_t wstr[1] = {(cuuint64_t)out_dim};
  const cuuint32_t wb[2] = {kTC, kTR};
  const cuuint64_t sd[2] = {(cuuint64_t)(out_dim / 64), (cuuint64_t)in_dim};
  const cuuint64_t sstr[1] = {(cuuint64_t)(out_dim / 64) * sizeof(float)};
  const cuuint32_t sbx[2] = {4, kTR};
  const cuuint32_t es[2] = {1, 1};
  if (cuTensorMapEncodeTiled(&g.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint32_t *>(w), wd, wstr, wb, es,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  return cuTensorMapEncodeTiled(&g.smap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(scales), sd, sstr,
                                sbx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool kCompat, bool kNorm, int NW, int NS>
int launch_tma_t(const GemvTmaParams &p, int ctas, cudaStream_t st) {
  const size_t smem = sizeof(GemvTmaSmem<NW, NS>) +
                      ((size_t)(kNorm ? 3 : 1) * p.in_dim + (size_t)(p.ks - 1) * NW * kTC) * sizeof(float);
  auto kern = q8_gemv_tma_kernel<kCompat, kNorm, NW, NS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "q8_gemv attributes");
  note_launch();
  (void)launch_kernel(kern, dim3(ctas, p.ks), dim3(kTThreads), smem, st, 1, (unsigned)p.ks, p);
  return check_cuda(cudaGetLastError(), "q8_gemv launch");
}

int launch_tma(GemvTmaParams &p, bool compat, bool norm, bool swiglu, cudaStream_t st) {
  p.status = device_status_word();
  int ctas = 0;
  for (int k = 0; k < p.nseg; ++k) ctas += p.seg[k].ncb;
  if (swiglu) ctas = p.seg[0].ncb;
  // row-box split KS: the largest of 8 / 4 / 2 that keeps the grid within two
  // CTAs per SM with the fused norm, one without (measured on B200 against a
  // split that evens out the CTAs per SM: the larger split with deeper rings
  // was faster on every decode shape; the plain out / down projections of the
  // 2B decode step were 1 % faster per token at KS 4 than at KS 8, same tokens)
  const int nst = (p.in_dim + kTR - 1) / kTR;
  const int per_sm = norm ? 2 : 1;
  p.ks = 1;
  for (int k : {8, 4, 2})
    if (ctas * k <= per_sm * device_sm_count() && k <= nst) {
      p.ks = k;
      break;
    }
  if (swiglu) {
    if (compat) return norm ? launch_tma_t<true, true, 2, 2>(p, ctas, st) : launch_tma_t<true, false, 2, 2>(p, ctas, st);
    return norm ? launch_tma_t<false, true, 2, 2>(p, ctas, st) : launch_tma_t<false, false, 2, 2>(p, ctas, st);
  }
  if (compat) return norm ? launch_tma_t<true, true, 1, 3>(p, ctas, st) : launch_tma_t<true, false, 1, 3>(p, ctas, st);
  return norm ? launch_tma_t<false, true, 1, 3>(p, ctas, st) : launch_tma_t<false, false, 1, 3>(p, ctas, st);
}

// Fills segment k from (w, scales, y, out_dim) with the row plan of `mode`.
bool fill_segment(GemvSeg &g, int in_dim, int out_dim, const uint32_t *w, const float *scales, float *y, int mode) {
  if (!encode_gemv_maps(g, w, scales, in_dim, out_dim)) return false;
  const GemvPlan pl = gemv_plan(in_dim, out_dim, mode, 148);
  g.y = y;
  g.out_dim = out_dim;
  g.ncb = out_dim / kTC;
  g.chunk = std::max(pl.chunk, 1);
  g.per_split = pl.per_split;
  g.ref_splits = pl.per_split > 0 ? pl.rows / pl.per_split : 0;
  return true;
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
    GemvTmaParams t = {};
    if (fill_segment(t.seg[0], in_dim, out_dim, w, scales, y, mode)) {
      t.x = x;
      t.in_dim = in_dim;
      t.nseg = 1;
      return launch_tma(t, mode == 1, false, false, st);
    }
  }
  if (mode == 1) return g.nq == 4 ? launch_nq<true, 4>(p, st) : launch_nq<true, 2>(p, st);
  return g.nq == 4 ? launch_nq<false, 4>(p, st) : launch_nq<false, 2>(p, st);
}

}  // namespace q35

namespace q35 {

int q8_gemv_fused_launch(int in_dim, int n_seg, const q35_q8_segment *segs, const float *x, const float *residual,
                         const float *norm_w, float eps, float *sum_out, float *x_out, int swiglu, int mode,
                         cudaStream_t st) {
  // shapes and pointers are validated at the C-ABI boundary
  GemvTmaParams t = {};
  for (int k = 0; k < n_seg; ++k) {
    Q35_REQUIRE(fill_segment(t.seg[k], in_dim, segs[k].out_dim, segs[k].w, segs[k].scales, segs[k].y, mode),
                Q35_ERR_INVALID_ARG, "q8_gemv_fused: tensor map rejected (alignment of w / scales)");
  }
  t.x = x;
  t.residual = residual;
  t.norm_w = norm_w;
  t.sum_out = sum_out;
  t.x_out = x_out;
  t.eps = eps;
  t.in_dim = in_dim;
  t.nseg = n_seg;
  return launch_tma(t, mode == 1, norm_w != nullptr, swiglu != 0, st);
}

}  // namespace q35
