// gdn_decode.cu -- fused Gated DeltaNet decode step for sm_100a.
//
// One kernel replaces the decode branch of GatedDeltaNet::forward between the
// input and output projections (inventwithdean/Qwen-3.5
// src/text_modules.rs:515-530 causal_conv1d_update + SiLU, :554-567 q/k/v
// split, :597-615 k-head expansion, :365-443 burn_recurrent_gated_delta_rule,
// :651-660 RMSNormGated).
//
// Work decomposition.  The delta-rule update is independent per value column
// v of the [DK x DV] state: kv_mem[v], delta[v], the rank-1 update of column v
// and o[v] touch column v only.  A thread-block cluster therefore owns one key
// head (all rf = Hv/Hk value heads that share it) and each CTA of the cluster
// owns DV/SPLIT columns of one value head.  Inside a CTA every thread holds
// NP float4 of the state in registers: the state is read from HBM once and
// written back once, 128-bit coalesced, with streaming cache hints.
// Reductions over the key dimension use warp shuffles plus one small shared
// memory pass.  The cluster shares the conv outputs of the q/k channels
// (computed once, spread over the CTAs) and the per-column sums of squares of
// the gated RMS norm through distributed shared memory.
//
// Race freedom of the in-place conv state: every conv channel is read and
// rewritten by exactly one thread of one CTA (q/k channels of key head hk are
// owned by cluster hk; v channels by the CTA owning those columns).
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace q35 {
namespace {

constexpr int kDK = 128;
constexpr int kDV = 128;

struct GdnDecodeParams {
  const float *mixed_qkv, *z, *beta, *g, *conv_w, *norm_w;
  float *conv_state, *rec_state, *out;
  uint32_t *status;  // device status word (streaming kernel): Q35_STATUS_WAIT_TIMEOUT
  int B, Hk, Hv, rf, C;
  float eps;
};

// bar.sync over `nthreads` that also returns whether every participating
// thread passed pred != 0.
__device__ __forceinline__ bool named_bar_and(uint32_t id, uint32_t nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

template <int SPLIT>
struct GdnDecodeCfg {
  static constexpr int CS = kDV / SPLIT;           // state columns per CTA
  static constexpr int QR = CS / 4;                // float4 quads per row
  static constexpr int NT = SPLIT <= 2 ? 256 : 128;
  static constexpr int RP = NT / QR;               // rows covered per pass
  static constexpr int NP = kDK / RP;              // float4 of state per thread
  static constexpr int NW = NT / 32;
  static_assert(QR >= 1 && QR <= 32 && 32 % QR == 0, "quad layout");
  static_assert(NP * RP == kDK, "row layout");
};

template <int KC>
__device__ __forceinline__ float conv_channel(const GdnDecodeParams &p, size_t xrow, int c) {
  // text_modules.rs:145-161: window = [state..., x]; y = sum_j w[c,j]*win[j];
  // new state = window[1..]; output silu(y).
  const float *w = p.conv_w + (size_t)c * KC;
  float *st = p.conv_state + (xrow + c) * (KC - 1);
  float win[KC];
#pragma unroll
  for (int j = 0; j < KC - 1; ++j) win[j] = st[j];
  win[KC - 1] = p.mixed_qkv[xrow + c];
  float acc = 0.0f;
#pragma unroll
  for (int j = 0; j < KC; ++j) acc = fmaf(w[j], win[j], acc);
#pragma unroll
  for (int j = 0; j < KC - 1; ++j) st[j] = win[j + 1];
  return siluf_dev(acc);
}

// SOLO: one CTA per key head (SPLIT == 1 and rf == 1), launched without a
// cluster, so no cluster barrier (whose release semantics would wait for the
// in-flight state loads) is needed.
template <int SPLIT, int KC, bool SOLO>
__global__ void __launch_bounds__(GdnDecodeCfg<SPLIT>::NT)
    gdn_decode_kernel(const GdnDecodeParams p) {
  pdl_entry();
  using Cfg = GdnDecodeCfg<SPLIT>;
  constexpr int CS = Cfg::CS, QR = Cfg::QR, NT = Cfg::NT, RP = Cfg::RP, NP = Cfg::NP, NW = Cfg::NW;
  static_assert(!SOLO || SPLIT == 1, "SOLO implies one CTA per head");

  const int ncl = SOLO ? 1 : p.rf * SPLIT;  // CTAs per cluster == gridDim.x
  const int crank = blockIdx.x;
  const int hk = blockIdx.y, b = blockIdx.z;
  const int r = crank / SPLIT, s = crank % SPLIT;
  const int h = hk * p.rf + r;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cq = tid % QR, r0 = tid / QR;
  const int col0 = s * CS;

  __shared__ float qk_loc[2 * kDK];  // q/k conv outputs owned by this CTA
  __shared__ float qk_all[2 * kDK];  // full q (0..DK) and k (DK..2DK) of head hk
  __shared__ float v_loc[CS];
  __shared__ __align__(16) float red[NW][CS];
  __shared__ __align__(16) float delta_s[CS];
  __shared__ float o_s[CS];
  __shared__ float sq_parts[SPLIT];
  __shared__ float inv_norm[2];

  // (1) Issue every state load first; they stay in flight during the conv.
  float *Sp = p.rec_state + ((size_t)b * p.Hv + h) * kDK * kDV + col0 + cq * 4;
  float4 S[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i)
    S[i] = __ldcs(reinterpret_cast<const float4 *>(Sp + (size_t)(r0 + i * RP) * kDV));
  // The per-head gate inputs and the gated-norm operands are requested now as
  // well, so that no global-memory round trip is left behind the barriers.
  const float g_h = p.g[(size_t)b * p.Hv + h];
  const float bt = p.beta[(size_t)b * p.Hv + h];
  const size_t oidx = ((size_t)b * p.Hv + h) * kDV + col0 + tid;
  float z_c = 0.0f, nw_c = 0.0f;
  if (tid < CS) {
    z_c = p.z[oidx];
    nw_c = p.norm_w[col0 + tid];
  }

  // (2) Causal conv update + SiLU.  q/k channels of key head hk are spread
  // over the cluster (channel i owned by rank i % ncl); v channels of the
  // CTA's own columns.
  const size_t xrow = (size_t)b * p.C;
  for (int i = crank + tid * ncl; i < 2 * kDK; i += NT * ncl) {
    const int c = i < kDK ? hk * kDK + i : p.Hk * kDK + hk * kDK + (i - kDK);
    (SOLO ? qk_all : qk_loc)[i] = conv_channel<KC>(p, xrow, c);
  }
  if (tid < CS) v_loc[tid] = conv_channel<KC>(p, xrow, 2 * p.Hk * kDK + h * kDV + col0 + tid);

  if constexpr (SOLO) {
    __syncthreads();
  } else {
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();  // q/k pieces of every rank are in shared memory
    for (int i = tid; i < 2 * kDK; i += NT) {
      const float *src = cluster.map_shared_rank(&qk_loc[i], i % ncl);
      qk_all[i] = *src;
    }
    __syncthreads();
  }

  // (3) l2norm of q and k (text_modules.rs:184-187, :389-390), eps 1e-6.
  if (warp < 2) {
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < kDK / 32; ++j) {
      const float v = qk_all[warp * kDK + lane + 32 * j];
      ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    if (lane == 0) inv_norm[warp] = 1.0f / sqrtf(ss + 1e-6f);
  }
  __syncthreads();

  const float qscale = rsqrtf((float)kDK);  // 128^-0.5 is exact in f32
  const float inv_q = inv_norm[0], inv_k = inv_norm[1];
  float kr[NP], qr[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int row = r0 + i * RP;
    kr[i] = qk_all[kDK + row] * inv_k;
    qr[i] = (qk_all[row] * inv_q) * qscale;
  }

  // (4) Delta rule (text_modules.rs:412-430).
  const float decay = expf(g_h);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    S[i].x *= decay; S[i].y *= decay; S[i].z *= decay; S[i].w *= decay;
    acc = f4_fma(kr[i], S[i], acc);
  }
#pragma unroll
  for (int off = QR; off < 32; off <<= 1) {
    acc.x += __shfl_xor_sync(0xffffffffu, acc.x, off);
    acc.y += __shfl_xor_sync(0xffffffffu, acc.y, off);
    acc.z += __shfl_xor_sync(0xffffffffu, acc.z, off);
    acc.w += __shfl_xor_sync(0xffffffffu, acc.w, off);
  }
  if (lane < QR) *reinterpret_cast<float4 *>(&red[warp][cq * 4]) = acc;
  __syncthreads();
  if (tid < CS) {
    float kv = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; ++w) kv += red[w][tid];
    delta_s[tid] = (v_loc[tid] - kv) * bt;
  }
  __syncthreads();

  const float4 dl = *reinterpret_cast<const float4 *>(&delta_s[cq * 4]);
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    S[i] = f4_fma(kr[i], dl, S[i]);
    o = f4_fma(qr[i], S[i], o);
    __stcs(reinterpret_cast<float4 *>(Sp + (size_t)(r0 + i * RP) * kDV), S[i]);
  }
#pragma unroll
  for (int off = QR; off < 32; off <<= 1) {
    o.x += __shfl_xor_sync(0xffffffffu, o.x, off);
    o.y += __shfl_xor_sync(0xffffffffu, o.y, off);
    o.z += __shfl_xor_sync(0xffffffffu, o.z, off);
    o.w += __shfl_xor_sync(0xffffffffu, o.w, off);
  }
  if (lane < QR) *reinterpret_cast<float4 *>(&red[warp][cq * 4]) = o;
  __syncthreads();
  if (tid < CS) {
    float ov = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; ++w) ov += red[w][tid];
    o_s[tid] = ov;
  }
  __syncthreads();

  // (5) RMSNormGated over the DV outputs of head h (text_modules.rs:93-101):
  // the SPLIT CTAs of head h exchange their partial sums of squares.
  if (warp == 0) {
    float ss = 0.0f;
    for (int c = lane; c < CS; c += 32) ss = fmaf(o_s[c], o_s[c], ss);
    ss = warp_sum(ss);
    if constexpr (SOLO) {
      if (lane == 0) sq_parts[0] = ss;
    } else {
      if (lane < SPLIT) *cg::this_cluster().map_shared_rank(&sq_parts[s], r * SPLIT + lane) = ss;
    }
  }
  if constexpr (SOLO) {
    __syncthreads();
  } else {
    cg::this_cluster().sync();
  }
  if (tid < CS) {
    float tot = 0.0f;
#pragma unroll
    for (int j = 0; j < SPLIT; ++j) tot += sq_parts[j];
    const float inv = 1.0f / sqrtf(tot / (float)kDV + p.eps);
    p.out[oidx] = (nw_c * (o_s[tid] * inv)) * siluf_dev(z_c);
  }
}

// ---------------------------------------------------------------------------
// Streaming variant for large batches: persistent CTAs (one per SM) walk a
// static list of (sequence, key head) items; each item has rf value-head
// tiles.  A producer thread moves every 64 KB state tile (contiguous in HBM)
// plus the tile's conv inputs and gate into a 3-stage shared-memory ring with
// bulk TMA copies (mbarrier complete_tx); 8 consumer warps run the delta rule
// out of shared memory, write the updated tile back in place, and one thread
// returns it to HBM with a bulk TMA store while the next tiles are already in
// flight.  The q/k conv and l2norm of a key head are computed on its first
// tile (r == 0) and reused by the other rf - 1 tiles of the item.
constexpr int kStages = 3;
constexpr int kCons = 256;                 // consumer threads (8 warps)
constexpr int kStreamThreads = kCons + 32; // + producer warp

template <int KC>
struct StreamStage {
  float S[kDK * kDV];
  float xqk[2 * kDK];
  float cqk[2 * kDK * (KC - 1)];
  float xv[kDV];
  float cv[kDV * (KC - 1)];
  float z[kDV];
};

template <int KC>
__global__ void __launch_bounds__(kStreamThreads, 1) gdn_decode_stream_kernel(const GdnDecodeParams p) {
  pdl_entry();
  extern __shared__ __align__(128) unsigned char smem_raw[];
  StreamStage<KC> *stg = reinterpret_cast<StreamStage<KC> *>(smem_raw);
  __shared__ __align__(8) uint64_t full_bar[kStages], empty_bar[kStages];
  __shared__ __align__(16) float qkn[2 * kDK];   // normalised q (scaled) | k of the current key head
  __shared__ __align__(16) float red[8][kDV];
  __shared__ __align__(16) float delta_s[kDV];
  __shared__ float v_loc[kDV];
  __shared__ float sq[4];
  __shared__ float inv_norm[2];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int items = p.B * p.Hk;
  const int n_my_items = items > (int)blockIdx.x ? (items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int ntiles = n_my_items * p.rf;
  constexpr uint32_t kStBytes = (KC - 1) * kDK * sizeof(float);

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kCons / 32) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int issued = 0;
      for (int t = 0; t < ntiles; ++t) {
        const int sidx = t % kStages;
        if (t >= kStages && !mbar_wait(&empty_bar[sidx], ((t / kStages) - 1) & 1)) {
          atomicOr(p.status, Q35_STATUS_WAIT_TIMEOUT);
          break;
        }
        issued = t + 1;
        const int item = blockIdx.x + (t / p.rf) * gridDim.x;
        const int r = t % p.rf;
        const int b = item / p.Hk, hk = item % p.Hk, h = hk * p.rf + r;
        StreamStage<KC> &sg = stg[sidx];
        const size_t xrow = (size_t)b * p.C;
        const int cq0 = hk * kDK, ck0 = p.Hk * kDK + hk * kDK, cv0 = 2 * p.Hk * kDK + h * kDV;
        uint32_t bytes = sizeof(sg.S) + 2 * kDV * sizeof(float) + kStBytes;
        if (r == 0) bytes += 2 * kDK * sizeof(float) + 2 * kStBytes;
        mbar_arrive_expect_tx(&full_bar[sidx], bytes);
        bulk_g2s(sg.S, p.rec_state + ((size_t)b * p.Hv + h) * kDK * kDV, sizeof(sg.S), &full_bar[sidx], pol);
        if (r == 0) {
          bulk_g2s(sg.xqk, p.mixed_qkv + xrow + cq0, kDK * sizeof(float), &full_bar[sidx], pol);
          bulk_g2s(sg.xqk + kDK, p.mixed_qkv + xrow + ck0, kDK * sizeof(float), &full_bar[sidx], pol);
          bulk_g2s(sg.cqk, p.conv_state + (xrow + cq0) * (KC - 1), kStBytes, &full_bar[sidx], pol);
          bulk_g2s(sg.cqk + kDK * (KC - 1), p.conv_state + (xrow + ck0) * (KC - 1), kStBytes, &full_bar[sidx], pol);
        }
        bulk_g2s(sg.xv, p.mixed_qkv + xrow + cv0, kDV * sizeof(float), &full_bar[sidx], pol);
        bulk_g2s(sg.cv, p.conv_state + (xrow + cv0) * (KC - 1), kStBytes, &full_bar[sidx], pol);
        bulk_g2s(sg.z, p.z + ((size_t)b * p.Hv + h) * kDV, kDV * sizeof(float), &full_bar[sidx], pol);
      }
      // every copy this thread started has landed before the CTA retires
      for (int t = max(0, issued - kStages); t < issued; ++t)
        (void)mbar_wait(&full_bar[t % kStages], (t / kStages) & 1);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const float qscale = rsqrtf((float)kDK);
  for (int t = 0; t < ntiles; ++t) {
    const int sidx = t % kStages;
    const int item = blockIdx.x + (t / p.rf) * gridDim.x;
    const int r = t % p.rf;
    const int b = item / p.Hk, hk = item % p.Hk, h = hk * p.rf + r;
    const size_t xrow = (size_t)b * p.C;
    const float decay = expf(__ldg(p.g + (size_t)b * p.Hv + h));
    const float bt = __ldg(p.beta + (size_t)b * p.Hv + h);
    StreamStage<KC> &sg = stg[sidx];
    const bool got = mbar_wait(&full_bar[sidx], (t / kStages) & 1);

    // causal conv update + SiLU (text_modules.rs:145-161) from the staged inputs
    auto conv = [&](const float *win_state, float xin, int c, float &y) {
      const float *w = p.conv_w + (size_t)c * KC;
      float win[KC];
#pragma unroll
      for (int j = 0; j < KC - 1; ++j) win[j] = win_state[j];
      win[KC - 1] = xin;
      float acc = 0.0f;
#pragma unroll
      for (int j = 0; j < KC; ++j) acc = fmaf(__ldg(w + j), win[j], acc);
      float *dst = p.conv_state + (xrow + c) * (KC - 1);
#pragma unroll
      for (int j = 0; j < KC - 1; ++j) dst[j] = win[j + 1];
      y = siluf_dev(acc);
    };
    if (r == 0) {
      const int i = tid;  // 256 q|k channels
      const int c = i < kDK ? hk * kDK + i : p.Hk * kDK + hk * kDK + (i - kDK);
      float y;
      conv(sg.cqk + i * (KC - 1), sg.xqk[i], c, y);
      qkn[i] = y;
    }
    if (tid < kDV) {
      float y;
      conv(sg.cv + tid * (KC - 1), sg.xv[tid], 2 * p.Hk * kDK + h * kDV + tid, y);
      v_loc[tid] = y;
    }
    // every consumer thread saw the tile land, or all stop together (a wait
    // gave up: the status word says so, the state of this tile is not valid)
    if (!named_bar_and(1, kCons, got)) {
      if (tid == 0) atomicOr(p.status, Q35_STATUS_WAIT_TIMEOUT);
      break;
    }
    if (r == 0) {
      if (warp < 2) {  // l2norm of q and k (text_modules.rs:184-187)
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < kDK / 32; ++j) {
          const float v = qkn[warp * kDK + lane + 32 * j];
          ss = fmaf(v, v, ss);
        }
        ss = warp_sum(ss);
        if (lane == 0) inv_norm[warp] = 1.0f / sqrtf(ss + 1e-6f);
      }
      named_bar_sync(1, kCons);
      const float v = qkn[tid];
      qkn[tid] = tid < kDK ? (v * inv_norm[0]) * qscale : v * inv_norm[1];
      named_bar_sync(1, kCons);
    }

    // delta rule (text_modules.rs:412-430): lane owns 4 columns, warp owns rows warp + 8i
    float4 Sv[16];
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int row = warp + 8 * i;
      Sv[i] = *reinterpret_cast<const float4 *>(&sg.S[row * kDV + 4 * lane]);
      Sv[i].x *= decay; Sv[i].y *= decay; Sv[i].z *= decay; Sv[i].w *= decay;
      acc = f4_fma(qkn[kDK + row], Sv[i], acc);
    }
    *reinterpret_cast<float4 *>(&red[warp][4 * lane]) = acc;
    named_bar_sync(1, kCons);
    if (tid < kDV) {
      float kv = 0.0f;
#pragma unroll
      for (int w = 0; w < 8; ++w) kv += red[w][tid];
      delta_s[tid] = (v_loc[tid] - kv) * bt;
    }
    named_bar_sync(1, kCons);
    const float4 dl = *reinterpret_cast<const float4 *>(&delta_s[4 * lane]);
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int row = warp + 8 * i;
      Sv[i] = f4_fma(qkn[kDK + row], dl, Sv[i]);
      o = f4_fma(qkn[row], Sv[i], o);
      *reinterpret_cast<float4 *>(&sg.S[row * kDV + 4 * lane]) = Sv[i];
    }
    *reinterpret_cast<float4 *>(&red[warp][4 * lane]) = o;
    fence_proxy_async_smem();
    named_bar_sync(1, kCons);
    if (tid == 0) {
      bulk_s2g(p.rec_state + ((size_t)b * p.Hv + h) * kDK * kDV, sg.S, sizeof(sg.S));
      bulk_commit();
      if (t > 0) {
        bulk_wait_read<1>();  // the previous tile's store has left shared memory
        mbar_arrive(&empty_bar[(t - 1) % kStages]);
      }
    }
    // RMSNormGated over the 128 outputs of head h (text_modules.rs:93-101)
    float ov = 0.0f;
    if (tid < kDV) {
#pragma unroll
      for (int w = 0; w < 8; ++w) ov += red[w][tid];
      const float ss = warp_sum(ov * ov);
      if (lane == 0) sq[warp] = ss;
    }
    named_bar_sync(1, kCons);
    if (tid < kDV) {
      const float inv = 1.0f / sqrtf((sq[0] + sq[1] + sq[2] + sq[3]) / (float)kDV + p.eps);
      p.out[((size_t)b * p.Hv + h) * kDV + tid] = (p.norm_w[tid] * (ov * inv)) * siluf_dev(sg.z[tid]);
    }
  }
  if (tid == 0) bulk_wait_read<0>();
}

template <int KC>
cudaError_t launch_stream(const GdnDecodeParams &p, int sms, cudaStream_t st) {
  const size_t smem = kStages * sizeof(StreamStage<KC>);
  cudaError_t e = cudaFuncSetAttribute(gdn_decode_stream_kernel<KC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  const int items = p.B * p.Hk;
  const int grid = items < sms ? items : sms;
  note_launch();
  (void)launch_kernel(gdn_decode_stream_kernel<KC>, dim3(grid), dim3(kStreamThreads), smem, st, 1, 1, p);
  return cudaGetLastError();
}

template <int SPLIT, int KC>
cudaError_t launch(const GdnDecodeParams &p, int ncl, cudaStream_t st) {
  if constexpr (SPLIT == 1) {
    if (ncl == 1) {
      note_launch();
      (void)launch_kernel(gdn_decode_kernel<1, KC, true>, dim3(1, p.Hk, p.B), dim3(GdnDecodeCfg<1>::NT), 0, st, 1, 1, p);
      return cudaGetLastError();
    }
  }
  note_launch();
  return launch_kernel(gdn_decode_kernel<SPLIT, KC, false>, dim3(ncl, p.Hk, p.B), dim3(GdnDecodeCfg<SPLIT>::NT), 0,
                       st, (unsigned)ncl, 1, p);
}

template <int KC>
cudaError_t launch_split(const GdnDecodeParams &p, int split, cudaStream_t st) {
  const int ncl = split * p.rf;
  switch (split) {
    case 1: return launch<1, KC>(p, ncl, st);
    case 2: return launch<2, KC>(p, ncl, st);
    case 4: return launch<4, KC>(p, ncl, st);
    default: return launch<8, KC>(p, ncl, st);
  }
}

}  // namespace

// Column split per head below the streaming threshold: none.  Measured on
// B200 with the state L2-resident (256 dependent steps in a CUDA graph), one
// CTA per head beat every cluster split (B=1: 4.52 us against 4.76-5.04 us for
// splits 2-8; B=4: 4.57 against 5.0-6.6; B=16: 7.9 against 13-17): the two
// cluster barriers of a split cost more than the wider state stream saves.
// A split (q35_gdn_decode_split) stays available to callers.
int gdn_decode_split(int B, int Hv, int rf, int sms) {
  (void)B, (void)Hv, (void)rf, (void)sms;
  return 1;
}

int gdn_decode_launch(const q35_gdn_dims *d, const float *mixed_qkv, const float *z, const float *beta,
                      const float *g, const float *conv_w, const float *norm_w, float *conv_state,
                      float *rec_state, float *out, cudaStream_t st, int force_split) {
  GdnDecodeParams p;
  p.mixed_qkv = mixed_qkv; p.z = z; p.beta = beta; p.g = g; p.conv_w = conv_w; p.norm_w = norm_w;
  p.conv_state = conv_state; p.rec_state = rec_state; p.out = out;
  p.B = d->batch; p.Hk = d->num_k_heads; p.Hv = d->num_v_heads; p.rf = p.Hv / p.Hk;
  p.C = 2 * p.Hk * kDK + p.Hv * kDV;
  p.eps = d->eps;
  p.status = device_status_word();
  const int sms = device_sm_count();
  // Large batches stream persistent tiles through shared memory; small ones
  // split each head's columns over a cluster to occupy every SM.
  const bool stream = force_split < 0 || (force_split == 0 && (long long)p.B * p.Hv >= 4LL * sms);
  if (stream) {
    Q35_REQUIRE((reinterpret_cast<uintptr_t>(mixed_qkv) & 15u) == 0 && (reinterpret_cast<uintptr_t>(z) & 15u) == 0 &&
                    (reinterpret_cast<uintptr_t>(conv_state) & 15u) == 0,
                Q35_ERR_INVALID_ARG, "gdn_decode: mixed_qkv, z and conv_state must be 16-byte aligned");
    cudaError_t e;
    switch (d->conv_kernel) {
      case 2: e = launch_stream<2>(p, sms, st); break;
      case 3: e = launch_stream<3>(p, sms, st); break;
      default: e = launch_stream<4>(p, sms, st); break;
    }
    return check_cuda(e, "gdn_decode (stream) launch");
  }
  const int split = force_split > 0 ? force_split : gdn_decode_split(p.B, p.Hv, p.rf, sms);
  Q35_REQUIRE(split * p.rf <= 8, Q35_ERR_UNSUPPORTED, "gdn_decode: num_v_heads/num_k_heads * split must be <= 8");
  cudaError_t e;
  switch (d->conv_kernel) {
    case 2: e = launch_split<2>(p, split, st); break;
    case 3: e = launch_split<3>(p, split, st); break;
    default: e = launch_split<4>(p, split, st); break;
  }
  return check_cuda(e, "gdn_decode launch");
}

}  // namespace q35
