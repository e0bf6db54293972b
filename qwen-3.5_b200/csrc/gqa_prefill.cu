// gqa_prefill.cu -- gated GQA attention over a prompt (prefill) on the sm_100a
// tensor cores.
//
// Replaces Attention::forward between the projections for seq_len = T
// (inventwithdean/Qwen-3.5 src/text_modules.rs:866-936): q/gate split, q_norm /
// k_norm (RMSNorm 1+w, :800-809), partial RoPE (:754-774), the KV-cache append
// (:899-909, in place at lens[b]), repeat_kv (:776-792, as head grouping), the
// causal scaled-dot-product attention (mask model.rs:59-67: query t of the
// prompt sees keys 0 .. lens[b] + t) and the sigmoid output gate.
//
// Four launches (five when a key range is split):
//  (1) qkv: per token, warp per head.  q: norm + RoPE + scale (log2 e / 16),
//      stored as blocked hi/lo tiles for the tensor cores.  k: norm + RoPE and
//      v, appended to the cache at lens[b] + t.
//  (2) kv tiles: the cache rows 0 .. lens[b] + T - 1 of every kv head as
//      blocked hi/lo tiles, K as [64 keys x 32 dims] chunks and V transposed
//      as [128 dims x 64 keys] halves (zero past the last key).
//  (3) attention: CTA = (128-query tile, q head, range of 4 key tiles: the
//      key range of a query tile is split so the causal triangle spreads over
//      the SMs).  A producer warp streams the
//      Q / K chunks and V halves into a 2 x 64 KB shared-memory ring with bulk
//      copies; an MMA warp issues S = Q K^T (M 128, N 64, K 256 in 32-dim
//      stages) and O += P V (two N 128 halves, K 64) as 3xTF32 tcgen05 MMAs
//      into TMEM (S: 64 columns, O: 256); four softmax warps own one TMEM lane
//      (query row) per thread: online softmax in the exp2 domain, causal mask,
//      P as blocked hi/lo into shared memory, and O rescaled in TMEM only when
//      the row max grows by more than 2^8 (the final O / l does not depend on
//      the reference max).  QK of the next key tile is issued before PV of the
//      current one, so the softmax overlaps the tensor pipe.  Epilogue:
//      O / l * sigmoid(gate), or, for a split key range, the unnormalised O and
//      (m, l), which (3b) merges before the gate.
//  (4) lens[b] += T.
#include "common.cuh"
#include "gqa_common.cuh"
#include "umma.cuh"

namespace q35 {
namespace {

using gqa::norm_rope;
using umma::blk_off;
constexpr int kD = gqa::kHeadDim;    // 256
constexpr int kBM = 128;             // query rows per CTA = TMEM lanes
constexpr int kBN = 64;              // keys per tile
constexpr int kDC = 32;              // head dims per QK stage
constexpr int kNQC = kD / kDC;       // 8 QK stages per key tile
constexpr int kQC = kBM * kDC;       // floats of a blocked [128 x 32] Q chunk
constexpr int kKC = kBN * kDC;       // [64 x 32] K chunk
constexpr int kVH = (kD / 2) * kBN;  // [128 dims x 64 keys] V^T half
constexpr int kSlot = 2 * kVH;       // ring slot: a V^T half, hi + lo (64 KB)
constexpr int kAttnThreads = 192;    // warps 0-3 softmax, 4 producer, 5 MMA
constexpr int kKvThreads = 256;
constexpr int kKvLd = kD + 4;        // padded row of the kv staging tiles
constexpr int kKS = 4;               // key tiles per attention CTA (load balance of the causal triangle)

struct PrefillParams {
  const float *q_gate, *k_new, *v_new, *qn_w, *kn_w, *cos, *sin;
  float *k_cache, *v_cache;
  int32_t *lens;
  float *out;
  float *qb, *kb, *vb;  // blocked scratch
  float *po, *pml;      // key-split partials: O [B][ntq][ns][Hq][128][256], (m, l) [..][128][2]
  uint32_t *status;
  long long cap, max_len;  // max_len: host bound on lens[b] + T (sizes the key scratch)
  int B, T, Hq, Hkv, rot, ntq, nkt, ns;  // ns: key splits per query tile (grid.z = B * ns)
  float eps, qscale;  // log2(e) / sqrt(D)
};

// Sequences whose cache cannot take the prompt, or whose length exceeds the
// host's bound, are skipped and reported through the status word.
__device__ __forceinline__ bool skip_seq(const PrefillParams &p, long long past) {
  return past + p.T > p.cap || past + p.T > p.max_len;
}

__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ void st4(float *p, float4 v) { *reinterpret_cast<float4 *>(p) = v; }
__device__ __forceinline__ float4 lo4(float4 v) {
  return make_float4(umma::tf32_lo(v.x), umma::tf32_lo(v.y), umma::tf32_lo(v.z), umma::tf32_lo(v.w));
}

// ---------------------------------------------------------------- (1) qkv
__global__ void __launch_bounds__(1024) gqa_prefill_qkv_kernel(const PrefillParams p) {
  pdl_entry();
  extern __shared__ __align__(16) float tmp_s[];  // [warps][256]
  const int t = blockIdx.x, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long past = p.lens[b];
  if (skip_seq(p, past)) {
    if (threadIdx.x == 0 && t == 0)
      atomicOr(p.status, past + p.T > p.cap ? Q35_STATUS_CACHE_FULL : Q35_STATUS_LEN_HINT);
    return;
  }
  const size_t tok = (size_t)b * p.T + t;
  const float *cs = p.cos + tok * p.rot, *sn = p.sin + tok * p.rot;
  float *tmp = tmp_s + warp * kD;
  if (warp < p.Hq) {
    const int h = warp;
    const float *qin = p.q_gate + (tok * p.Hq + h) * 2 * kD;
    float4 x0 = ld4(qin + 4 * lane), x1 = ld4(qin + 128 + 4 * lane);
    norm_rope(x0, x1, p.qn_w, cs, sn, p.rot, p.eps, tmp, lane);
    const float s = p.qscale;
    x0 = make_float4(x0.x * s, x0.y * s, x0.z * s, x0.w * s);
    x1 = make_float4(x1.x * s, x1.y * s, x1.z * s, x1.w * s);
    const int qt = t / kBM, r = t % kBM;
    float *base = p.qb + (((size_t)b * p.Hq + h) * p.ntq + qt) * kNQC * 2 * kQC;
    // dims 4 lane .. 4 lane + 3 are columns 4 (lane % 8) .. of chunk lane / 8 (x1: chunk 4 + lane / 8)
    const int off = blk_off(r, 4 * (lane & 7), kDC);
    const int c0 = lane >> 3, c1 = 4 + (lane >> 3);
    st4(base + (2 * c0) * kQC + off, x0);
    st4(base + (2 * c0 + 1) * kQC + off, lo4(x0));
    st4(base + (2 * c1) * kQC + off, x1);
    st4(base + (2 * c1 + 1) * kQC + off, lo4(x1));
  } else if (warp < p.Hq + p.Hkv) {
    const int kh = warp - p.Hq;
    const float *kin = p.k_new + (tok * p.Hkv + kh) * kD;
    const float *vin = p.v_new + (tok * p.Hkv + kh) * kD;
    float4 x0 = ld4(kin + 4 * lane), x1 = ld4(kin + 128 + 4 * lane);
    norm_rope(x0, x1, p.kn_w, cs, sn, p.rot, p.eps, tmp, lane);
    const size_t row = (((size_t)b * p.Hkv + kh) * p.cap + past + t) * kD;
    st4(p.k_cache + row + 4 * lane, x0);
    st4(p.k_cache + row + 128 + 4 * lane, x1);
    st4(p.v_cache + row + 4 * lane, ld4(vin + 4 * lane));
    st4(p.v_cache + row + 128 + 4 * lane, ld4(vin + 128 + 4 * lane));
  }
}

// ---------------------------------------------------------------- (2) kv tiles
__global__ void __launch_bounds__(kKvThreads) gqa_prefill_kv_kernel(const PrefillParams p) {
  pdl_entry();
  extern __shared__ __align__(16) float kv_s[];  // K [64][kKvLd], V [64][kKvLd]
  float *Ks = kv_s, *Vs = kv_s + kBN * kKvLd;
  const int kt = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x;
  const long long past = p.lens[b];
  if (skip_seq(p, past)) return;
  const long long kend = past + p.T;
  const long long k0 = (long long)kt * kBN;
  if (k0 >= kend) return;
  const size_t cb = ((size_t)b * p.Hkv + kh) * p.cap * kD;
  for (int e = tid; e < kBN * (kD / 4); e += kKvThreads) {
    const int r = e / (kD / 4), c4 = e % (kD / 4);
    const long long key = k0 + r;
    float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
    if (key < kend) {
      kv = ld4(p.k_cache + cb + (size_t)key * kD + 4 * c4);
      vv = ld4(p.v_cache + cb + (size_t)key * kD + 4 * c4);
    }
    st4(Ks + r * kKvLd + 4 * c4, kv);
    st4(Vs + r * kKvLd + 4 * c4, vv);
  }
  __syncthreads();
  float *kb = p.kb + (((size_t)b * p.Hkv + kh) * p.nkt + kt) * kNQC * 2 * kKC;
  for (int e = tid; e < kNQC * kKC; e += kKvThreads) {
    const int c = e / kKC, w = e % kKC;
    const int cm = w >> 5, wi = w & 31;
    const int r = (cm >> 3) * 8 + (wi >> 2), dd = (cm & 7) * 4 + (wi & 3);  // blocked [64 x 32]
    const float v = Ks[r * kKvLd + c * kDC + dd];
    kb[(size_t)(2 * c) * kKC + w] = v;
    kb[(size_t)(2 * c + 1) * kKC + w] = umma::tf32_lo(v);
  }
  float *vb = p.vb + (((size_t)b * p.Hkv + kh) * p.nkt + kt) * 2 * 2 * kVH;
  for (int e = tid; e < 2 * kVH; e += kKvThreads) {
    const int h2 = e / kVH, w = e % kVH;
    const int cm = w >> 5, wi = w & 31;
    const int d = h2 * (kD / 2) + (cm >> 4) * 8 + (wi >> 2), key = (cm & 15) * 4 + (wi & 3);  // blocked [128 x 64]
    const float v = Vs[key * kKvLd + d];
    vb[(size_t)(2 * h2) * kVH + w] = v;
    vb[(size_t)(2 * h2 + 1) * kVH + w] = umma::tf32_lo(v);
  }
}

// ---------------------------------------------------------------- (3) attention
struct AttnSmem {
  float ring[2][kSlot];    // stage: Q chunk hi, lo | K chunk hi, lo   or   V^T half hi, lo
  float P[2][kBM * kBN];   // P hi, lo, blocked [128 x 64]
  uint32_t tbase;
  uint64_t full[2], empty[2], s_full, s_free, p_ready, o_full;
};

__global__ void __launch_bounds__(kAttnThreads, 1) gqa_prefill_attn_kernel(const PrefillParams p) {
  pdl_entry();
  extern __shared__ __align__(128) unsigned char smem_raw[];
  AttnSmem &sm = *reinterpret_cast<AttnSmem *>(smem_raw);
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z / p.ns, ks = blockIdx.z % p.ns;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kh = h / (p.Hq / p.Hkv);
  const long long past = p.lens[b];
  if (skip_seq(p, past)) return;
  const int q0 = qt * kBM, rows = min(kBM, p.T - q0);
  const long long kend = past + p.T;
  const long long klim = min(kend, past + q0 + rows);  // keys seen by the tile's last row
  const int ntk = (int)((klim + kBN - 1) / kBN);       // key tiles of this query tile
  const int nsplit = (ntk + kKS - 1) / kKS;
  const int t0 = ks * kKS;                              // first key tile of this CTA
  if (t0 >= ntk) return;
  const int nt = min(kKS, ntk - t0);
  const float *qbase = p.qb + (((size_t)b * p.Hq + h) * p.ntq + qt) * kNQC * 2 * kQC;
  const float *kbase = p.kb + ((size_t)b * p.Hkv + kh) * p.nkt * kNQC * 2 * kKC;
  const float *vbase = p.vb + ((size_t)b * p.Hkv + kh) * p.nkt * 2 * 2 * kVH;

  if (warp == 0) {
    umma::tmem_alloc(&sm.tbase, 512);
    umma::tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
    }
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.s_free, 4);
    mbar_init(&sm.p_ready, 4);
    mbar_init(&sm.o_full, 1);
    fence_mbar_init();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tb = sm.tbase;
  const uint32_t tS = tb, tO = tb + 256;
  bool ok = true;
  // diagnostics words after the status word: [1] barriers whose wait gave up,
  // [2] CTAs past the TMEM allocation, [3] CTAs done
  uint32_t *diag = p.status;
  if (tid == 0) atomicAdd(diag + 2, 1u);

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int n = 0;
      // stage n uses slot n % 2; the slot is refilled once the MMAs of stage n - 2 released it
      auto slot_for = [&](uint32_t bytes) -> int {
        const int s = n & 1;
        if (n >= 2 && ok && !mbar_wait(&sm.empty[s], ((n >> 1) - 1) & 1)) {
          ok = false;
          atomicOr(diag + 1, 0x1u);
        }
        ++n;
        if (!ok) return -1;
        mbar_arrive_expect_tx(&sm.full[s], bytes);
        return s;
      };
      auto qk = [&](int j) {
        for (int c = 0; c < kNQC; ++c) {
          const int s = slot_for((2 * kQC + 2 * kKC) * sizeof(float));
          if (s < 0) return;
          bulk_g2s(sm.ring[s], qbase + (size_t)c * 2 * kQC, 2 * kQC * sizeof(float), &sm.full[s], pol);
          bulk_g2s(sm.ring[s] + 2 * kQC, kbase + ((size_t)j * kNQC + c) * 2 * kKC, 2 * kKC * sizeof(float),
                   &sm.full[s], pol);
        }
      };
      auto pv = [&](int j) {
        for (int h2 = 0; h2 < 2; ++h2) {
          const int s = slot_for(2 * kVH * sizeof(float));
          if (s < 0) return;
          bulk_g2s(sm.ring[s], vbase + ((size_t)j * 2 + h2) * 2 * kVH, 2 * kVH * sizeof(float), &sm.full[s], pol);
        }
      };
      qk(t0);
      for (int j = 0; j < nt && ok; ++j) {
        if (j + 1 < nt) qk(t0 + j + 1);
        pv(t0 + j);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int n = 0;
      const uint32_t idS = umma::idesc_tf32(128, 64, 0, 0), idO = umma::idesc_tf32(128, 128, 0, 0);
      auto take = [&]() -> int {
        const int s = n & 1;
        if (ok && !mbar_wait(&sm.full[s], (n >> 1) & 1)) {
          ok = false;
          atomicOr(diag + 1, 0x2u);
        }
        ++n;
        umma::fence_after_sync();
        return s;
      };
      auto issue_qk = [&]() {
        for (int c = 0; c < kNQC && ok; ++c) {
          const int s = take();
          if (!ok) return;
          const float *Qh = sm.ring[s], *Ql = Qh + kQC, *Kh = Qh + 2 * kQC, *Kl = Kh + kKC;
#pragma unroll
          for (int ks = 0; ks < kDC / 8; ++ks) {
            constexpr uint32_t sbo = (kDC / 4) * 128;
            const uint64_t qh = umma::smem_desc(Qh + ks * 64, 128, sbo), ql = umma::smem_desc(Ql + ks * 64, 128, sbo);
            const uint64_t kh_ = umma::smem_desc(Kh + ks * 64, 128, sbo), kl = umma::smem_desc(Kl + ks * 64, 128, sbo);
            umma::mma_tf32(tS, qh, kh_, idS, (c > 0 || ks > 0) ? 1u : 0u);
            umma::mma_tf32(tS, qh, kl, idS, 1);
            umma::mma_tf32(tS, ql, kh_, idS, 1);
          }
          umma::commit(&sm.empty[s]);
        }
      };
      auto issue_pv = [&](int j) {
        for (int h2 = 0; h2 < 2 && ok; ++h2) {
          const int s = take();
          if (!ok) return;
          const float *Vh = sm.ring[s], *Vl = Vh + kVH;
#pragma unroll
          for (int ks = 0; ks < kBN / 8; ++ks) {
            constexpr uint32_t sbo = (kBN / 4) * 128;
            const uint64_t ph = umma::smem_desc(sm.P[0] + ks * 64, 128, sbo);
            const uint64_t pl = umma::smem_desc(sm.P[1] + ks * 64, 128, sbo);
            const uint64_t vh = umma::smem_desc(Vh + ks * 64, 128, sbo), vl = umma::smem_desc(Vl + ks * 64, 128, sbo);
            const uint32_t d = tO + 128 * h2;
            umma::mma_tf32(d, ph, vh, idO, (j > 0 || ks > 0) ? 1u : 0u);
            umma::mma_tf32(d, ph, vl, idO, 1);
            umma::mma_tf32(d, pl, vh, idO, 1);
          }
          umma::commit(&sm.empty[s]);
        }
      };
      issue_qk();
      umma::commit(&sm.s_full);
      for (int j = 0; j < nt; ++j) {
        if (ok && !mbar_wait(&sm.s_free, j & 1)) {  // softmax holds S(j) in registers
          ok = false;
          atomicOr(diag + 1, 0x4u);
        }
        if (j + 1 < nt) issue_qk();
        if (ok && !mbar_wait(&sm.p_ready, j & 1)) {  // P(j) written, O rescaled
          ok = false;
          atomicOr(diag + 1, 0x8u);
        }
        umma::fence_after_sync();
        issue_pv(j);
        umma::commit(j + 1 < nt ? &sm.s_full : &sm.o_full);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warps
    const int r = tid;  // query row = TMEM lane
    const long long qpos = past + q0 + r;
    const long long rlim = min(kend, qpos + 1);  // keys of this row: 0 .. rlim - 1
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
    float m_use = -INFINITY, l = 0.0f;
    for (int j = 0; j < nt; ++j) {
      if (ok && !mbar_wait(&sm.s_full, j & 1)) {
        ok = false;
        atomicOr(diag + 1, 0x10u);
      }
      umma::fence_after_sync();
      float s[kBN];
#pragma unroll
      for (int q = 0; q < kBN / 16; ++q)
        umma::ld_32x32b_x16(tS + lane_base + 16 * q, *reinterpret_cast<float(*)[16]>(&s[16 * q]));
      umma::wait_ld();
      umma::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.s_free);
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kBN; ++c) {
        const long long kidx = (long long)(t0 + j) * kBN + c;
        s[c] = kidx < rlim ? s[c] : -INFINITY;
        mx = fmaxf(mx, s[c]);
      }
      // New reference max when the row max grew by more than 2^8 (always on
      // the first tile).  tcgen05.ld / st are warp-collective (.sync.aligned),
      // so the O rescale runs for the whole warp when any of its rows needs
      // it; the other rows multiply by 1.
      const bool grow = mx > m_use + 8.0f;
      float f = 1.0f;
      if (grow && j > 0) f = exp2f(m_use - mx);
      if (grow) m_use = mx;
      const bool rescaled = j > 0 && __any_sync(0xffffffffu, grow);
      if (rescaled) {
        l *= f;
#pragma unroll 1
        for (int q = 0; q < kD / 16; ++q) {
          float o[16];
          umma::ld_32x32b_x16(tO + lane_base + 16 * q, o);
          umma::wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) o[e] *= f;
          umma::st_32x32b_x16(tO + lane_base + 16 * q, o);
        }
      }
      float sum = 0.0f;
#pragma unroll
      for (int c4 = 0; c4 < kBN / 4; ++c4) {
        float4 pv;
        // a row with no key in this CTA's range so far keeps m = -inf and p = 0
        const float mu = m_use == -INFINITY ? 0.0f : m_use;
        pv.x = exp2f(s[4 * c4 + 0] - mu);
        pv.y = exp2f(s[4 * c4 + 1] - mu);
        pv.z = exp2f(s[4 * c4 + 2] - mu);
        pv.w = exp2f(s[4 * c4 + 3] - mu);
        sum += (pv.x + pv.y) + (pv.z + pv.w);
        const int off = blk_off(r, 4 * c4, kBN);
        st4(sm.P[0] + off, pv);
        st4(sm.P[1] + off, lo4(pv));
      }
      l += sum;
      if (rescaled) umma::wait_st();
      fence_proxy_async_smem();
      umma::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_ready);
    }
    if (ok && !mbar_wait(&sm.o_full, 0)) {
      ok = false;
      atomicOr(diag + 1, 0x20u);
    }
    umma::fence_after_sync();
    // every lane takes part in the warp-collective TMEM loads; rows past the
    // prompt only skip the stores.  One key split: the final output; several:
    // this split's unnormalised O and (m, l) for the combine kernel.
    const bool live = r < rows;
    const size_t tok = (size_t)b * p.T + q0 + (live ? r : 0);
    const float *gate = p.q_gate + (tok * p.Hq + h) * 2 * kD + kD;
    const size_t pidx = ((((size_t)b * p.ntq + qt) * p.ns + ks) * p.Hq + h) * kBM + r;
    float *dst = nsplit == 1 ? p.out + (tok * p.Hq + h) * kD : p.po + pidx * kD;
    const float poison = __int_as_float(0x7fc00000);  // a bounded wait gave up
    const float inv = nsplit == 1 ? (ok ? 1.0f / l : poison) : (ok ? 1.0f : poison);
    if (nsplit > 1 && live) *reinterpret_cast<float2 *>(p.pml + 2 * pidx) = make_float2(m_use, l);
#pragma unroll 1
    for (int q = 0; q < kD / 16; ++q) {
      float o[16];
      umma::ld_32x32b_x16(tO + lane_base + 16 * q, o);
      umma::wait_ld();
      if (live) {
#pragma unroll
        for (int e = 0; e < 16; e += 4) {
          float4 v = make_float4(o[e] * inv, o[e + 1] * inv, o[e + 2] * inv, o[e + 3] * inv);
          if (nsplit == 1) {
            const float4 g = ld4(gate + 16 * q + e);
            v = make_float4(v.x * sigmoidf_dev(g.x), v.y * sigmoidf_dev(g.y), v.z * sigmoidf_dev(g.z),
                            v.w * sigmoidf_dev(g.w));
          }
          st4(dst + 16 * q + e, v);
        }
      }
    }
  }
  if (!ok) atomicOr(p.status, Q35_STATUS_WAIT_TIMEOUT);
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tb, 512);
  if (tid == 0) atomicAdd(diag + 3, 1u);
}

// ---------------------------------------------------------------- (3b) combine
// Query tiles with several key splits: merge the splits' (O, m, l) (base-2
// exponents) and apply the gate.  Grid (T, B), one warp per q head.
__global__ void gqa_prefill_combine_kernel(const PrefillParams p) {
  pdl_entry();
  const int t = blockIdx.x, b = blockIdx.y;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (h >= p.Hq) return;
  const long long past = p.lens[b];
  if (skip_seq(p, past)) return;
  const int qt = t / kBM, r = t % kBM, q0 = qt * kBM, rows = min(kBM, p.T - q0);
  const long long klim = min(past + p.T, past + q0 + rows);
  const int nsplit = (int)((klim + kBN - 1) / kBN + kKS - 1) / kKS;
  if (nsplit <= 1) return;
  const size_t base = (((size_t)b * p.ntq + qt) * p.ns * p.Hq + h) * kBM + r;  // split s: + s * Hq * kBM
  const size_t sstride = (size_t)p.Hq * kBM;
  float m = -INFINITY;
  for (int s = 0; s < nsplit; ++s) m = fmaxf(m, p.pml[2 * (base + s * sstride)]);
  float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
  float l = 0.0f;
  for (int s = 0; s < nsplit; ++s) {
    const size_t i = base + s * sstride;
    const float ms = p.pml[2 * i], ls = p.pml[2 * i + 1];
    const float w = ms == -INFINITY ? 0.0f : exp2f(ms - m);
    l = fmaf(ls, w, l);
    const float4 o0 = ld4(p.po + i * kD + 4 * lane), o1 = ld4(p.po + i * kD + 128 + 4 * lane);
    a0 = make_float4(fmaf(o0.x, w, a0.x), fmaf(o0.y, w, a0.y), fmaf(o0.z, w, a0.z), fmaf(o0.w, w, a0.w));
    a1 = make_float4(fmaf(o1.x, w, a1.x), fmaf(o1.y, w, a1.y), fmaf(o1.z, w, a1.z), fmaf(o1.w, w, a1.w));
  }
  const float inv = 1.0f / l;
  const size_t tok = (size_t)b * p.T + t;
  const float *gate = p.q_gate + (tok * p.Hq + h) * 2 * kD + kD;
  float *dst = p.out + (tok * p.Hq + h) * kD;
  const float4 g0 = ld4(gate + 4 * lane), g1 = ld4(gate + 128 + 4 * lane);
  st4(dst + 4 * lane, make_float4((a0.x * inv) * sigmoidf_dev(g0.x), (a0.y * inv) * sigmoidf_dev(g0.y),
                                  (a0.z * inv) * sigmoidf_dev(g0.z), (a0.w * inv) * sigmoidf_dev(g0.w)));
  st4(dst + 128 + 4 * lane, make_float4((a1.x * inv) * sigmoidf_dev(g1.x), (a1.y * inv) * sigmoidf_dev(g1.y),
                                        (a1.z * inv) * sigmoidf_dev(g1.z), (a1.w * inv) * sigmoidf_dev(g1.w)));
}

// ---------------------------------------------------------------- (4) lens
__global__ void gqa_prefill_lens_kernel(const PrefillParams p) {
  pdl_entry();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < p.B && !skip_seq(p, p.lens[b])) p.lens[b] += p.T;
}

struct PrefillWs {
  size_t qb, kb, vb, po, pml, total;  // float offsets after the 256-byte status block
  int ns;
};

PrefillWs prefill_ws(int B, int T, int Hq, int Hkv, long long max_len) {
  const size_t ntq = (size_t)(T + kBM - 1) / kBM, nkt = (size_t)((max_len + kBN - 1) / kBN);
  PrefillWs w;
  w.ns = (int)((nkt + kKS - 1) / kKS);
  w.qb = 64;  // floats: 256-byte status block first
  w.kb = w.qb + (size_t)B * Hq * ntq * kNQC * 2 * kQC;
  w.vb = w.kb + (size_t)B * Hkv * nkt * kNQC * 2 * kKC;
  w.po = w.vb + (size_t)B * Hkv * nkt * 2 * 2 * kVH;
  const size_t nrow = w.ns > 1 ? (size_t)B * ntq * w.ns * Hq * kBM : 0;
  w.pml = w.po + nrow * kD;
  w.total = w.pml + 2 * nrow;
  return w;
}

}  // namespace

size_t gqa_prefill_workspace_bytes(int B, int T, int Hq, int Hkv, long long max_len) {
  return prefill_ws(B, T, Hq, Hkv, max_len).total * sizeof(float);
}

int gqa_prefill_launch(const q35_gqa_dims *d, int T, long long max_len, const float *q_gate, const float *k_new,
                       const float *v_new, const float *qn_w, const float *kn_w, const float *cos,
                       const float *sin, float *k_cache, float *v_cache, int32_t *lens, float *out, void *ws,
                       size_t ws_bytes, cudaStream_t st) {
  const PrefillWs w = prefill_ws(d->batch, T, d->num_q_heads, d->num_kv_heads, max_len);
  Q35_REQUIRE(ws != nullptr && ws_bytes >= w.total * sizeof(float) && (reinterpret_cast<uintptr_t>(ws) & 255u) == 0,
              Q35_ERR_WORKSPACE,
              "gqa_prefill: workspace missing, not 256-byte aligned or too small (need " +
                  std::to_string(w.total * sizeof(float)) + " bytes)");
  float *wf = static_cast<float *>(ws);
  PrefillParams p;
  p.q_gate = q_gate; p.k_new = k_new; p.v_new = v_new; p.qn_w = qn_w; p.kn_w = kn_w; p.cos = cos; p.sin = sin;
  p.k_cache = k_cache; p.v_cache = v_cache; p.lens = lens; p.out = out;
  p.status = static_cast<uint32_t *>(ws);
  p.qb = wf + w.qb; p.kb = wf + w.kb; p.vb = wf + w.vb; p.po = wf + w.po; p.pml = wf + w.pml;
  p.ns = w.ns;
  p.cap = d->capacity;
  p.max_len = max_len;
  p.B = d->batch; p.T = T; p.Hq = d->num_q_heads; p.Hkv = d->num_kv_heads; p.rot = d->rotary_dim;
  p.ntq = (T + kBM - 1) / kBM;
  p.nkt = (int)((max_len + kBN - 1) / kBN);
  p.eps = d->eps;
  p.qscale = kLog2e / sqrtf((float)kD);
  Q35_REQUIRE(p.Hq + p.Hkv <= 32, Q35_ERR_UNSUPPORTED, "gqa_prefill: num_q_heads + num_kv_heads must be <= 32");
  Q35_REQUIRE(p.ntq <= 65535 && p.nkt <= 2147483647, Q35_ERR_UNSUPPORTED, "gqa_prefill: seq_len too large");

  cudaError_t e = cudaFuncSetAttribute(gqa_prefill_kv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)(2 * kBN * kKvLd * sizeof(float)));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gqa_prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(AttnSmem));
  if (e != cudaSuccess) return check_cuda(e, "gqa_prefill attributes");
  const int nw = p.Hq + p.Hkv;
  Q35_REQUIRE((long long)p.B * p.ns <= 65535, Q35_ERR_UNSUPPORTED, "gqa_prefill: batch x key splits too large");
  note_launch(p.ns > 1 ? 5 : 4);
  (void)launch_kernel(gqa_prefill_qkv_kernel, dim3(T, p.B), dim3(32 * nw), nw * kD * sizeof(float), st, 1, 1, p);
  (void)launch_kernel(gqa_prefill_kv_kernel, dim3(p.nkt, p.Hkv, p.B), dim3(kKvThreads), 2 * kBN * kKvLd * sizeof(float), st, 1, 1, p);
  (void)launch_kernel(gqa_prefill_attn_kernel, dim3(p.ntq, p.Hq, p.B * p.ns), dim3(kAttnThreads), sizeof(AttnSmem), st, 1, 1, p);
  if (p.ns > 1) (void)launch_kernel(gqa_prefill_combine_kernel, dim3(T, p.B), dim3(32 * p.Hq), 0, st, 1, 1, p);
  (void)launch_kernel(gqa_prefill_lens_kernel, dim3((p.B + 127) / 128), dim3(128), 0, st, 1, 1, p);
  return check_cuda(cudaGetLastError(), "gqa_prefill launch");
}

}  // namespace q35
