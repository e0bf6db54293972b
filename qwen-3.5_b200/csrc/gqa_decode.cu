// gqa_decode.cu -- fused gated-GQA decode step (split-K flash-decode) for sm_100a.
//
// Replaces Attention::forward between the projections for seq_len == 1
// (inventwithdean/Qwen-3.5 src/text_modules.rs:866-936): q/gate split, q_norm /
// k_norm (RMSNorm with 1 + w, :800-809), partial RoPE (:754-774), the KV-cache
// append (:899-909, here in place at lens[b]), repeat_kv (:776-792, as head
// grouping with no copy), scaled-dot-product attention and the sigmoid gate.
//
// Grid (nsplit, Hkv, B); one CTA streams keys [s*kps, min((s+1)*kps, L)) of one
// (sequence, kv head) for all G = Hq/Hkv query heads of the group, so each K/V
// byte is read from HBM exactly once.  Warp roles:
//   * warp NW (producer): writes the new token's normalised, rotated key and
//     its value into the cache (only the CTA whose range holds position
//     lens[b]), then streams K and V tiles with bulk TMA copies
//     (cp.async.bulk + mbarrier complete_tx) into an NS-stage ring, with an
//     evict-first L2 policy;
//   * warps 0..NW-1 (consumers): each keeps its own online-softmax state
//     (running max / sum per head, G x 8 output accumulators per lane) over
//     KPW keys of every tile; a lane owns 8 of the 256 dims, q.k partial dots
//     are finished with a butterfly reduce-scatter across the warp.
// The CTA merges its warps in shared memory and writes an (m, l, o) partial to
// the workspace.  The splits are then merged in one of two ways:
//   * many sequences (long splits, several waves of CTAs): the last CTA of each
//     (sequence, kv head) to arrive (atomic ticket, no spin-wait) merges them
//     in a two-level tree, applies sigmoid(gate) and writes the output, while
//     other CTAs still stream; the last pair of a sequence increments lens[b];
//   * few sequences (one wave): the tree's chain of fences, tickets and
//     dependent L2 reads would sit after the stream (about 10 us on B200), so
//     the kernel just ends and gqa_split_combine_kernel, launched behind it,
//     merges every split in one pass and increments lens[b].
#include "common.cuh"
#include "gqa_common.cuh"

namespace q35 {
namespace {

using gqa::norm_rope;

constexpr int kD = 256;
constexpr int kNW = 8;            // consumer warps
constexpr int kThreads = (kNW + 1) * 32;
constexpr int kTK = 16;           // keys per pipeline stage
constexpr int kNS = 3;            // pipeline stages
constexpr int kKPW = kTK / kNW;   // keys per consumer warp per stage
constexpr int kFanIn = 8;         // partials merged per node of the combine tree

struct GqaParams {
  const float *q_gate, *k_new, *v_new, *qn_w, *kn_w, *cos, *sin;
  float *k_cache, *v_cache;
  int32_t *lens;
  float *out;
  float *part_out;     // optional [B, Hq, D+2] (o unnormalised | m (log2 units) | l) instead of `out`
  float *part_o;       // level 0: [B, Hkv, nsplit, G, D]
  float *part_ml;      // level 0: [B, Hkv, nsplit, G, 2]
  float *grp_o;        // level 1: [B, Hkv, ngroups, G, D]
  float *grp_ml;       // level 1: [B, Hkv, ngroups, G, 2]
  uint32_t *grp_cnt;   // [B * Hkv * ngroups]
  uint32_t *pair_cnt;  // [B * Hkv]
  uint32_t *seq_cnt;   // [B]
  int32_t *lsnap;      // [B]: keys attended this step (-1: the step was refused), for the split combine
  uint32_t *status;
  long long cap;
  int B, Hq, Hkv, rot, nsplit, kps, ngroups;
  int tree;  // 1: merge the splits in-kernel (ticket tree); 0: gqa_split_combine_kernel does
  int fault;  // test hook: CTA (0, 0, 0) issues none of its copies, so its waits run out
  uint64_t wait_ns;  // limit of every bounded wait
  float eps, qscale_log2;
};

struct GqaSmem {
  float k[kNS][kTK][kD];
  float v[kNS][kTK][kD];
};

// Butterfly reduce-scatter of V = 2^m partial sums across the warp: on return
// v[0] holds the full sum of value index (lane >> (5 - m)).
template <int V>
__device__ __forceinline__ void reduce_scatter(float (&v)[V], int lane) {
#pragma unroll
  for (int lvl = 0; lvl < 5; ++lvl) {
    const int off = 16 >> lvl;
    const int cnt = V >> lvl;
    if (cnt >= 2) {
      const bool upper = (lane & off) != 0;
#pragma unroll
      for (int i = 0; i < cnt / 2; ++i) {
        const float send = upper ? v[i] : v[i + cnt / 2];
        const float keep = upper ? v[i + cnt / 2] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
      }
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
    }
  }
}

// Final value of output element (head h, dim d): the gated, normalised
// attention output, or -- for a context-parallel caller -- the unnormalised
// (o, m, l) triple that q35_gqa_combine_partials merges across GPUs.
__device__ __forceinline__ void write_final(const GqaParams &p, int b, int h, int d, float O, float M, float Ls) {
  if (p.part_out != nullptr) {
    float *dst = p.part_out + ((size_t)b * p.Hq + h) * (kD + 2);
    dst[d] = O;
    if (d == 0) {
      dst[kD] = M;
      dst[kD + 1] = Ls;
    }
  } else {
    const float gate = p.q_gate[((size_t)b * p.Hq + h) * 2 * kD + kD + d];
    p.out[((size_t)b * p.Hq + h) * kD + d] = (O / Ls) * sigmoidf_dev(gate);
  }
}

// Merge n (m, l, o) partials (m in log2 units, o unnormalised) laid out as
// pml [n][G][2], po [n][G][D].  With out_ml == nullptr the result is final:
// out = o / l * sigmoid(gate); otherwise it is written as one partial of the
// same format to (out_ml, out_o).  Run by the 256 consumer threads.  Warp w
// takes partials w, w+NW, ...; a lane owns G*2 float4 of the [G][D] output, so
// it keeps G*2 independent 16-byte loads in flight per partial.  The per-head
// maxima come first (one online pass, lanes striding over partials); the
// warps' sums are merged through shared memory.
template <int G>
__device__ __forceinline__ void merge_partials(const GqaParams &p, const float *pml, const float *po_f, int n,
                                               float *out_ml, float *out_o, int kvh, int b, float *scratch,
                                               int warp, int lane, int tid) {
  constexpr int F = G * kD / 4 / 32;  // float4 per lane
  float *Mh = scratch + kNW * G * kD;  // [G] global max, [G] sum of l
  const float4 *po = reinterpret_cast<const float4 *>(po_f);
  if (warp < G) {
    const int g = warp;
    float M = -INFINITY, Ls = 0.0f;
#pragma unroll 4
    for (int j = lane; j < n; j += 32) {
      const float mj = __ldcg(pml + (j * G + g) * 2);
      const float lj = __ldcg(pml + (j * G + g) * 2 + 1);
      if (mj > M) {
        Ls = Ls * exp2f(M - mj) + lj;  // exp2(-inf) = 0 while M is still -inf
        M = mj;
      } else if (mj != -INFINITY) {
        Ls = fmaf(lj, exp2f(mj - M), Ls);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float Mo = __shfl_xor_sync(0xffffffffu, M, o);
      const float Lo = __shfl_xor_sync(0xffffffffu, Ls, o);
      const float Mn = fmaxf(M, Mo);
      Ls = (M == -INFINITY ? 0.0f : Ls * exp2f(M - Mn)) + (Mo == -INFINITY ? 0.0f : Lo * exp2f(Mo - Mn));
      M = Mn;
    }
    if (lane == 0) {
      Mh[g] = M;
      Mh[G + g] = Ls;
    }
  }
  named_bar_sync(1, kNW * 32);
  float Mg[G];
#pragma unroll
  for (int g = 0; g < G; ++g) Mg[g] = Mh[g];
  float4 acc[F];
#pragma unroll
  for (int f = 0; f < F; ++f) acc[f] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
  for (int j = warp; j < n; j += kNW) {
    float wgt[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float mj = __ldcg(pml + (j * G + g) * 2);
      wgt[g] = mj == -INFINITY ? 0.0f : exp2f(mj - Mg[g]);
    }
#pragma unroll
    for (int f = 0; f < F; ++f) {
      const float4 v = __ldcg(po + (size_t)j * (G * kD / 4) + lane + 32 * f);
      acc[f] = f4_fma(wgt[(32 * f) / (kD / 4)], v, acc[f]);  // lane < 32: head is f / 2
    }
  }
#pragma unroll
  for (int f = 0; f < F; ++f)
    reinterpret_cast<float4 *>(scratch)[(size_t)warp * (G * kD / 4) + lane + 32 * f] = acc[f];
  named_bar_sync(1, kNW * 32);
  for (int i = tid; i < G * kD; i += kNW * 32) {
    const int g = i / kD, d = i % kD;
    float O = 0.0f;
#pragma unroll
    for (int w = 0; w < kNW; ++w) O += scratch[(size_t)w * G * kD + i];
    if (out_ml == nullptr) {
      write_final(p, b, kvh * G + g, d, O, Mh[g], Mh[G + g]);
    } else {
      __stcg(out_o + i, O);
      if (d == 0) {
        __stcg(out_ml + g * 2 + 0, Mh[g]);
        __stcg(out_ml + g * 2 + 1, Mh[G + g]);
      }
    }
  }
}

template <int G>
__global__ void __launch_bounds__(kThreads, (G <= 4 ? 2 : 1)) gqa_decode_kernel(const GqaParams p) {
  constexpr int V = kKPW * G;  // (key, head) dots per warp per stage
  constexpr int LOGV = V == 1 ? 0 : V == 2 ? 1 : V == 4 ? 2 : V == 8 ? 3 : V == 16 ? 4 : 5;
  static_assert((1 << LOGV) == V && V <= 32, "V must be a power of two <= 32");

  extern __shared__ __align__(128) unsigned char smem_raw[];
  GqaSmem &sm = *reinterpret_cast<GqaSmem *>(smem_raw);
  __shared__ __align__(16) float q_s[G][kD];
  __shared__ __align__(16) float tmp_s[kNW + 1][kD];
  __shared__ __align__(8) uint64_t full_bar[kNS], empty_bar[kNS];
  __shared__ int last_flag;

  const int s = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const size_t pair = (size_t)b * p.Hkv + kvh;
  float *Kc = p.k_cache + pair * (size_t)p.cap * kD;
  float *Vc = p.v_cache + pair * (size_t)p.cap * kD;

  // Before the grid-dependency wait, only what no earlier kernel writes: the
  // ring barriers, and (few-sequence schedule, where this grid is launched
  // while the previous kernel drains) an L2 prefetch of the first ring's worth
  // of this split's cached keys and values.  Positions at or beyond lens[b]
  // may be fetched too (lens is not read yet); they stay inside the cache.
  if (tid == 0) {
    for (int i = 0; i < kNS; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], kNW);
    }
    fence_mbar_init();
  }
  if (!p.tree && warp == kNW && lane == 0) {
    const long long k0 = (long long)s * p.kps;
    const long long k1 = min(min(k0 + kNS * kTK, k0 + p.kps), p.cap);
    if (k1 > k0) {
      const uint32_t bytes = (uint32_t)(k1 - k0) * kD * sizeof(float);
      bulk_prefetch_l2(Kc + k0 * kD, bytes);
      bulk_prefetch_l2(Vc + k0 * kD, bytes);
    }
  }
  __syncthreads();
  pdl_entry();

  const int len = p.lens[b];
  const bool append = p.k_new != nullptr;  // false: attend the cached keys only (context-parallel shard)
  const int L = append ? len + 1 : len;
  const bool full = append && len >= p.cap, over = !full && L > p.nsplit * p.kps;
  if (s == 0 && kvh == 0 && tid == 0) {
    if (full) atomicOr(p.status, Q35_STATUS_CACHE_FULL);
    if (over) atomicOr(p.status, Q35_STATUS_LEN_HINT);
    if (!p.tree && p.nsplit > 1) p.lsnap[b] = (full || over) ? -1 : L;  // read by the split combine
  }
  if (full || over) return;
  const int kbeg = s * p.kps;
  const int kend = min(kbeg + p.kps, L);
  const int nkeys = max(kend - kbeg, 0);
  const int ntiles = (nkeys + kTK - 1) / kTK;

  if (warp == kNW) {
    // ---------------------------------------------------------- producer
    if (append && len >= kbeg && len < kend) {
      // This CTA owns the new position: k_norm + RoPE, append k and v.
      const float *kin = p.k_new + pair * kD;
      const float *vin = p.v_new + pair * kD;
      float4 x0 = *reinterpret_cast<const float4 *>(kin + 4 * lane);
      float4 x1 = *reinterpret_cast<const float4 *>(kin + 128 + 4 * lane);
      norm_rope(x0, x1, p.kn_w, p.cos + (size_t)b * p.rot, p.sin + (size_t)b * p.rot, p.rot, p.eps,
                tmp_s[kNW], lane);
      float *kd = Kc + (size_t)len * kD;
      float *vd = Vc + (size_t)len * kD;
      *reinterpret_cast<float4 *>(kd + 4 * lane) = x0;
      *reinterpret_cast<float4 *>(kd + 128 + 4 * lane) = x1;
      *reinterpret_cast<float4 *>(vd + 4 * lane) = *reinterpret_cast<const float4 *>(vin + 4 * lane);
      *reinterpret_cast<float4 *>(vd + 128 + 4 * lane) = *reinterpret_cast<const float4 *>(vin + 128 + 4 * lane);
      fence_proxy_async_global();
      __syncwarp();
    }
    if (lane == 0 && ntiles > 0) {
      const uint64_t pol = l2_policy_evict_first();
      const bool withhold = p.fault && s == 0 && kvh == 0 && b == 0;
      int issued = 0;
      for (int t = 0; t < ntiles && !withhold; ++t) {
        const int st = t % kNS;
        if (t >= kNS && !mbar_wait_ns(&empty_bar[st], ((t / kNS) - 1) & 1, p.wait_ns)) {
          atomicOr(p.status, Q35_STATUS_WAIT_TIMEOUT);
          break;
        }
        const int k0 = kbeg + t * kTK;
        const int nk = min(kTK, kend - k0);
        const uint32_t bytes = (uint32_t)nk * kD * sizeof(float);
        mbar_arrive_expect_tx(&full_bar[st], 2 * bytes);
        bulk_g2s(&sm.k[st][0][0], Kc + (size_t)k0 * kD, bytes, &full_bar[st], pol);
        bulk_g2s(&sm.v[st][0][0], Vc + (size_t)k0 * kD, bytes, &full_bar[st], pol);
        issued = t + 1;
      }
      // every copy this thread started has landed before the ring is reused
      for (int t = max(0, issued - kNS); t < issued; ++t)
        (void)mbar_wait_ns(&full_bar[t % kNS], (t / kNS) & 1, p.wait_ns);
    }
    __syncwarp();
    named_bar_arrive(2, (kNW + 1) * 32);  // the consumers may now reuse the ring
    return;
  }

  // ------------------------------------------------------------ consumers
  // q prologue: warp g < G normalises + rotates query head g of the group.
  if (warp < G) {
    const int h = kvh * G + warp;
    const float *qin = p.q_gate + ((size_t)b * p.Hq + h) * 2 * kD;
    float4 x0 = *reinterpret_cast<const float4 *>(qin + 4 * lane);
    float4 x1 = *reinterpret_cast<const float4 *>(qin + 128 + 4 * lane);
    norm_rope(x0, x1, p.qn_w, p.cos + (size_t)b * p.rot, p.sin + (size_t)b * p.rot, p.rot, p.eps,
              tmp_s[warp], lane);
    const float sc = p.qscale_log2;
    *reinterpret_cast<float4 *>(&q_s[warp][4 * lane]) = make_float4(x0.x * sc, x0.y * sc, x0.z * sc, x0.w * sc);
    *reinterpret_cast<float4 *>(&q_s[warp][128 + 4 * lane]) =
        make_float4(x1.x * sc, x1.y * sc, x1.z * sc, x1.w * sc);
  }
  named_bar_sync(1, kNW * 32);

  float4 q0[G], q1[G], a0[G], a1[G];
  float m_run[G], l_run[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    q0[g] = *reinterpret_cast<const float4 *>(&q_s[g][4 * lane]);
    q1[g] = *reinterpret_cast<const float4 *>(&q_s[g][128 + 4 * lane]);
    a0[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    a1[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    m_run[g] = -INFINITY;
    l_run[g] = 0.0f;
  }

  bool ok = true;
  for (int t = 0; t < ntiles && ok; ++t) {
    const int st = t % kNS;
    // warp-uniform: every lane of a warp leaves together (the shuffles below
    // need the full warp)
    if (!__all_sync(0xffffffffu, mbar_wait_ns(&full_bar[st], (t / kNS) & 1, p.wait_ns))) {
      if (lane == 0) atomicOr(p.status, Q35_STATUS_WAIT_TIMEOUT);
      ok = false;
      break;
    }
    const int nk = min(kTK, kend - (kbeg + t * kTK));
    float sv[V];
#pragma unroll
    for (int kk = 0; kk < kKPW; ++kk) {
      const int j = warp * kKPW + kk;
      if (j < nk) {
        const float4 k0 = *reinterpret_cast<const float4 *>(&sm.k[st][j][4 * lane]);
        const float4 k1 = *reinterpret_cast<const float4 *>(&sm.k[st][j][128 + 4 * lane]);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float d = q0[g].x * k0.x;
          d = fmaf(q0[g].y, k0.y, d); d = fmaf(q0[g].z, k0.z, d); d = fmaf(q0[g].w, k0.w, d);
          d = fmaf(q1[g].x, k1.x, d); d = fmaf(q1[g].y, k1.y, d); d = fmaf(q1[g].z, k1.z, d);
          d = fmaf(q1[g].w, k1.w, d);
          sv[kk * G + g] = d;
        }
      } else {
#pragma unroll
        for (int g = 0; g < G; ++g) sv[kk * G + g] = 0.0f;
      }
    }
    reduce_scatter<V>(sv, lane);
    // broadcast the V finished dots; invalid keys become -inf
    float sc[V];
#pragma unroll
    for (int i = 0; i < V; ++i) {
      sc[i] = __shfl_sync(0xffffffffu, sv[0], i << (5 - LOGV));
      if (warp * kKPW + i / G >= nk) sc[i] = -INFINITY;
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mt = sc[g];
#pragma unroll
      for (int kk = 1; kk < kKPW; ++kk) mt = fmaxf(mt, sc[kk * G + g]);
      if (mt > m_run[g]) {  // warp-uniform: every lane holds the same scores
        const float alpha = exp2f(m_run[g] - mt);  // exp2(-inf) = 0 on the first key
        l_run[g] *= alpha;
        a0[g].x *= alpha; a0[g].y *= alpha; a0[g].z *= alpha; a0[g].w *= alpha;
        a1[g].x *= alpha; a1[g].y *= alpha; a1[g].z *= alpha; a1[g].w *= alpha;
        m_run[g] = mt;
      }
    }
#pragma unroll
    for (int kk = 0; kk < kKPW; ++kk) {
      const int j = warp * kKPW + kk;
      if (j < nk) {
        const float4 v0 = *reinterpret_cast<const float4 *>(&sm.v[st][j][4 * lane]);
        const float4 v1 = *reinterpret_cast<const float4 *>(&sm.v[st][j][128 + 4 * lane]);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float pr = exp2f(sc[kk * G + g] - m_run[g]);
          l_run[g] += pr;
          a0[g] = f4_fma(pr, v0, a0[g]);
          a1[g] = f4_fma(pr, v1, a1[g]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[st]);
  }

  // ---- merge the NW warps of this CTA.  The producer has seen all its copies
  // land (barrier 2), so the ring is free for reuse.  A warp whose wait gave up
  // contributes nothing (m = -inf); the status word already says so.
  if (!ok) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m_run[g] = -INFINITY;
      l_run[g] = 0.0f;
      a0[g] = a1[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  named_bar_sync(2, (kNW + 1) * 32);
  float *wacc = &sm.k[0][0][0];            // [NW][G][D]
  float *wml = wacc + kNW * G * kD;        // [NW][G][2]
#pragma unroll
  for (int g = 0; g < G; ++g) {
    *reinterpret_cast<float4 *>(wacc + ((size_t)warp * G + g) * kD + 4 * lane) = a0[g];
    *reinterpret_cast<float4 *>(wacc + ((size_t)warp * G + g) * kD + 128 + 4 * lane) = a1[g];
    if (lane == 0) {
      wml[(warp * G + g) * 2 + 0] = m_run[g];
      wml[(warp * G + g) * 2 + 1] = l_run[g];
    }
  }
  named_bar_sync(1, kNW * 32);

  const bool single = p.nsplit == 1;
  float *po = p.part_o + (pair * p.nsplit + s) * G * kD;
  float *pml = p.part_ml + (pair * p.nsplit + s) * G * 2;
  for (int i = tid; i < G * kD; i += kNW * 32) {
    const int g = i / kD, d = i % kD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kNW; ++w) M = fmaxf(M, wml[(w * G + g) * 2]);
    float Ls = 0.0f, O = 0.0f;
#pragma unroll
    for (int w = 0; w < kNW; ++w) {
      const float mw = wml[(w * G + g) * 2];
      const float sc = mw == -INFINITY ? 0.0f : exp2f(mw - M);
      Ls = fmaf(wml[(w * G + g) * 2 + 1], sc, Ls);
      O = fmaf(wacc[((size_t)w * G + g) * kD + d], sc, O);
    }
    if (single) {
      write_final(p, b, kvh * G + g, d, O, M, Ls);
    } else {
      __stcg(po + i, O);
      if (d == 0) {
        __stcg(pml + g * 2 + 0, M);
        __stcg(pml + g * 2 + 1, Ls);
      }
    }
  }

  if (!single && !p.tree) return;  // gqa_split_combine_kernel merges the splits

  // ---- cross-CTA combine: a two-level ticket tree (fan-in 8, no spin-wait).
  // The last split of each group of 8 to arrive merges the group; the last
  // group to finish merges the group partials into the output.
  if (!single) {
    __threadfence();
    named_bar_sync(1, kNW * 32);
    const int grp = s / kFanIn;
    const int gsize = min(kFanIn, p.nsplit - grp * kFanIn);
    uint32_t *gc = p.grp_cnt + pair * p.ngroups + grp;
    if (tid == 0) last_flag = atomicAdd(gc, 1u) == (uint32_t)(gsize - 1);
    named_bar_sync(1, kNW * 32);
    if (!last_flag) return;
    __threadfence();
    const float *gml = p.part_ml + (pair * p.nsplit + grp * kFanIn) * G * 2;
    const float *go = p.part_o + (pair * p.nsplit + grp * kFanIn) * G * kD;
    if (p.ngroups == 1) {
      merge_partials<G>(p, gml, go, gsize, nullptr, nullptr, kvh, b, wacc, warp, lane, tid);
      if (tid == 0) *gc = 0u;
    } else {
      merge_partials<G>(p, gml, go, gsize, p.grp_ml + (pair * p.ngroups + grp) * G * 2,
                        p.grp_o + (pair * p.ngroups + grp) * G * kD, kvh, b, wacc, warp, lane, tid);
      if (tid == 0) *gc = 0u;
      __threadfence();
      named_bar_sync(1, kNW * 32);
      if (tid == 0) last_flag = atomicAdd(&p.pair_cnt[pair], 1u) == (uint32_t)(p.ngroups - 1);
      named_bar_sync(1, kNW * 32);
      if (!last_flag) return;
      __threadfence();
      merge_partials<G>(p, p.grp_ml + pair * p.ngroups * G * 2, p.grp_o + pair * p.ngroups * G * kD, p.ngroups,
                        nullptr, nullptr, kvh, b, wacc, warp, lane, tid);
      if (tid == 0) p.pair_cnt[pair] = 0u;
    }
  }
  // ---- the last (sequence, kv head) pair of sequence b advances lens[b]
  if (tid == 0) {
    __threadfence();
    const uint32_t t2 = atomicAdd(&p.seq_cnt[b], 1u);
    if (t2 == (uint32_t)(p.Hkv - 1)) {
      p.seq_cnt[b] = 0u;
      if (append) p.lens[b] = len + 1;
    }
  }
}

// Merge of the split partials of one decode step (the few-sequence regime):
// CTA (pair, head g, 32-dim slice), lane = one output dim.  Warp w takes the
// live splits w, w + 8, ... and merges them online (running maximum, rescaled
// sums), so no load waits for another: each warp issues all its splits' loads
// (up to kCombBatch) in one round, which is the whole critical path after the
// decode grid ends.  The warps' (m, l, o) meet in shared memory and go through
// write_final (gate, or the context-parallel triple).  One CTA per sequence
// advances lens[b]; no CTA of this kernel reads lens.
constexpr int kCombSlice = 32;
constexpr int kCombBatch = 20;

__device__ __forceinline__ void merge_online(float &m, float &l, float &o, float mj, float lj, float oj) {
  if (mj == -INFINITY) return;  // a split without keys adds nothing
  if (mj > m) {
    const float sc = exp2f(m - mj);  // exp2(-inf) = 0 while m is still -inf
    l = fmaf(l, sc, lj);
    o = fmaf(o, sc, oj);
    m = mj;
  } else {
    const float w = exp2f(mj - m);
    l = fmaf(lj, w, l);
    o = fmaf(oj, w, o);
  }
}

template <int G>
__global__ void __launch_bounds__(256) gqa_split_combine_kernel(const GqaParams p) {
  pdl_entry();
  __shared__ float red[8][32][3];  // [warp][lane][m, l, o]
  const int pg = blockIdx.x, slice = blockIdx.y;
  const size_t pair = (size_t)pg / G;
  const int g = pg % G;
  const int b = (int)(pair / p.Hkv), kvh = (int)(pair % p.Hkv);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int L = __ldcg(p.lsnap + b);
  if (L < 0) return;  // the decode step was refused (cache full / length hint): no output, lens unchanged
  const int d = slice * kCombSlice + lane;
  const float *pml = p.part_ml + pair * p.nsplit * G * 2 + g * 2;
  const float *po = p.part_o + pair * p.nsplit * G * kD + g * kD + d;
  const int nlive = min((L + p.kps - 1) / p.kps, p.nsplit);
  float m = -INFINITY, l = 0.0f, o = 0.0f;
  for (int j0 = warp; j0 < nlive; j0 += 8 * kCombBatch) {
    float mj[kCombBatch], lj[kCombBatch], oj[kCombBatch];
#pragma unroll
    for (int c = 0; c < kCombBatch; ++c) {
      const int j = j0 + 8 * c;
      if (j < nlive) {
        const float2 ml = __ldcg(reinterpret_cast<const float2 *>(pml + (size_t)j * G * 2));
        mj[c] = ml.x;
        lj[c] = ml.y;
        oj[c] = __ldcg(po + (size_t)j * G * kD);
      } else {
        mj[c] = -INFINITY;
        lj[c] = oj[c] = 0.0f;
      }
    }
#pragma unroll
    for (int c = 0; c < kCombBatch; ++c) merge_online(m, l, o, mj[c], lj[c], oj[c]);
  }
  red[warp][lane][0] = m;
  red[warp][lane][1] = l;
  red[warp][lane][2] = o;
  __syncthreads();
  if (warp == 0) {
    float M = -INFINITY, Ls = 0.0f, O = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) merge_online(M, Ls, O, red[w][lane][0], red[w][lane][1], red[w][lane][2]);
    write_final(p, b, kvh * G + g, d, O, M, Ls);
    if (lane == 0 && kvh == 0 && g == 0 && slice == 0 && p.k_new != nullptr) p.lens[b] = L;
  }
}

// out[b, h, :] = (sum_r o_r 2^(m_r - M)) / (sum_r l_r 2^(m_r - M)) * sigmoid(gate),
// M = max_r m_r, over n_parts partials [n][B][Hq][D+2] (one per context shard).
__global__ void gqa_combine_kernel(int B, int Hq, int n_parts, const float *__restrict__ parts,
                                   const float *__restrict__ q_gate, float *__restrict__ out) {
  pdl_entry();
  const int bh = blockIdx.x, d = threadIdx.x;
  const size_t stride = (size_t)B * Hq * (kD + 2);
  const float *base = parts + (size_t)bh * (kD + 2);
  float M = -INFINITY;
  for (int r = 0; r < n_parts; ++r) M = fmaxf(M, base[r * stride + kD]);
  float Ls = 0.0f, O = 0.0f;
  for (int r = 0; r < n_parts; ++r) {
    const float mr = base[r * stride + kD];
    const float sc = mr == -INFINITY ? 0.0f : exp2f(mr - M);
    Ls = fmaf(base[r * stride + kD + 1], sc, Ls);
    O = fmaf(base[r * stride + d], sc, O);
  }
  const float gate = q_gate[(size_t)bh * 2 * kD + kD + d];
  out[(size_t)bh * kD + d] = (O / Ls) * sigmoidf_dev(gate);
}

template <int G>
cudaError_t launch_g(const GqaParams &p, cudaStream_t st) {
  const size_t smem = sizeof(GqaSmem);
  static bool configured = false;  // per-process attribute set-up
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(gqa_decode_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  dim3 grid(p.nsplit, p.Hkv, p.B);
  note_launch();
  // The many-sequence schedule measured 8-10% slower with programmatic dependent
  // launch (its early-resident CTAs compete with the previous kernel); the
  // few-sequence one gains a little, its previous kernel being the combine.
  if (p.tree)
    (void)launch_kernel_serial(gqa_decode_kernel<G>, dim3(grid), dim3(kThreads), smem, st, 1, 1, p);
  else
    (void)launch_kernel(gqa_decode_kernel<G>, dim3(grid), dim3(kThreads), smem, st, 1, 1, p);
  if (p.nsplit > 1 && !p.tree) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    note_launch();
    (void)launch_kernel(gqa_split_combine_kernel<G>, dim3(p.B * p.Hkv * G, kD / kCombSlice), dim3(256), 0, st, 1,
                        1, p);
  }
  return cudaGetLastError();
}

}  // namespace

// Keys per split.  Large problems (many tiles per SM) use long splits so the
// combine traffic stays negligible; small ones are cut so that about one full
// wave of CTAs (2 per SM) is resident.
constexpr int kLongKps = 2048;  // split length of the many-sequence regime (in-kernel merge tree)

int gqa_keys_per_split(int B, int Hkv, long long max_len, int sms) {
  const long long pairs = (long long)B * Hkv;
  const long long slots = 2LL * sms;
  const long long long_kps = kLongKps;
  if (pairs * ((max_len + long_kps - 1) / long_kps) >= 8 * slots) return (int)long_kps;
  long long per = (max_len * pairs + slots - 1) / slots;
  per = (per + kTK - 1) / kTK * kTK;
  if (per < 2 * kTK) per = 2 * kTK;  // 2 tiles: both in flight at once (config 1: 13.2 -> 13.0 us per step)
  if (per > long_kps) per = long_kps;
  return (int)per;
}

struct GqaWsLayout {
  size_t status, grp_cnt, pair_cnt, seq_cnt, lsnap, part_o, part_ml, grp_o, grp_ml, total;
  int kps, nsplit, ngroups;
};

GqaWsLayout gqa_ws_layout(int B, int Hq, int Hkv, long long max_len, int sms) {
  GqaWsLayout l;
  l.kps = gqa_keys_per_split(B, Hkv, max_len, sms);
  l.nsplit = (int)((max_len + l.kps - 1) / l.kps);
  l.ngroups = (l.nsplit + kFanIn - 1) / kFanIn;
  const size_t G = (size_t)(Hq / Hkv), pairs = (size_t)B * Hkv;
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  l.status = 0;
  l.grp_cnt = 256;
  l.pair_cnt = l.grp_cnt + pairs * l.ngroups * sizeof(uint32_t);
  l.seq_cnt = l.pair_cnt + pairs * sizeof(uint32_t);
  l.lsnap = l.seq_cnt + (size_t)B * sizeof(uint32_t);
  l.part_o = up(l.lsnap + (size_t)B * sizeof(int32_t));
  l.part_ml = up(l.part_o + pairs * l.nsplit * G * kD * sizeof(float));
  l.grp_o = up(l.part_ml + pairs * l.nsplit * G * 2 * sizeof(float));
  l.grp_ml = up(l.grp_o + pairs * l.ngroups * G * kD * sizeof(float));
  l.total = up(l.grp_ml + pairs * l.ngroups * G * 2 * sizeof(float));
  return l;
}

size_t gqa_workspace_bytes(int B, int Hq, int Hkv, long long max_len, int sms) {
  return gqa_ws_layout(B, Hq, Hkv, max_len, sms).total;
}

// Bytes at the front of the workspace holding the status word and counters.
size_t gqa_workspace_counter_bytes(int B, int Hq, int Hkv, long long max_len, int sms) {
  return gqa_ws_layout(B, Hq, Hkv, max_len, sms).part_o;
}

int gqa_combine_launch(int B, int Hq, int n_parts, const float *parts, const float *q_gate, float *out,
                       cudaStream_t st) {
  if (B == 0) return Q35_OK;
  note_launch();
  (void)launch_kernel_serial(gqa_combine_kernel, dim3(B * Hq), dim3(kD), 0, st, 1, 1, B, Hq, n_parts, parts, q_gate, out);
  return check_cuda(cudaGetLastError(), "gqa_combine launch");
}

int gqa_decode_launch(const q35_gqa_dims *d, long long max_len, const float *q_gate, const float *k_new,
                      const float *v_new, const float *qn_w, const float *kn_w, const float *cos,
                      const float *sin, float *k_cache, float *v_cache, int32_t *lens, float *out,
                      void *ws, size_t ws_bytes, cudaStream_t st, float *part_out) {
  const int sms = device_sm_count();
  GqaParams p = {};
  p.B = d->batch; p.Hq = d->num_q_heads; p.Hkv = d->num_kv_heads; p.rot = d->rotary_dim;
  p.cap = d->capacity; p.eps = d->eps;
  const GqaWsLayout lay = gqa_ws_layout(p.B, p.Hq, p.Hkv, max_len, sms);
  p.kps = lay.kps;
  p.nsplit = lay.nsplit;
  p.ngroups = lay.ngroups;
  p.tree = lay.kps >= kLongKps;
  Q35_REQUIRE(ws != nullptr && ws_bytes >= lay.total && (reinterpret_cast<uintptr_t>(ws) & 255u) == 0,
              Q35_ERR_WORKSPACE,
              "gqa_decode: workspace missing, not 256-byte aligned or too small (need " +
                  std::to_string(lay.total) + " bytes)");
  Q35_REQUIRE(p.nsplit <= 65535, Q35_ERR_UNSUPPORTED, "gqa_decode: max_len too large for the split grid");
  p.q_gate = q_gate; p.k_new = k_new; p.v_new = v_new; p.qn_w = qn_w; p.kn_w = kn_w; p.cos = cos; p.sin = sin;
  p.k_cache = k_cache; p.v_cache = v_cache; p.lens = lens; p.out = out; p.part_out = part_out;
  p.qscale_log2 = (1.0f / sqrtf((float)kD)) * kLog2e;
  p.fault = take_fault(kFaultGqaDecode) ? 1 : 0;
  p.wait_ns = p.fault ? kFaultWaitLimitNs : kWaitLimitNs;
  unsigned char *base = static_cast<unsigned char *>(ws);
  p.status = reinterpret_cast<uint32_t *>(base + lay.status);
  p.grp_cnt = reinterpret_cast<uint32_t *>(base + lay.grp_cnt);
  p.pair_cnt = reinterpret_cast<uint32_t *>(base + lay.pair_cnt);
  p.seq_cnt = reinterpret_cast<uint32_t *>(base + lay.seq_cnt);
  p.lsnap = reinterpret_cast<int32_t *>(base + lay.lsnap);
  p.part_o = reinterpret_cast<float *>(base + lay.part_o);
  p.part_ml = reinterpret_cast<float *>(base + lay.part_ml);
  p.grp_o = reinterpret_cast<float *>(base + lay.grp_o);
  p.grp_ml = reinterpret_cast<float *>(base + lay.grp_ml);
  const int G = p.Hq / p.Hkv;
  cudaError_t e;
  switch (G) {
    case 1: e = launch_g<1>(p, st); break;
    case 2: e = launch_g<2>(p, st); break;
    case 4: e = launch_g<4>(p, st); break;
    case 8: e = launch_g<8>(p, st); break;
    default: return fail(Q35_ERR_UNSUPPORTED, "gqa_decode: group size must be 1, 2, 4 or 8");
  }
  return check_cuda(e, "gqa_decode launch");
}

}  // namespace q35
