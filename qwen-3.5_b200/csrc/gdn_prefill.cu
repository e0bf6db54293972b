// gdn_prefill.cu -- Gated DeltaNet chunked prefill (WY form, chunk 64).
//
// Replaces the chunked branch of GatedDeltaNet::forward between the
// projections (inventwithdean/Qwen-3.5 src/text_modules.rs:531-552
// causal_conv1d_fn + conv-state capture, :554-615 split/expansion,
// :189-363 burn_chunk_gated_delta_rule, :651-660 RMSNormGated).
//
// Two kernels:
//  (1) gdn_prefill_chunk_kernel, grid (chunks, Hv, B), fully parallel: causal
//      conv + SiLU of the chunk's q/k/v channels (3-token halo from the
//      previous chunk or the cached conv state), l2norm, beta scaling,
//      cumulative decay gamma, the strictly-lower system
//      A = -tril((k*beta) k^T o D, -1) and Aqk = (q k^T) o D, the 63-row
//      forward substitution (text_modules.rs:280-287), T = A + I,
//      U = T (v*beta), W = T (k*beta*e^gamma), q' = q e^gamma,
//      k' = k e^(gamma_last - gamma).  Results go to the workspace.
//  (2) gdn_prefill_state_kernel, grid (8, Hv, B) with 8-CTA clusters, walks
//      the chunks in order; each CTA keeps 16 of the 128 value columns of the
//      state in shared memory: v' = U - W S, o = q' S + Aqk v',
//      S <- S e^(gamma_last) + k'^T v'.  The cluster exchanges per-token sums
//      of squares through distributed shared memory for the gated RMS norm,
//      and the kernel finally stores the state and the new conv state.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace q35 {
namespace {

constexpr int kC = 64;      // chunk length (text_modules.rs:645)
constexpr int kD = 128;     // head_k_dim == head_v_dim
constexpr int kPad = 4;     // row padding (floats) of [64][128] smem tiles
constexpr int kLd = kD + kPad;
constexpr int kCS = 16;     // value columns per CTA in the state kernel
constexpr int kSplit = kD / kCS;
constexpr int kThreads = 256;
// workspace record per (b, h, chunk): U, W, q', k' [64x128] + Aqk [64x64] + decay
constexpr size_t kRec = 4 * (size_t)kC * kD + (size_t)kC * kC + 16;

struct PrefillParams {
  const float *x, *z, *beta, *g, *conv_w, *norm_w;
  float *conv_state, *rec_state, *out, *ws;
  int B, T, NC, Hk, Hv, rf, C, has_prev, has_init;
  float eps;
};

struct ChunkSmem {
  float q[kC][kLd];
  float k[kC][kLd];
  float v[kC][kLd];
  float A[kC][kC + 1];
  float Aqk[kC][kC + 1];
  float gam[kC], bet[kC], row[kC];
};

template <int KC>
__global__ void __launch_bounds__(kThreads) gdn_prefill_chunk_kernel(const PrefillParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  ChunkSmem &sm = *reinterpret_cast<ChunkSmem *>(smem_raw);
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / p.rf;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t0 = c * kC;

  // (1) causal conv + SiLU (text_modules.rs:164-182); tokens >= T are the
  // zero padding of :224-236 (q, k, v, beta, g all zero).
  for (int idx = tid; idx < kC * 3 * kD; idx += kThreads) {
    const int i = idx / (3 * kD), ch = idx % (3 * kD);
    const int t = t0 + i;
    float y = 0.0f;
    if (t < p.T) {
      int cg_;
      if (ch < kD) cg_ = hk * kD + ch;
      else if (ch < 2 * kD) cg_ = p.Hk * kD + hk * kD + (ch - kD);
      else cg_ = 2 * p.Hk * kD + h * kD + (ch - 2 * kD);
      const float *w = p.conv_w + (size_t)cg_ * KC;
      float acc = 0.0f;
#pragma unroll
      for (int j = 0; j < KC; ++j) {
        const int tau = t - (KC - 1) + j;
        float xv;
        if (tau >= 0) xv = p.x[((size_t)b * p.T + tau) * p.C + cg_];
        else xv = p.has_prev ? p.conv_state[((size_t)b * p.C + cg_) * (KC - 1) + (KC - 1) + tau] : 0.0f;
        acc = fmaf(w[j], xv, acc);
      }
      y = siluf_dev(acc);
    }
    float *dst = ch < kD ? &sm.q[i][ch] : ch < 2 * kD ? &sm.k[i][ch - kD] : &sm.v[i][ch - 2 * kD];
    *dst = y;
  }
  if (tid < kC) {
    const int t = t0 + tid;
    sm.bet[tid] = t < p.T ? p.beta[((size_t)b * p.T + t) * p.Hv + h] : 0.0f;
    sm.gam[tid] = t < p.T ? p.g[((size_t)b * p.T + t) * p.Hv + h] : 0.0f;
  }
  __syncthreads();

  // (2) l2norm of q and k per token, q scaled by DK^-0.5 (:218-222).
  const float qscale = rsqrtf((float)kD);
  for (int i = warp; i < kC; i += kThreads / 32) {
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int j = 0; j < kD / 32; ++j) {
      const float a = sm.q[i][lane + 32 * j], bb = sm.k[i][lane + 32 * j];
      sq = fmaf(a, a, sq);
      sk = fmaf(bb, bb, sk);
    }
    sq = warp_sum(sq);
    sk = warp_sum(sk);
    const float iq = 1.0f / sqrtf(sq + 1e-6f), ik = 1.0f / sqrtf(sk + 1e-6f);
#pragma unroll
    for (int j = 0; j < kD / 32; ++j) {
      sm.q[i][lane + 32 * j] = (sm.q[i][lane + 32 * j] * iq) * qscale;
      sm.k[i][lane + 32 * j] = sm.k[i][lane + 32 * j] * ik;
    }
  }
  if (tid == 0) {  // cum_decay = cumsum(decay), sequential (:255)
    float a = 0.0f;
    for (int i = 0; i < kC; ++i) {
      a += sm.gam[i];
      sm.gam[i] = a;
    }
  }
  __syncthreads();

  // (3) A = -tril((k*beta) k^T o D, -1), Aqk = tril((q k^T) o D) (:259-279).
  {
    const int i = tid / 4, jq = tid % 4;
    float aA[16], aQ[16];
#pragma unroll
    for (int m = 0; m < 16; ++m) aA[m] = aQ[m] = 0.0f;
    const float bi = sm.bet[i];
    for (int d = 0; d < kD; ++d) {
      const float qi = sm.q[i][d];
      const float kbi = sm.k[i][d] * bi;
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const float kj = sm.k[jq + 4 * m][d];
        aA[m] = fmaf(kbi, kj, aA[m]);
        aQ[m] = fmaf(qi, kj, aQ[m]);
      }
    }
    const float gi = sm.gam[i];
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      const int j = jq + 4 * m;
      const float dec = j <= i ? expf(gi - sm.gam[j]) : 0.0f;
      sm.A[i][j] = j < i ? -(aA[m] * dec) : 0.0f;
      sm.Aqk[i][j] = aQ[m] * dec;
    }
  }
  __syncthreads();

  // (4) forward substitution, row by row (:280-287):
  //     A[i,:i] <- A[i,:i] + A[i,:i] @ A[:i,:i]
  for (int i = 1; i < kC; ++i) {
    float nv = 0.0f;
    if (tid < i) {
      const int j = tid;
      float s = 0.0f;
      for (int m = j + 1; m < i; ++m) s = fmaf(sm.A[i][m], sm.A[m][j], s);
      nv = sm.A[i][j] + s;
    }
    __syncthreads();
    if (tid < i) sm.A[i][tid] = nv;
    __syncthreads();
  }
  if (tid < kC) sm.A[tid][tid] = 1.0f;  // T = A + I (:289-290)
  __syncthreads();

  // (5) U = T (v*beta), W = T (k*beta*e^gamma) (:292-293), q' and k' (:303-311)
  float *rec = p.ws + (((size_t)b * p.Hv + h) * p.NC + c) * kRec;
  float *U = rec, *W = rec + kC * kD, *Qp = rec + 2 * kC * kD, *Kp = rec + 3 * kC * kD;
  float *Aq = rec + 4 * kC * kD;
  {
    const int i = tid / 4, dq = tid % 4;
    float u[32], w[32];
#pragma unroll
    for (int m = 0; m < 32; ++m) u[m] = w[m] = 0.0f;
    for (int j = 0; j <= i; ++j) {
      const float tij = sm.A[i][j];
      const float bj = sm.bet[j];
      const float ej = bj * expf(sm.gam[j]);
#pragma unroll
      for (int m = 0; m < 32; ++m) {
        const int d = dq + 4 * m;
        u[m] = fmaf(tij, sm.v[j][d] * bj, u[m]);
        w[m] = fmaf(tij, sm.k[j][d] * ej, w[m]);
      }
    }
#pragma unroll
    for (int m = 0; m < 32; ++m) {
      const int d = dq + 4 * m;
      U[i * kD + d] = u[m];
      W[i * kD + d] = w[m];
    }
  }
  const float glast = sm.gam[kC - 1];
  for (int idx = tid; idx < kC * kD; idx += kThreads) {
    const int i = idx / kD, d = idx % kD;
    Qp[idx] = sm.q[i][d] * expf(sm.gam[i]);
    Kp[idx] = sm.k[i][d] * expf(glast - sm.gam[i]);
  }
  for (int idx = tid; idx < kC * kC; idx += kThreads) {
    const int i = idx / kC, j = idx % kC;
    Aq[idx] = j <= i ? sm.Aqk[i][j] : 0.0f;
  }
  if (tid == 0) Aq[kC * kC] = expf(glast);
}

struct StateSmem {
  float W[kC][kLd];
  float Q[kC][kLd];
  float K[kC][kD];
  float Aq[kC][kC + 4];
  float U[kC][kCS];
  float Vn[kC][kCS];
  float S[kD][kCS];
  float sq[2][kSplit][kC];
  float decay;
};

template <int KC>
__global__ void __launch_bounds__(kThreads) gdn_prefill_state_kernel(const PrefillParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  StateSmem &sm = *reinterpret_cast<StateSmem *>(smem_raw);
  cg::cluster_group cluster = cg::this_cluster();
  const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x;
  const int col0 = s * kCS;
  float *Sg = p.rec_state + ((size_t)b * p.Hv + h) * kD * kD;

  for (int idx = tid; idx < kD * kCS; idx += kThreads) {
    const int r = idx / kCS, cc = idx % kCS;
    sm.S[r][cc] = p.has_init ? Sg[(size_t)r * kD + col0 + cc] : 0.0f;
  }

  const int i = tid / 4, cq = tid % 4;  // output row / float4 column group
  for (int c = 0; c < p.NC; ++c) {
    const float *rec = p.ws + (((size_t)b * p.Hv + h) * p.NC + c) * kRec;
    const float *U = rec, *W = rec + kC * kD, *Qp = rec + 2 * kC * kD, *Kp = rec + 3 * kC * kD;
    const float *Aq = rec + 4 * kC * kD;
    __syncthreads();  // previous chunk is done with every smem tile
    for (int idx = tid; idx < kC * kD / 4; idx += kThreads) {
      const int r = idx / (kD / 4), q4 = idx % (kD / 4);
      *reinterpret_cast<float4 *>(&sm.W[r][4 * q4]) = __ldcg(reinterpret_cast<const float4 *>(W) + idx);
      *reinterpret_cast<float4 *>(&sm.Q[r][4 * q4]) = __ldcg(reinterpret_cast<const float4 *>(Qp) + idx);
      *reinterpret_cast<float4 *>(&sm.K[r][4 * q4]) = __ldcg(reinterpret_cast<const float4 *>(Kp) + idx);
    }
    for (int idx = tid; idx < kC * kC / 4; idx += kThreads) {
      const int r = idx / (kC / 4), q4 = idx % (kC / 4);
      *reinterpret_cast<float4 *>(&sm.Aq[r][4 * q4]) = __ldcg(reinterpret_cast<const float4 *>(Aq) + idx);
    }
    for (int idx = tid; idx < kC * kCS / 4; idx += kThreads) {
      const int r = idx / (kCS / 4), q4 = idx % (kCS / 4);
      *reinterpret_cast<float4 *>(&sm.U[r][4 * q4]) =
          __ldcg(reinterpret_cast<const float4 *>(U + (size_t)r * kD + col0) + q4);
    }
    if (tid == 0) sm.decay = __ldcg(Aq + kC * kC);
    __syncthreads();

    // v' = U - W S  (:315-324)
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < kD; ++k) acc = f4_fma(sm.W[i][k], *reinterpret_cast<const float4 *>(&sm.S[k][4 * cq]), acc);
    const float4 u = *reinterpret_cast<const float4 *>(&sm.U[i][4 * cq]);
    *reinterpret_cast<float4 *>(&sm.Vn[i][4 * cq]) =
        make_float4(u.x - acc.x, u.y - acc.y, u.z - acc.z, u.w - acc.w);
    __syncthreads();

    // o = q' S + Aqk v'  (:325-341)
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < kD; ++k) o = f4_fma(sm.Q[i][k], *reinterpret_cast<const float4 *>(&sm.S[k][4 * cq]), o);
    float4 o2 = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j <= i; ++j) o2 = f4_fma(sm.Aq[i][j], *reinterpret_cast<const float4 *>(&sm.Vn[j][4 * cq]), o2);
    o = make_float4(o.x + o2.x, o.y + o2.y, o.z + o2.z, o.w + o2.w);

    // per-token partial sum of squares over this CTA's 16 columns -> every
    // CTA of the cluster (double-buffered by chunk parity)
    float ss = o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w;
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    if (cq < kSplit / 2) {
      // lanes cq = 0..3 each push to two of the eight ranks
      *cluster.map_shared_rank(&sm.sq[c & 1][s][i], 2 * cq) = ss;
      *cluster.map_shared_rank(&sm.sq[c & 1][s][i], 2 * cq + 1) = ss;
    }

    // S <- S * decay + k'^T v'  (:342-349); rows r and r + 64
    float4 ns[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int r = i + 64 * hh;
      float4 a = *reinterpret_cast<const float4 *>(&sm.S[r][4 * cq]);
      a = make_float4(a.x * sm.decay, a.y * sm.decay, a.z * sm.decay, a.w * sm.decay);
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int t = 0; t < kC; ++t) kv = f4_fma(sm.K[t][r], *reinterpret_cast<const float4 *>(&sm.Vn[t][4 * cq]), kv);
      ns[hh] = make_float4(a.x + kv.x, a.y + kv.y, a.z + kv.z, a.w + kv.w);
    }
    __syncthreads();  // every thread finished reading S for this chunk
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) *reinterpret_cast<float4 *>(&sm.S[i + 64 * hh][4 * cq]) = ns[hh];

    cluster.sync();  // all sums of squares of this chunk have arrived
    const int t = c * kC + i;
    if (t < p.T) {
      float tot = 0.0f;
#pragma unroll
      for (int j = 0; j < kSplit; ++j) tot += sm.sq[c & 1][j][i];
      const float inv = 1.0f / sqrtf(tot / (float)kD + p.eps);
      const size_t obase = ((size_t)b * p.T + t) * p.Hv * kD + (size_t)h * kD + col0 + 4 * cq;
      const float ov[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = col0 + 4 * cq + e;
        p.out[obase + e] = (p.norm_w[col] * (ov[e] * inv)) * siluf_dev(p.z[obase + e]);
      }
    }
  }
  __syncthreads();
  for (int idx = tid; idx < kD * kCS; idx += kThreads) {
    const int r = idx / kCS, cc = idx % kCS;
    Sg[(size_t)r * kD + col0 + cc] = sm.S[r][cc];
  }

  // new conv state = last K-1 inputs of [history, x] (:538-540): v channels of
  // this CTA's columns, and (first value head of the key head) 32 of its 256
  // q/k channels.
  auto write_conv = [&](int ch) {
    float vals[KC - 1];
#pragma unroll
    for (int j = 0; j < KC - 1; ++j) {
      const int tau = p.T - (KC - 1) + j;
      vals[j] = tau >= 0 ? p.x[((size_t)b * p.T + tau) * p.C + ch]
                         : (p.has_prev ? p.conv_state[((size_t)b * p.C + ch) * (KC - 1) + (KC - 1) + tau] : 0.0f);
    }
#pragma unroll
    for (int j = 0; j < KC - 1; ++j) p.conv_state[((size_t)b * p.C + ch) * (KC - 1) + j] = vals[j];
  };
  if (tid < kCS) write_conv(2 * p.Hk * kD + h * kD + col0 + tid);
  if (h % p.rf == 0 && tid >= 32 && tid < 32 + 2 * kD / kSplit) {
    const int hk = h / p.rf;
    const int li = s * (2 * kD / kSplit) + (tid - 32);
    write_conv(li < kD ? hk * kD + li : p.Hk * kD + hk * kD + (li - kD));
  }
  cluster.sync();  // keep shared memory alive until all remote stores landed
}

template <int KC>
int launch_kc(const PrefillParams &p, cudaStream_t st) {
  const size_t s1 = sizeof(ChunkSmem), s2 = sizeof(StateSmem);
  cudaError_t e = cudaFuncSetAttribute(gdn_prefill_chunk_kernel<KC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)s1);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gdn_prefill_state_kernel<KC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s2);
  if (e != cudaSuccess) return check_cuda(e, "gdn_prefill attributes");
  note_launch();
  gdn_prefill_chunk_kernel<KC><<<dim3(p.NC, p.Hv, p.B), kThreads, s1, st>>>(p);
  if ((e = cudaGetLastError()) != cudaSuccess) return check_cuda(e, "gdn_prefill chunk launch");

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kSplit, p.Hv, p.B);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = s2;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kSplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  note_launch();
  return check_cuda(cudaLaunchKernelEx(&cfg, gdn_prefill_state_kernel<KC>, p), "gdn_prefill state launch");
}

}  // namespace

size_t gdn_prefill_workspace_bytes(const q35_gdn_dims *d, int T) {
  const size_t NC = (size_t)(T + kC - 1) / kC;
  return (size_t)d->batch * d->num_v_heads * NC * kRec * sizeof(float);
}

int gdn_prefill_launch(const q35_gdn_dims *d, int T, const float *mixed_qkv, const float *z, const float *beta,
                       const float *g, const float *conv_w, const float *norm_w, float *conv_state, int has_prev,
                       float *rec_state, int has_init, float *out, void *ws, size_t ws_bytes, cudaStream_t st) {
  const size_t need = gdn_prefill_workspace_bytes(d, T);
  Q35_REQUIRE(ws != nullptr && ws_bytes >= need && (reinterpret_cast<uintptr_t>(ws) & 15u) == 0, Q35_ERR_WORKSPACE,
              "gdn_prefill: workspace missing, unaligned or too small (need " + std::to_string(need) + " bytes)");
  PrefillParams p;
  p.x = mixed_qkv; p.z = z; p.beta = beta; p.g = g; p.conv_w = conv_w; p.norm_w = norm_w;
  p.conv_state = conv_state; p.rec_state = rec_state; p.out = out; p.ws = static_cast<float *>(ws);
  p.B = d->batch; p.T = T; p.NC = (T + kC - 1) / kC; p.Hk = d->num_k_heads; p.Hv = d->num_v_heads;
  p.rf = p.Hv / p.Hk; p.C = 2 * p.Hk * kD + p.Hv * kD; p.has_prev = has_prev; p.has_init = has_init;
  p.eps = d->eps;
  Q35_REQUIRE(p.NC <= 2147483647 / 1, Q35_ERR_UNSUPPORTED, "gdn_prefill: too many chunks");
  switch (d->conv_kernel) {
    case 2: return launch_kc<2>(p, st);
    case 3: return launch_kc<3>(p, st);
    default: return launch_kc<4>(p, st);
  }
}

}  // namespace q35
