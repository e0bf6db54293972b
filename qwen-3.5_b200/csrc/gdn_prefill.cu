// gdn_prefill.cu -- Gated DeltaNet chunked prefill (WY form, chunk 64).
//
// Replaces the chunked branch of GatedDeltaNet::forward between the
// projections (inventwithdean/Qwen-3.5 src/text_modules.rs:531-552
// causal_conv1d_fn + conv-state capture, :554-615 split/expansion,
// :189-363 burn_chunk_gated_delta_rule, :651-660 RMSNormGated).
//
// Three kernels:
//  (1) gdn_prefill_chunk_kernel, grid (Hv, chunks, B), fully parallel: causal
//      conv + SiLU of the chunk's q/k/v channels (3-token halo from the
//      previous chunk or the cached conv state), l2norm, beta scaling,
//      cumulative decay gamma, the strictly-lower system
//      A = -tril((k*beta) k^T o D, -1) and Aqk = (q k^T) o D, the 63-row
//      forward substitution (text_modules.rs:280-287) as a blocked inverse,
//      T = A + I, U = T (v*beta), W = T (k*beta*e^gamma), q' = q e^gamma,
//      k' = k e^(gamma_last - gamma).  The contractions run on the tcgen05
//      tensor cores (3xTF32, TMEM accumulators).  Results go to the workspace.
//  (2) gdn_prefill_state_kernel, grid (8, Hv, B), walks the chunks in order.
//      The value columns of the state are independent recurrences, so each
//      CTA keeps 16 of them in shared memory, with no communication:
//      v' = U - W S, S <- S e^(gamma_last) + k'^T v' as 8 x 8 register tiles
//      (one shared-memory byte per FMA) with the contraction split across
//      thread groups, the next chunk's operands prefetched meanwhile.  It publishes the state at every chunk
//      start and v', and finally stores the state and the new conv state.
//  (3) gdn_prefill_output_kernel, grid (Hv, chunks, B), fully parallel:
//      o = q' S_c + Aqk v' on the tensor cores, then the gated RMS norm.
//  Only (2) is sequential, and it carries just the two contractions that the
//  recurrence needs.
#include "common.cuh"
#include "umma.cuh"

namespace q35 {
namespace {

constexpr int kC = 64;      // chunk length (text_modules.rs:645)
constexpr int kD = 128;     // head_k_dim == head_v_dim
constexpr int kCS = 16;     // value columns per CTA in the state kernel
constexpr int kSplit = kD / kCS;
constexpr int kThreads = 512;  // 16 warps: the chunk phases are latency-bound
constexpr int kStateThreads = 256;  // state pass: 4 compute warps (8 x 8 register tiles) + 4 for the merges
// Workspace record per (b, h, chunk), offsets in floats.  Tiles that the
// output kernel feeds to the tensor cores are stored in the 8x4-blocked
// K-major layout of umma.cuh, split into 64-column slabs so that every
// pipeline stage is one contiguous bulk copy.
constexpr int kOffU = 0;                  // U [64 t][128 v], row-major
constexpr int kOffWt = kC * kD;           // W^T [128 k][64 t], row-major
constexpr int kOffKp = 2 * kC * kD;       // k' [64 t][128 k], row-major
constexpr int kOffQs = 3 * kC * kD;       // q' [64 t][128 k]: 2 slabs of blocked [64][64]
constexpr int kOffAq = 4 * kC * kD;       // Aqk [64 i][64 j], blocked
constexpr int kOffDec = kOffAq + kC * kC; // e^(gamma_last) of the chunk, slot of 64
constexpr int kOffSc = kOffDec + 64;      // S_c^T [128 v][128 k] (state before the chunk): 2 slabs of blocked [128][64]
constexpr int kOffVt = kOffSc + kD * kD;  // v'^T [128 v][64 t], blocked
constexpr size_t kRec = (size_t)kOffVt + (size_t)kD * kC;
static_assert((kOffSc * 4) % 16 == 0 && (kOffVt * 4) % 16 == 0 && (kRec * 4) % 16 == 0, "16-byte aligned slots");

struct PrefillParams {
  const float *x, *z, *beta, *g, *conv_w, *norm_w;
  float *conv_state, *rec_state, *out, *ws;
  int B, T, NC, Hk, Hv, rf, C, has_prev, has_init;
  float eps;
};

// ---------------------------------------------------------------------------
// Kernel 1 on the 5th-generation tensor cores.  The four intra-chunk
// contractions run as tcgen05 kind::tf32 MMAs with f32 accumulators in TMEM,
// as 3xTF32 (hi*hi + hi*lo + lo*hi; the f32 buffer is the hi term because the
// tensor core reads f32 as truncated tf32) so the result keeps f32 accuracy:
//   G12 : D[128 x 64] = [k ; q] k^T           (rows 0-63: k k^T, 64-127: q k^T)
//   GU  : D[128 x 64] = v^T (T diag(beta))^T   = U^T
//   GW  : D[128 x 64] = k^T (T diag(beta e^g))^T = W^T
// All operands are K-major in the 8x4-blocked layout of umma.cuh.  Every
// shared-memory pass maps one warp onto one 8x4 core matrix (lane = row*4 +
// column), which keeps the blocked layout free of bank conflicts.
struct ChunkSmem {
  float r1[4][kC * kD];  // k | q | k_lo | q_lo  (blocked [64 x 128]); after G12:
                         // Tb+Tb_lo | kT | Te+Te_lo | kT_lo  (kT blocked [128 x 64])
  float vT[kD * kC];     // v^T blocked [128 x 64]
  float vT_lo[kD * kC];
  float Am[kC][kC + 4];  // A = -tril(diag(beta) k k^T o D, -1), then T = (I - A)^-1
  float gam[kC], bet[kC], eg[kC], ek[kC];
  uint32_t tbase;
  uint64_t bar1, bar2;
};

template <int KC>
__global__ void __launch_bounds__(kThreads, 1) gdn_prefill_chunk_kernel(const PrefillParams p) {
  pdl_entry();
  extern __shared__ __align__(128) unsigned char smem_raw[];
  ChunkSmem &sm = *reinterpret_cast<ChunkSmem *>(smem_raw);
  float *kS = sm.r1[0], *qS = sm.r1[1], *kL = sm.r1[2], *qL = sm.r1[3];
  // heads vary fastest: one wave then reads every head's channel columns of
  // its token rows instead of one 512-byte column group at the row stride
  const int h = blockIdx.x, c = blockIdx.y, b = blockIdx.z;
  const int hk = h / p.rf;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int lr = lane >> 2, lc = lane & 3;  // (row, column) inside an 8 x 4 core matrix
  const int t0 = c * kC;
  using umma::blk_off;

  if (warp == 0) {
    umma::tmem_alloc(&sm.tbase, 256);
    umma::tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&sm.bar1, 1);
    mbar_init(&sm.bar2, 1);
    fence_mbar_init();
  }

  // (1) causal conv + SiLU (text_modules.rs:164-182).  The chunk's raw q, k
  // and v rows (64 tokens x 128 channels each) are all requested at once with
  // 16-byte cp.async copies (96 KB in flight per SM) into the k_lo, q_lo and
  // v_lo slots, which are free until step (2); the 16-byte column groups of
  // row t are XOR-swizzled by t % 8 so that the conv reads below are free of
  // bank conflicts.  Rows >= T are zero-filled (the padding of :224-236).  The
  // K-1 history rows (previous chunk, or the cached conv state before the
  // first chunk) and the weights go to the A slot.
  {
    auto raw = [&](int sl) { return sl == 0 ? qL : (sl == 1 ? kL : sm.vT_lo); };
    float *hist = &sm.Am[0][0];              // [KC-1][3*128]
    float *wts = hist + (KC - 1) * 3 * kD;   // [3*128][KC]
    auto cbase = [&](int sl) {
      return sl == 0 ? (size_t)hk * kD : (sl == 1 ? (size_t)(p.Hk + hk) * kD : (size_t)2 * p.Hk * kD + (size_t)h * kD);
    };
#pragma unroll 4
    for (int e = tid; e < 3 * kC * (kD / 4); e += kThreads) {
      const int sl = e / (kC * (kD / 4)), rem = e % (kC * (kD / 4));
      const int t = rem >> 5, q4 = rem & 31;
      const bool in = t0 + t < p.T;
      const float *src = p.x + ((size_t)b * p.T + (in ? t0 + t : 0)) * p.C + cbase(sl) + 4 * q4;
      cp_async16_zfill(raw(sl) + t * kD + ((q4 ^ (t & 7)) << 2), src, in ? 16u : 0u);
    }
    if (t0 > 0) {  // history rows t0-KC+1 .. t0-1 of the three column slices
      for (int e = tid; e < (KC - 1) * 3 * (kD / 4); e += kThreads) {
        const int j = e / (3 * (kD / 4)), r = e % (3 * (kD / 4));
        const float *src = p.x + ((size_t)b * p.T + t0 - (KC - 1) + j) * p.C + cbase(r / (kD / 4)) + 4 * (r % (kD / 4));
        cp_async16(hist + j * 3 * kD + 4 * r, src);
      }
    } else {  // before the first chunk: the cached conv state, or zeros
      for (int e = tid; e < (KC - 1) * 3 * kD; e += kThreads) {
        const int j = e / (3 * kD), r = e % (3 * kD);
        const size_t cgl = cbase(r / kD) + (r % kD);
        hist[e] = p.has_prev ? p.conv_state[((size_t)b * p.C + cgl) * (KC - 1) + j] : 0.0f;
      }
    }
    for (int e = tid; e < 3 * kD * KC; e += kThreads) {
      const int r = e / KC, j = e % KC;
      cp_async4(wts + e, p.conv_w + (cbase(r / kD) + (r % kD)) * KC + j);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    // Lane (lr, lc) of warp w computes tokens 8 tg + lr (tg = w / 8 mod 2) of
    // channels 4 (w8 + 8 m) + lc, w8 = w % 8, m < 4: per store one whole 8 x 4
    // core matrix.  The swizzle only touches the low 3 bits of the column
    // group w8 + 8 m, so the read offset of row tau is
    // ((w8 ^ (tau % 8)) * 4 + lc) + 32 m.
    const int w8 = warp & 7;
#pragma unroll
    for (int sl = 0; sl < 3; ++sl) {
      const float *rs = raw(sl);
      float wv[4][KC];
#pragma unroll
      for (int m = 0; m < 4; ++m)
#pragma unroll
        for (int j = 0; j < KC; ++j) wv[m][j] = wts[(sl * kD + 4 * (w8 + 8 * m) + lc) * KC + j];
      int coff[KC];
#pragma unroll
      for (int j = 0; j < KC; ++j) coff[j] = ((w8 ^ ((lr - (KC - 1) + j) & 7)) << 2) + lc;
#pragma unroll 2
      for (int tg = warp >> 3; tg < kC / 8; tg += 2) {
        const int i = 8 * tg + lr;
        float xin[KC][4];
#pragma unroll
        for (int j = 0; j < KC; ++j) {
          const int tau = i - (KC - 1) + j;
          if (tau >= 0) {
#pragma unroll
            for (int m = 0; m < 4; ++m) xin[j][m] = rs[tau * kD + coff[j] + 32 * m];
          } else {
#pragma unroll
            for (int m = 0; m < 4; ++m) xin[j][m] = hist[(KC - 1 + tau) * 3 * kD + sl * kD + 4 * (w8 + 8 * m) + lc];
          }
        }
        const bool live = t0 + i < p.T;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          float acc = 0.0f;
#pragma unroll
          for (int j = 0; j < KC; ++j) acc = fmaf(wv[m][j], xin[j][m], acc);
          const float v = live ? __fdividef(acc, 1.0f + __expf(-acc)) : 0.0f;  // SiLU
          const int ch = 4 * (w8 + 8 * m) + lc;
          if (sl == 0) qS[blk_off(i, ch, kD)] = v;
          else if (sl == 1) kS[blk_off(i, ch, kD)] = v;
          else sm.vT[blk_off(ch, i, kC)] = v;
        }
      }
    }
  }
  if (tid < kC) {
    const int t = t0 + tid;
    sm.bet[tid] = t < p.T ? p.beta[((size_t)b * p.T + t) * p.Hv + h] : 0.0f;
    sm.gam[tid] = t < p.T ? p.g[((size_t)b * p.T + t) * p.Hv + h] : 0.0f;
  }
  __syncthreads();
  if (tid == 0) {  // cum_decay = cumsum(decay), sequential (:255)
    float a = 0.0f;
    for (int i = 0; i < kC; ++i) {
      a += sm.gam[i];
      sm.gam[i] = a;
    }
  }

  // (2) l2norm of q and k rows, q scaled by DK^-0.5 (:218-222), and the lo
  // terms; one warp per 8-row group (16 groups).
  const float qscale = rsqrtf((float)kD);
  for (int grp = warp; grp < 16; grp += kThreads / 32) {
    float *M = grp < 8 ? qS : kS, *ML = grp < 8 ? qL : kL;
    const int i = 8 * (grp & 7) + lr;
    float ss = 0.0f;
#pragma unroll 8
    for (int jj = 0; jj < kD / 4; ++jj) {
      const float v = M[blk_off(i, 4 * jj + lc, kD)];
      ss = fmaf(v, v, ss);
    }
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    const float inv = 1.0f / sqrtf(ss + 1e-6f);
    const float sc = grp < 8 ? qscale : 1.0f;
#pragma unroll 8
    for (int jj = 0; jj < kD / 4; ++jj) {
      const int off = blk_off(i, 4 * jj + lc, kD);
      const float v = (M[off] * inv) * sc;
      M[off] = v;
      ML[off] = umma::tf32_lo(v);
    }
  }
  for (int e = tid; e < kD * kC / 4; e += kThreads) {
    const float4 v = reinterpret_cast<const float4 *>(sm.vT)[e];
    reinterpret_cast<float4 *>(sm.vT_lo)[e] =
        make_float4(umma::tf32_lo(v.x), umma::tf32_lo(v.y), umma::tf32_lo(v.z), umma::tf32_lo(v.w));
  }
  fence_proxy_async_smem();
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tb = sm.tbase;
  if (tid < kC) {
    sm.eg[tid] = expf(sm.gam[tid]);
    sm.ek[tid] = expf(sm.gam[kC - 1] - sm.gam[tid]);
  }

  // (3) G12 (thread 0): D12 = [k ; q] k^T, K = 128 in 16 steps of 8
  if (tid == 0) {
    const uint32_t id = umma::idesc_tf32(128, 64, 0, 0);
    for (int st = 0; st < kD / 8; ++st) {
      const uint64_t hi = umma::smem_desc(kS + st * 64, 128, (kD / 4) * 128);
      const uint64_t lo = umma::smem_desc(kL + st * 64, 128, (kD / 4) * 128);
      umma::mma_tf32(tb, hi, hi, id, st > 0);
      umma::mma_tf32(tb, hi, lo, id, 1);
      umma::mma_tf32(tb, lo, hi, id, 1);
    }
    umma::commit(&sm.bar1);
  }
  __syncthreads();  // eg / ek ready

  float *rec = p.ws + (((size_t)b * p.Hv + h) * p.NC + c) * kRec;
  float *U = rec + kOffU, *Wt = rec + kOffWt, *Kp = rec + kOffKp;

  if (tid == 0) rec[kOffDec] = expf(sm.gam[kC - 1]);

  const bool g12_ok = mbar_wait(&sm.bar1, 0);
  umma::fence_after_sync();

  // (4) epilogue of G12: TMEM lane = row of [k k^T ; q k^T]; the four warps
  // w = quad + 4 qtr of lane quadrant quad read columns 16 qtr .. 16 qtr + 15.
  {
    const int quad = warp & 3, qtr = warp >> 2;
    const int row = 32 * quad + lane;
    float v[16];
    umma::ld_32x32b_x16(tb + ((uint32_t)(32 * quad) << 16) + 16 * qtr, v);
    umma::wait_ld();
    if (row < kC) {  // A = -tril(diag(beta) k k^T o D, -1) (:259-279)
      const int i = row;
      const float bi = sm.bet[i], gi = sm.gam[i];
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const int j = 16 * qtr + jj;
        sm.Am[i][j] = j < i ? -((v[jj] * bi) * expf(gi - sm.gam[j])) : 0.0f;
      }
    } else {  // Aqk = tril(q k^T o D), blocked [64 x 64] in the free k_lo slot
      const int i = row - kC;
      const float gi = sm.gam[i];
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const int j = 16 * qtr + jj;
        kL[blk_off(i, j, kC)] = j <= i ? v[jj] * expf(gi - sm.gam[j]) : 0.0f;
      }
    }
    if (!g12_ok && tid == 0) rec[kOffDec] = __int_as_float(0x7fc00000);  // poisons state and outputs
  }
  // q' = q e^gamma (:303-307) in place, then q' (as two blocked [64 x 64]
  // slabs: each 8-row group of the [64 x 128] tile is two 2 KB halves) and
  // Aqk go to the workspace as bulk copies.  Both slots are overwritten
  // from (5) on, so thread 0 waits until the copies have read them.
  for (int f = tid; f < kC * kD / 4; f += kThreads) {
    const float e = sm.eg[((f >> 8) << 3) + (f & 7)];
    float4 v = reinterpret_cast<const float4 *>(qS)[f];
    v = make_float4(v.x * e, v.y * e, v.z * e, v.w * e);
    reinterpret_cast<float4 *>(qS)[f] = v;
  }
  fence_proxy_async_smem();
  __syncthreads();
  if (tid == 0) {
#pragma unroll 1
    for (int rg = 0; rg < kC / 8; ++rg)
#pragma unroll
      for (int sl = 0; sl < 2; ++sl)
        bulk_s2g(rec + kOffQs + sl * kC * 64 + rg * 512, qS + rg * 1024 + sl * 512, 512 * sizeof(float));
    bulk_s2g(rec + kOffAq, kL, kC * kC * sizeof(float));
    bulk_commit();
    bulk_wait_read<0>();
  }
  __syncthreads();  // q and the Aqk staging are free from here on

  // (5) k^T (blocked [128 x 64]) + lo into the free q / q_lo slots, and
  // k' = k e^(gamma_last - gamma) (:308-311) to the workspace, on warps 2-15
  // while warps 0-1 run level 0 of (6).
  //
  // (6) T = (I - A)^-1 (the row recursion of :280-287 solves (I - A) T = I
  // for the strictly lower A), by 16 x 16 blocks in place in Am.  With
  // T = [[T0, 0], [X, T1]] for any split, X = T1 A10 T0.  Level 0 solves the
  // four diagonal blocks column by column; level 1 forms the blocks under
  // them (16 x 16 products), level 2 the lower-left 32 x 32 block.  The upper
  // triangle of Am stays zero; products go through the free k slot.
  float *kT = sm.r1[1], *kTL = sm.r1[3];
  constexpr int ld = kC + 4;
  float *Am = &sm.Am[0][0];
  if (warp >= 2) {
    constexpr int nw = kThreads / 32 - 2;
    for (int cm = warp - 2; cm < (kD / 8) * (kC / 4); cm += nw) {
      const int d = 8 * (cm / (kC / 4)) + lr, i = 4 * (cm % (kC / 4)) + lc;
      const float v = kS[blk_off(i, d, kD)];
      kT[blk_off(d, i, kC)] = v;
      kTL[blk_off(d, i, kC)] = umma::tf32_lo(v);
    }
    for (int it = warp - 2; it < (kC / 8) * (kD / 16); it += nw) {
      const int r = lane & 7, c4 = lane >> 3;
      const int i = 8 * (it / (kD / 16)) + r, d0 = 16 * (it % (kD / 16)) + 4 * c4;
      const float4 v = *reinterpret_cast<const float4 *>(&kS[blk_off(i, d0, kD)]);
      const float e = sm.ek[i];
      *reinterpret_cast<float4 *>(Kp + (size_t)i * kD + d0) = make_float4(v.x * e, v.y * e, v.z * e, v.w * e);
    }
  } else {  // level 0: block bb, column j
    const int bb = tid >> 4, j = tid & 15, o = 16 * bb;
    float cv[16];
#pragma unroll
    for (int m = 0; m < 16; ++m) cv[m] = m == j ? 1.0f : 0.0f;
#pragma unroll
    for (int i = 1; i < 16; ++i) {
      const float *arow = Am + (o + i) * ld + o;
      float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
      for (int m4 = 0; m4 < (i + 3) / 4; ++m4) {
        const float4 a = *reinterpret_cast<const float4 *>(arow + 4 * m4);  // a[m >= i] is 0
        s0 = fmaf(a.x, cv[4 * m4 + 0], s0);
        s1 = fmaf(a.y, cv[4 * m4 + 1], s1);
        s0 = fmaf(a.z, cv[4 * m4 + 2], s0);
        s1 = fmaf(a.w, cv[4 * m4 + 3], s1);
      }
      if (i > j) cv[i] = s0 + s1;
    }
    __syncwarp();  // both blocks of this warp are done reading A
#pragma unroll
    for (int i = 0; i < 16; ++i) Am[(o + i) * ld + o + j] = cv[i];
  }
  {
    float *Xs = sm.r1[0];  // [32][36], free once k^T and k' are out
    constexpr int xld = 36;
    __syncthreads();
    // level 1: X_p = A[2p+1][2p] T[2p][2p] -> Xs rows 16p.., then T[2p+1][2p] = T[2p+1][2p+1] X_p
    const int p1 = (tid >> 6) & 1, i1 = (tid & 63) >> 2, j1 = 4 * (tid & 3);
    const int o1 = 32 * p1;
    if (tid < 128) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const float a = Am[(o1 + 16 + i1) * ld + o1 + m];
        const float4 t = *reinterpret_cast<const float4 *>(Am + (o1 + m) * ld + o1 + j1);
        acc = f4_fma(a, t, acc);
      }
      *reinterpret_cast<float4 *>(Xs + (16 * p1 + i1) * xld + j1) = acc;
    }
    __syncthreads();
    if (tid < 128) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const float a = Am[(o1 + 16 + i1) * ld + o1 + 16 + m];
        const float4 x = *reinterpret_cast<const float4 *>(Xs + (16 * p1 + m) * xld + j1);
        acc = f4_fma(a, x, acc);
      }
      *reinterpret_cast<float4 *>(Am + (o1 + 16 + i1) * ld + o1 + j1) = acc;
    }
    __syncthreads();
    // level 2: X = A[32:][:32] T0 -> Xs, then T[32:][:32] = T1 X (2 columns per thread)
    const int i2 = tid >> 4, j2 = 2 * (tid & 15);
    {
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int m = 0; m < 32; ++m) {
        const float a = Am[(32 + i2) * ld + m];
        const float2 t = *reinterpret_cast<const float2 *>(Am + m * ld + j2);
        acc.x = fmaf(a, t.x, acc.x);
        acc.y = fmaf(a, t.y, acc.y);
      }
      *reinterpret_cast<float2 *>(Xs + i2 * xld + j2) = acc;
    }
    __syncthreads();
    {
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int m = 0; m < 32; ++m) {
        const float a = Am[(32 + i2) * ld + 32 + m];
        const float2 x = *reinterpret_cast<const float2 *>(Xs + m * xld + j2);
        acc.x = fmaf(a, x.x, acc.x);
        acc.y = fmaf(a, x.y, acc.y);
      }
      *reinterpret_cast<float2 *>(Am + (32 + i2) * ld + j2) = acc;
    }
  }
  __syncthreads();
  // T diag(beta) and T diag(beta e^gamma) (+ lo) blocked [64 (i) x 64 (j)]
  float *Tb = sm.r1[0], *TbL = sm.r1[0] + kC * kC, *Te = sm.r1[2], *TeL = sm.r1[2] + kC * kC;
  for (int cm = warp; cm < (kC / 8) * (kC / 4); cm += kThreads / 32) {
    const int i = 8 * (cm / (kC / 4)) + lr, j = 4 * (cm % (kC / 4)) + lc;
    const float t = sm.Am[i][j];
    const float tbv = t * sm.bet[j], tev = t * (sm.bet[j] * sm.eg[j]);
    const int off = blk_off(i, j, kC);
    Tb[off] = tbv;
    TbL[off] = umma::tf32_lo(tbv);
    Te[off] = tev;
    TeL[off] = umma::tf32_lo(tev);
  }
  fence_proxy_async_smem();
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();

  // (7) GU and GW (thread 0): K = 64 tokens in 8 steps
  if (tid == 0) {
    const uint32_t id = umma::idesc_tf32(128, 64, 0, 0);
    constexpr uint32_t sbo = (kC / 4) * 128;
    for (int st = 0; st < kC / 8; ++st) {
      const uint64_t vh = umma::smem_desc(sm.vT + st * 64, 128, sbo), vl = umma::smem_desc(sm.vT_lo + st * 64, 128, sbo);
      const uint64_t bh = umma::smem_desc(Tb + st * 64, 128, sbo), bl = umma::smem_desc(TbL + st * 64, 128, sbo);
      umma::mma_tf32(tb + 64, vh, bh, id, st > 0);
      umma::mma_tf32(tb + 64, vh, bl, id, 1);
      umma::mma_tf32(tb + 64, vl, bh, id, 1);
      const uint64_t kh = umma::smem_desc(kT + st * 64, 128, sbo), kl = umma::smem_desc(kTL + st * 64, 128, sbo);
      const uint64_t eh = umma::smem_desc(Te + st * 64, 128, sbo), el = umma::smem_desc(TeL + st * 64, 128, sbo);
      umma::mma_tf32(tb + 128, kh, eh, id, st > 0);
      umma::mma_tf32(tb + 128, kh, el, id, 1);
      umma::mma_tf32(tb + 128, kl, eh, id, 1);
    }
    umma::commit(&sm.bar2);
  }
  const bool g2_ok = mbar_wait(&sm.bar2, 0);
  umma::fence_after_sync();

  // (8) epilogue: TMEM lane = d.  U[i][d] from U^T (warps with (w / 4) % 2 = 0),
  // Wt[d][i] = W^T (the others); warps w >= 8 take column blocks 2 and 3.
  {
    const int quad = warp & 3, d = 32 * quad + lane;
    const bool isU = ((warp >> 2) & 1) == 0;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int cb = 2 * (warp >> 3) + cc;
      float v[16];
      umma::ld_32x32b_x16(tb + ((uint32_t)(32 * quad) << 16) + (isU ? 64 : 128) + 16 * cb, v);
      umma::wait_ld();
      if (isU) {
#pragma unroll
        for (int e = 0; e < 16; ++e) U[(size_t)(16 * cb + e) * kD + d] = v[e];
      } else {
#pragma unroll
        for (int e = 0; e < 16; e += 4)
          *reinterpret_cast<float4 *>(Wt + (size_t)d * kC + 16 * cb + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
      }
    }
    if (!g2_ok && tid == 0) rec[kOffDec] = __int_as_float(0x7fc00000);
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tb, 256);
  if (tid == 0) bulk_wait<0>();  // the q' / Aqk copies are complete before the CTA retires
}

// ---------------------------------------------------------------------------
// Kernel 2: the sequential pass over the chunks (:314-350 without the output
// term).  The value columns of the state are independent recurrences, so a
// CTA owns 16 of them ([128 k x 16 v] in shared memory) and needs no peer:
//   v' = U - W S,   S <- S e^(gamma_last) + k'^T v'.
// Per chunk it also publishes, as blocked tiles for the output kernel, the
// state at the chunk start (S_c^T) and v'^T.  W^T, k' and the decay of the
// next chunk are fetched by bulk copies (U by cp.async) during the current one.
struct StateSmem {
  float Wt[2][kD][kC];   // W^T of chunks c, c+1
  float Kp[2][kC][kD];   // k' of chunks c, c+1
  float U[2][kC][kCS];   // this CTA's 16 columns of U
  float dec[2][64];      // decay slot of the record
  float S[kD][kCS];      // the CTA's 16 state columns, [k][v]
  float4 Pv[128 * 16];   // partial tiles: float4 q of compute thread i at 16 i + (q ^ (i % 16))
  float Vn[kC][kCS];     // v'
  float Sst[2][2][16 * 64];  // staging of S^T (2 slabs of blocked [16 v x 64 k]), by chunk parity
  float Vst[2][16 * 64];     // staging of v'^T (blocked [16 v x 64 t]), by chunk parity
  uint64_t barW[2];
};

// W^T, k' and the decay of one chunk (bulk copies by thread 0) and this CTA's
// U columns (one 16-byte cp.async per thread: 64 rows x 4) into buffer `buf`.
__device__ __forceinline__ void fetch_chunk(StateSmem &sm, const float *rec, int col0, int buf, uint64_t pol,
                                            int tid) {
  if (tid == 0) {
    mbar_arrive_expect_tx(&sm.barW[buf], sizeof(sm.Wt[0]) + sizeof(sm.Kp[0]) + sizeof(sm.dec[0]));
    bulk_g2s(&sm.Wt[buf][0][0], rec + kOffWt, sizeof(sm.Wt[0]), &sm.barW[buf], pol);
    bulk_g2s(&sm.Kp[buf][0][0], rec + kOffKp, sizeof(sm.Kp[0]), &sm.barW[buf], pol);
    bulk_g2s(&sm.dec[buf][0], rec + kOffDec, sizeof(sm.dec[0]), &sm.barW[buf], pol);
  }
  if (tid < kC * kCS / 4) {
    const int r = tid >> 2, q4 = tid & 3;
    cp_async16(&sm.U[buf][r][4 * q4], rec + kOffU + (size_t)r * kD + col0 + 4 * q4);
  }
}

// Thread (r, q4) holds S[r][4 q4 .. 4 q4 + 3]; stage them as S^T rows 4 q4 + e.
__device__ __forceinline__ void stage_state(float (&st)[2][16 * 64], int r, int q4, float4 a) {
  using umma::blk_off;
  float *d = st[r >> 6];
  const int k = r & 63;
  d[blk_off(4 * q4 + 0, k, 64)] = a.x;
  d[blk_off(4 * q4 + 1, k, 64)] = a.y;
  d[blk_off(4 * q4 + 2, k, 64)] = a.z;
  d[blk_off(4 * q4 + 3, k, 64)] = a.w;
}

template <int KC>
__global__ void __launch_bounds__(kStateThreads) gdn_prefill_state_kernel(const PrefillParams p) {
  pdl_entry();
  extern __shared__ __align__(128) unsigned char smem_raw[];
  StateSmem &sm = *reinterpret_cast<StateSmem *>(smem_raw);
  const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x;
  const int col0 = s * kCS;
  float *Sg = p.rec_state + ((size_t)b * p.Hv + h) * kD * kD;
  float *rec0 = p.ws + ((size_t)b * p.Hv + h) * p.NC * kRec;
  uint64_t pol = 0;

  // thread roles.  Compute threads (tid < 128) hold an 8 x 8 register tile:
  //   W S   : k-slice ks = tid / 16 (16 of the 128 k), rows 8 tr .. 8 tr + 7 of
  //           the 64 tokens, columns 8 tc .. 8 tc + 7 of the 16;
  //   k'^T v': token slice ts = tid / 32 (16 of the 64 t), rows 8 kr .. of the
  //           128 k, columns 8 tc ...
  // A tile's float4 q (= 2 * row-in-tile + half) goes to slot 16 i + (q ^ (i
  // % 16)) of Pv: each store instruction of a warp spreads over all 32 banks,
  // and the two tiles of one row block (tc = 0, 1) are 512 contiguous bytes.
  // A merge warp takes one row block: lane l reads float4 l of that block in
  // every slice (conflict-free), which is row 8 rb + q / 2, quad 2 (l / 16) +
  // q % 2 with q = (l % 16) ^ ((2 rb + l / 16) % 16), so its writes of S, v'
  // rows are again 512 contiguous bytes.
  // (ur, uq0 .. uq0 + 1) are the two float4 of S this thread loads and stores.
  const int lane = tid & 31, warp = tid >> 5;
  const int ur = tid >> 1, uq0 = 2 * (tid & 1);
  auto merge_q = [&](int rb) { return (lane & 15) ^ ((2 * rb + (lane >> 4)) & 15); };

  {  // initial state, also published as S_0 (staging parity 1 = "chunk -1")
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
      if (p.has_init) a = *reinterpret_cast<const float4 *>(Sg + (size_t)ur * kD + col0 + 4 * (uq0 + e));
      *reinterpret_cast<float4 *>(&sm.S[ur][4 * (uq0 + e)]) = a;
      stage_state(sm.Sst[1], ur, uq0 + e, a);
    }
  }
  if (tid == 0) {
    mbar_init(&sm.barW[0], 1);
    mbar_init(&sm.barW[1], 1);
    fence_mbar_init();
    pol = l2_policy_evict_first();
  }
  fence_proxy_async_smem();
  __syncthreads();
  if (tid == 0) {
    bulk_s2g(rec0 + kOffSc + 16 * 64 * s, sm.Sst[1][0], 16 * 64 * sizeof(float));
    bulk_s2g(rec0 + kOffSc + kD * 64 + 16 * 64 * s, sm.Sst[1][1], 16 * 64 * sizeof(float));
    bulk_commit();
  }
  fetch_chunk(sm, rec0, col0, 0, pol, tid);
  cp_async_commit();

  // A wait that gives up (ok = false) stops this thread waiting and issuing
  // copies, but every barrier below is still executed; the final state is
  // then poisoned.
  bool ok = true;
  for (int c = 0; c < p.NC; ++c) {
    const int buf = c & 1;
    float *rec = rec0 + (size_t)c * kRec;
    if (ok && !mbar_wait(&sm.barW[buf], (c >> 1) & 1)) ok = false;  // W^T, k', decay of chunk c
    cp_async_wait<0>();                                                 // U of chunk c
    if (tid == 0) bulk_wait_read<1>();  // the stores of chunk c-2 have read staging buffer `buf`
    __syncthreads();  // chunk c-1 is done with buffer buf ^ 1 and with Pv
    if (c + 1 < p.NC && ok) fetch_chunk(sm, rec + kRec, col0, buf ^ 1, pol, tid);
    cp_async_commit();

    // v' = U - W S  (:315-324): [64 t x 128 k] x [128 k x 16 v], k split 8 ways
    if (tid < 128) {
      const int ks = tid >> 4, tr = (tid >> 1) & 7, tc = tid & 1;
      float acc[8][8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
#pragma unroll 4
      for (int kk = 0; kk < kD / 8; ++kk) {
        const int k = (kD / 8) * ks + kk;
        const float4 w0 = *reinterpret_cast<const float4 *>(&sm.Wt[buf][k][8 * tr]);
        const float4 w1 = *reinterpret_cast<const float4 *>(&sm.Wt[buf][k][8 * tr + 4]);
        const float4 s0 = *reinterpret_cast<const float4 *>(&sm.S[k][8 * tc]);
        const float4 s1 = *reinterpret_cast<const float4 *>(&sm.S[k][8 * tc + 4]);
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(wv[i], sv[j], acc[i][j]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        sm.Pv[16 * tid + ((2 * i) ^ (tid & 15))] = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
        sm.Pv[16 * tid + ((2 * i + 1) ^ (tid & 15))] = make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
      }
    }
    __syncthreads();
    {  // merge the 8 k-slices: warp w takes token rows 8 w .. 8 w + 7
      const int q = merge_q(warp);
      const int mt = 8 * warp + (q >> 1), mvq = 2 * (lane >> 4) + (q & 1);
      float4 v = *reinterpret_cast<const float4 *>(&sm.U[buf][mt][4 * mvq]);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const float4 pv = sm.Pv[16 * (16 * ks + 2 * warp) + lane];
        v = make_float4(v.x - pv.x, v.y - pv.y, v.z - pv.z, v.w - pv.w);
      }
      *reinterpret_cast<float4 *>(&sm.Vn[mt][4 * mvq]) = v;
      using umma::blk_off;
      sm.Vst[buf][blk_off(4 * mvq + 0, mt, kC)] = v.x;
      sm.Vst[buf][blk_off(4 * mvq + 1, mt, kC)] = v.y;
      sm.Vst[buf][blk_off(4 * mvq + 2, mt, kC)] = v.z;
      sm.Vst[buf][blk_off(4 * mvq + 3, mt, kC)] = v.w;
    }
    __syncthreads();

    // k'^T v'  (:342-349): [128 k x 64 t] x [64 t x 16 v], t split 4 ways
    if (tid < 128) {
      const int ts = tid >> 5, kr = lane >> 1, tc = lane & 1;
      float acc[8][8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
#pragma unroll 4
      for (int tt = 0; tt < kC / 4; ++tt) {
        const int t = (kC / 4) * ts + tt;
        const float4 k0 = *reinterpret_cast<const float4 *>(&sm.Kp[buf][t][8 * kr]);
        const float4 k1 = *reinterpret_cast<const float4 *>(&sm.Kp[buf][t][8 * kr + 4]);
        const float4 v0 = *reinterpret_cast<const float4 *>(&sm.Vn[t][8 * tc]);
        const float4 v1 = *reinterpret_cast<const float4 *>(&sm.Vn[t][8 * tc + 4]);
        const float kv[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
        const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(kv[i], vv[j], acc[i][j]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        sm.Pv[16 * tid + ((2 * i) ^ (tid & 15))] = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
        sm.Pv[16 * tid + ((2 * i + 1) ^ (tid & 15))] = make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
      }
    }
    __syncthreads();

    // S <- S e^(gamma_last) + k'^T v'  (:350); publish it as S_{c+1}.  Warp w
    // merges the k row blocks rb = 2 w, 2 w + 1 over the 4 t-slices.
    {
      const float dec = sm.dec[buf][0];
#pragma unroll
      for (int it = 0; it < 2; ++it) {
        const int rb = 2 * warp + it, q = merge_q(rb);
        const int k = 8 * rb + (q >> 1), vq = 2 * (lane >> 4) + (q & 1);
        float4 ps = sm.Pv[16 * (2 * rb) + lane];
#pragma unroll
        for (int t4 = 1; t4 < 4; ++t4) {
          const float4 pq = sm.Pv[16 * (32 * t4 + 2 * rb) + lane];
          ps = make_float4(ps.x + pq.x, ps.y + pq.y, ps.z + pq.z, ps.w + pq.w);
        }
        float4 a = *reinterpret_cast<const float4 *>(&sm.S[k][4 * vq]);
        a = make_float4(a.x * dec + ps.x, a.y * dec + ps.y, a.z * dec + ps.z, a.w * dec + ps.w);
        *reinterpret_cast<float4 *>(&sm.S[k][4 * vq]) = a;
        if (c + 1 < p.NC) stage_state(sm.Sst[buf], k, vq, a);
      }
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      bulk_s2g(rec + kOffVt + 16 * kC * s, sm.Vst[buf], 16 * kC * sizeof(float));
      if (c + 1 < p.NC) {
        bulk_s2g(rec + kRec + kOffSc + 16 * 64 * s, sm.Sst[buf][0], 16 * 64 * sizeof(float));
        bulk_s2g(rec + kRec + kOffSc + kD * 64 + 16 * 64 * s, sm.Sst[buf][1], 16 * 64 * sizeof(float));
      }
      bulk_commit();
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // the last update's rows were written by other threads
#pragma unroll
  for (int e = 0; e < 2; ++e)
    *reinterpret_cast<float4 *>(Sg + (size_t)ur * kD + col0 + 4 * (uq0 + e)) =
        *reinterpret_cast<const float4 *>(&sm.S[ur][4 * (uq0 + e)]);
  if (!ok && tid == 0) Sg[col0] = __int_as_float(0x7fc00000);  // a bounded wait gave up: poison the state

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
  if (tid == 0) bulk_wait<0>();  // every published tile is complete before the CTA retires
}

// ---------------------------------------------------------------------------
// Kernel 3: per (chunk, head), fully parallel, on the tensor cores:
//   o^T [128 v x 64 t] = S_c^T q'^T + v'^T Aqk^T   (:325-341)
// in three K = 64 stages (S_c^T / q' slab 0, slab 1, then v'^T / Aqk), each a
// bulk copy into one shared-memory buffer set; the lo terms of the 3xTF32
// split are formed in place.  One buffer set (98 KB) lets two CTAs share an
// SM, so one CTA's copies overlap the other's tensor-core work.  Epilogue:
// gated RMS norm over the 128 values of each token (:651-660, :85-117) and the
// output store.
constexpr int kOutThreads = 256;
struct OutSmem {
  float A[2][kD * 64];  // [hi, lo], blocked [128 x 64]
  float Bm[2][kC * 64]; // [hi, lo], blocked [64 x 64]
  float part[4][kC];
  float inv[kC];
  uint32_t tbase;
  uint64_t barL, barM;
};

__global__ void __launch_bounds__(kOutThreads, 2) gdn_prefill_output_kernel(const PrefillParams p) {
  pdl_entry();
  extern __shared__ __align__(128) unsigned char smem_raw[];
  OutSmem &sm = *reinterpret_cast<OutSmem *>(smem_raw);
  const int h = blockIdx.x, c = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t0 = c * kC;
  const float *rec = p.ws + (((size_t)b * p.Hv + h) * p.NC + c) * kRec;
  constexpr uint32_t kStageBytes = (kD * 64 + kC * 64) * sizeof(float);
  // stage st: (A, B) = (S_c^T slab st, q' slab st) for st < 2, (v'^T, Aqk) for st = 2
  auto load_stage = [&](int st, uint64_t pol) {
    mbar_arrive_expect_tx(&sm.barL, kStageBytes);
    const float *a = st < 2 ? rec + kOffSc + st * kD * 64 : rec + kOffVt;
    const float *bm = st < 2 ? rec + kOffQs + st * kC * 64 : rec + kOffAq;
    bulk_g2s(sm.A[0], a, kD * 64 * sizeof(float), &sm.barL, pol);
    bulk_g2s(sm.Bm[0], bm, kC * 64 * sizeof(float), &sm.barL, pol);
  };

  if (warp == 0) {
    umma::tmem_alloc(&sm.tbase, 64);
    umma::tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&sm.barL, 1);
    mbar_init(&sm.barM, 1);
    fence_mbar_init();
    load_stage(0, l2_policy_evict_first());
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tb = sm.tbase;
  const uint32_t id = umma::idesc_tf32(128, 64, 0, 0);
  bool ok = true;

  // the gate z of this thread's 32 (token, value) outputs, requested now so
  // that the loads overlap the contractions: TMEM lane = value column v,
  // warps w and w + 4 take tokens 0-31 and 32-63 of lane quadrant w % 4
  const int quad = warp & 3, half = warp >> 2;
  const int v = 32 * quad + lane;
  const size_t rs = (size_t)p.Hv * kD;
  const int nt = min(32, p.T - t0 - 32 * half);
  const float *__restrict__ zb = p.z + ((size_t)b * p.T + t0 + 32 * half) * rs + (size_t)h * kD + v;
  float zv[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) zv[j] = j < nt ? __ldg(zb + (size_t)j * rs) : 0.0f;

#pragma unroll 1
  for (int st = 0; st < 3; ++st) {
    if (ok && !mbar_wait(&sm.barL, st & 1)) ok = false;
    {  // lo terms
      const float4 *ah = reinterpret_cast<const float4 *>(sm.A[0]);
      float4 *al = reinterpret_cast<float4 *>(sm.A[1]);
      for (int e = tid; e < kD * 64 / 4; e += kOutThreads) {
        const float4 v = ah[e];
        al[e] = make_float4(umma::tf32_lo(v.x), umma::tf32_lo(v.y), umma::tf32_lo(v.z), umma::tf32_lo(v.w));
      }
      const float4 *bh = reinterpret_cast<const float4 *>(sm.Bm[0]);
      float4 *bl = reinterpret_cast<float4 *>(sm.Bm[1]);
      for (int e = tid; e < kC * 64 / 4; e += kOutThreads) {
        const float4 v = bh[e];
        bl[e] = make_float4(umma::tf32_lo(v.x), umma::tf32_lo(v.y), umma::tf32_lo(v.z), umma::tf32_lo(v.w));
      }
    }
    fence_proxy_async_smem();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (tid == 0) {
      constexpr uint32_t sbo = (64 / 4) * 128;
#pragma unroll 1
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t ah = umma::smem_desc(sm.A[0] + ks * 64, 128, sbo);
        const uint64_t al = umma::smem_desc(sm.A[1] + ks * 64, 128, sbo);
        const uint64_t bh = umma::smem_desc(sm.Bm[0] + ks * 64, 128, sbo);
        const uint64_t bl = umma::smem_desc(sm.Bm[1] + ks * 64, 128, sbo);
        umma::mma_tf32(tb, ah, bh, id, (st > 0 || ks > 0) ? 1u : 0u);
        umma::mma_tf32(tb, ah, bl, id, 1);
        umma::mma_tf32(tb, al, bh, id, 1);
      }
      umma::commit(&sm.barM);
      // the buffers take the next stage once this stage's MMAs have read them
      if (st < 2) {
        if (ok && !mbar_wait(&sm.barM, st & 1)) ok = false;
        if (ok) load_stage(st + 1, l2_policy_evict_first());
      }
    }
  }
  // stage 2 (and so every MMA) complete: the barrier's third phase (parity 0);
  // every thread has passed stage 2's barrier, so phases 0 and 1 are done
  if (ok && !mbar_wait(&sm.barM, 0)) ok = false;
  umma::fence_after_sync();

  // epilogue
  float o[32];
  umma::ld_32x32b_x16(tb + ((uint32_t)(32 * quad) << 16) + 32 * half, *reinterpret_cast<float(*)[16]>(&o[0]));
  umma::ld_32x32b_x16(tb + ((uint32_t)(32 * quad) << 16) + 32 * half + 16, *reinterpret_cast<float(*)[16]>(&o[16]));
  umma::wait_ld();
  {  // per-token sum of squares over the warp's 32 values: reduce-scatter, lane l ends with token 32 half + l
    float sq[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) sq[j] = o[j] * o[j];
#pragma unroll
    for (int w = 16; w >= 1; w >>= 1) {
      const bool upper = (lane & w) != 0;
#pragma unroll
      for (int j = 0; j < w; ++j) {
        const float send = upper ? sq[j] : sq[j + w];
        const float keep = upper ? sq[j + w] : sq[j];
        sq[j] = keep + __shfl_xor_sync(0xffffffffu, send, w);
      }
    }
    sm.part[quad][32 * half + lane] = sq[0];
  }
  __syncthreads();
  if (tid < kC) {
    const float tot = sm.part[0][tid] + sm.part[1][tid] + sm.part[2][tid] + sm.part[3][tid];
    sm.inv[tid] = 1.0f / sqrtf(tot / (float)kD + p.eps);
  }
  __syncthreads();
  const float wv = p.norm_w[v];
  float *__restrict__ ob = p.out + ((size_t)b * p.T + t0 + 32 * half) * rs + (size_t)h * kD + v;
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (j < nt) ob[(size_t)j * rs] = (wv * (o[j] * sm.inv[32 * half + j])) * siluf_dev(zv[j]);
  if (!ok && tid == 0 && nt > 0) ob[0] = __int_as_float(0x7fc00000);  // a bounded wait gave up: poison
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tb, 64);
}

template <int KC>
int launch_kc(const PrefillParams &p, cudaStream_t st) {
  const size_t s1 = sizeof(ChunkSmem), s2 = sizeof(StateSmem), s3 = sizeof(OutSmem);
  cudaError_t e = cudaFuncSetAttribute(gdn_prefill_chunk_kernel<KC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)s1);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gdn_prefill_state_kernel<KC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s2);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gdn_prefill_output_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s3);
  if (e != cudaSuccess) return check_cuda(e, "gdn_prefill attributes");
  note_launch();
  (void)launch_kernel(gdn_prefill_chunk_kernel<KC>, dim3(p.Hv, p.NC, p.B), dim3(kThreads), s1, st, 1, 1, p);
  if ((e = cudaGetLastError()) != cudaSuccess) return check_cuda(e, "gdn_prefill chunk launch");
  note_launch();
  (void)launch_kernel(gdn_prefill_state_kernel<KC>, dim3(kSplit, p.Hv, p.B), dim3(kStateThreads), s2, st, 1, 1, p);
  if ((e = cudaGetLastError()) != cudaSuccess) return check_cuda(e, "gdn_prefill state launch");
  note_launch();
  (void)launch_kernel(gdn_prefill_output_kernel, dim3(p.Hv, p.NC, p.B), dim3(kOutThreads), s3, st, 1, 1, p);
  return check_cuda(cudaGetLastError(), "gdn_prefill output launch");
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
  Q35_REQUIRE(p.NC <= 65535, Q35_ERR_UNSUPPORTED, "gdn_prefill: seq_len above 65535 chunks of 64");
  switch (d->conv_kernel) {
    case 2: return launch_kc<2>(p, st);
    case 3: return launch_kc<3>(p, st);
    default: return launch_kc<4>(p, st);
  }
}

}  // namespace q35
