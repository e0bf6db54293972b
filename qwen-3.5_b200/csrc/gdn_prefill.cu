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
//      CTA owns 16 of them, with no communication: v' = U - W S and
//      S <- S e^(gamma_last) + k'^T v' as two small tcgen05 MMAs per chunk
//      (3xTF32), the state in registers, the next chunk's operands copied
//      meanwhile.  It publishes the state at every chunk start and v', and
//      finally stores the state and the new conv state.
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
constexpr int kStateThreads = 384;  // state pass: 4 row warps, the MMA issuer warp, 3 W-lo warps, 4 k'^T warps
// Workspace record per (b, h, chunk), offsets in floats.  Tiles that the
// output kernel feeds to the tensor cores are stored in the 8x4-blocked
// K-major layout of umma.cuh, split into 64-column slabs so that every
// pipeline stage is one contiguous bulk copy.
constexpr int kOffU = 0;                  // U [64 t][128 v], row-major
constexpr int kOffW = kC * kD;           // W [64 t][128 k]: 2 slabs of blocked [64][64]
constexpr int kOffKp = 2 * kC * kD;       // k'^T [128 k][64 t], blocked
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
  uint32_t *status;   // word 0 of the workspace: Q35_STATUS_* bits
  uint64_t wait_ns;   // limit of every bounded wait
  int B, T, NC, Hk, Hv, rf, C, has_prev, has_init;
  int fault;          // test hook: the state pass withholds chunk 1's W copy
  float eps;
};

// Bytes in front of the per-(head, chunk) records: the status word.
constexpr size_t kWsHeader = 256;

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
  float *U = rec + kOffU, *Wk = rec + kOffW, *Kp = rec + kOffKp;

  if (tid == 0) rec[kOffDec] = expf(sm.gam[kC - 1]);

  const bool g12_ok = mbar_wait_ns(&sm.bar1, 0, p.wait_ns);
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
    if (!g12_ok && tid == 0) {
      rec[kOffDec] = __int_as_float(0x7fc00000);  // poisons state and outputs
      atomicOr(p.status, Q35_STATUS_WAIT_TIMEOUT);
    }
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
      Kp[blk_off(d, i, kC)] = v * sm.ek[i];  // k'^T, the A operand of the state pass
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
  const bool g2_ok = mbar_wait_ns(&sm.bar2, 0, p.wait_ns);
  umma::fence_after_sync();

  // (8) epilogue: TMEM lane = d.  U[i][d] from U^T (warps with (w / 4) % 2 = 0),
  // W[i][d] from W^T (the others); warps w >= 8 take column blocks 2 and 3.
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
        // W K-major, the A operand of the state pass: slab d / 64, blocked [64 t][64 k]
#pragma unroll
        for (int e = 0; e < 16; ++e) Wk[(d >> 6) * (kC * 64) + blk_off(16 * cb + e, d & 63, 64)] = v[e];
      }
    }
    if (!g2_ok && tid == 0) {
      rec[kOffDec] = __int_as_float(0x7fc00000);
      atomicOr(p.status, Q35_STATUS_WAIT_TIMEOUT);
    }
  }
  // Neither MMA group may still be writing TMEM when it is freed: after a
  // wait that gave up, warp 0 waits (bounded) once more for both commits.
  if (warp == 0 && !(g12_ok && g2_ok)) {
    (void)mbar_wait_ns(&sm.bar1, 0, p.wait_ns);
    (void)mbar_wait_ns(&sm.bar2, 0, p.wait_ns);
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tb, 256);
  if (tid == 0) bulk_wait<0>();  // the q' / Aqk copies are complete before the CTA retires
}

// ---------------------------------------------------------------------------
// Kernel 2: the sequential pass over the chunks (:314-350 without the output
// term), on the tensor cores.  The value columns of the state are independent
// recurrences, so a CTA owns 16 of them and needs no peer.  Per chunk:
//   MMA1  D1 = [W_hi; W_lo] [S_hi; S_lo]^T           M = 128, N = 32, K = 128
//   v' = U - (W_hi S_hi + W_hi S_lo + W_lo S_hi + W_lo S_lo)
//   MMA2  D2 = k'_hi [v'_hi; v'_lo]^T + k'_lo v'_hi^T   M = 128, K = 64
//   S_{c+1} = e^(gamma_last) S_c + D2
// with f32 accumulators in TMEM (3xTF32 or better).  A small tf32 MMA holds
// the tensor pipe for about 45-50 cycles whatever its N, its layout or where
// its A operand lives, so a chunk's time goes with its MMA count: W_lo is
// stacked under W_hi as rows 64-127 of one A operand, and the hi and lo rows
// of each B operand (S_c^T, v'^T) sit one above the other, for 16 + 16 MMAs.
// W (hi and lo) is double-buffered in shared memory; k'^T (hi and lo) is the
// A operand of MMA2 straight from TMEM.  The state itself stays in registers:
// thread k holds row k of the CTA's 16 columns.  Roles:
//   warps 0-3   the state rows; warps 2-3 hand the W_lo rows of D1 to warps
//               0-1 through shared memory, and warps 0-1 form v'.  They write
//               S_c^T and v'^T as hi / lo K-major operands (a per-lane
//               rotation of the 16 columns keeps the stores free of bank
//               conflicts);
//   thread 128  issues the MMAs, the bulk copies of the next chunk's W, an L2
//               prefetch two chunks ahead, and the stores that publish S_c^T
//               and v'^T for the output kernel;
//   warps 5-7   form the tf32 lo half of each W buffer;
//   warps 8-11  (one per TMEM lane quadrant) load k'^T rows into registers
//               ahead of time and store them, hi and lo, to TMEM once MMA2 of
//               the previous chunk is complete.
// The roles hand over through mbarriers only (every wait bounded), so each
// waits on its true dependency and nothing else.
struct StateSmem {
  float Wb[2][2 * kC * kD];  // W of chunks c, c+1: per k slab [hi, lo], each blocked [64 t][64 k]
  float Sb[2][2][kCS * 64];  // S_c^T, per k slab [hi, lo] of blocked [16 v][64 k]
  float Vb[2][kCS * kC];     // v'^T [hi, lo] of blocked [16 v][64 t]
  float X[kC][kCS + 4];      // the W_lo rows of D1, warps 2-3 -> warps 0-1
  uint64_t wfull[2], wlo, kready, sready, vready, m1, m2;
  uint32_t tbase;
};
static_assert(sizeof(StateSmem) <= 227 * 1024, "state pass shared memory");

constexpr int kStateRowThreads = 128;   // warps 0-3
constexpr int kStateIssuer = 128;       // warp 4, lane 0
constexpr int kStateLoThreads = 96;     // warps 5-7
constexpr int kStateKWarp0 = 8;         // warps 8-11: k'^T into TMEM
constexpr uint32_t kBarRows = 3;        // named barrier of the row warps
// TMEM columns: D1 0-31, D2 64-111, k'^T hi 128-191 and lo 192-255
constexpr uint32_t kTmemCols = 256, kColD2 = 64, kColKh = 128, kColKl = 192;

__device__ __forceinline__ void prefetch_l2_bulk(const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// tcgen05.mma with the A operand in tensor memory (columns = K, lane = row).
__device__ __forceinline__ void mma_tf32_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Row r (0..63) of a 16-column tile, written as column r of the K-major
// blocked [16][64] operand (hi and tf32 lo).  Lane group g = (lane / 4) % 8
// stores its columns rotated by g, so each store instruction of a warp covers
// all 32 banks.
__device__ __forceinline__ void store_operand_row(float *hi, float *lo, int r, const float (&v)[16], int lane) {
  const int rot = (lane >> 2) & 7;
  float a[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) a[i] = v[i];
#pragma unroll
  for (int sh = 1; sh < 8; sh <<= 1) {
    const bool on = (rot & sh) != 0;
    float t[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) t[i] = a[(i & 8) | ((i + sh) & 7)];
#pragma unroll
    for (int i = 0; i < 16; ++i) a[i] = on ? t[i] : a[i];
  }
  const int base = (r >> 2) * 32 + (r & 3);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int off = base + (i >> 3) * 512 + (((i + rot) & 7) << 2);
    hi[off] = a[i];
    lo[off] = umma::tf32_lo(a[i]);
  }
}

template <int KC>
__global__ void __launch_bounds__(kStateThreads, 1) gdn_prefill_state_kernel(const PrefillParams p) {
  pdl_entry();
  extern __shared__ __align__(128) unsigned char smem_raw[];
  StateSmem &sm = *reinterpret_cast<StateSmem *>(smem_raw);
  const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int col0 = s * kCS;
  const int NC = p.NC;
  float *Sg = p.rec_state + ((size_t)b * p.Hv + h) * kD * kD;
  float *rec0 = p.ws + ((size_t)b * p.Hv + h) * NC * kRec;

  if (warp == 4) {
    umma::tmem_alloc(&sm.tbase, kTmemCols);
    umma::tmem_relinquish();
  }
  if (tid == kStateIssuer) {
    mbar_init(&sm.wfull[0], 1);
    mbar_init(&sm.wfull[1], 1);
    mbar_init(&sm.wlo, kStateLoThreads);
    mbar_init(&sm.kready, 128);
    mbar_init(&sm.sready, kStateRowThreads);
    mbar_init(&sm.vready, kC);
    mbar_init(&sm.m1, 1);
    mbar_init(&sm.m2, 1);
    fence_mbar_init();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tb = sm.tbase;
  // A wait that gives up (ok = false) stops this thread waiting and writing
  // operands (its loop still runs, so every named barrier is met); the
  // issuer stops issuing and drains what it started; the final state is then
  // poisoned and the status word flagged.
  bool ok = true;
  const uint64_t wns = p.wait_ns;

  if (warp < 4) {
    // ---- state rows (k = tid); warps 0-1 are also the v' rows (t = tid)
    const int k = tid;
    const bool vrow = tid < kC;
    float S[16];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
      if (p.has_init) a = *reinterpret_cast<const float4 *>(Sg + (size_t)k * kD + col0 + 4 * q);
      S[4 * q] = a.x; S[4 * q + 1] = a.y; S[4 * q + 2] = a.z; S[4 * q + 3] = a.w;
    }
    store_operand_row(sm.Sb[k >> 6][0], sm.Sb[k >> 6][1], k & 63, S, lane);
    fence_proxy_async_smem();
    mbar_arrive(&sm.sready);

    float Un[16];
    auto load_u = [&](const float *rec) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 a = __ldcg(reinterpret_cast<const float4 *>(rec + kOffU + (size_t)tid * kD + col0 + 4 * q));
        Un[4 * q] = a.x; Un[4 * q + 1] = a.y; Un[4 * q + 2] = a.z; Un[4 * q + 3] = a.w;
      }
    };
    if (vrow) load_u(rec0);
    float decn = __ldcg(rec0 + kOffDec);
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
    for (int c = 0; c < NC; ++c) {
      const float *rec = rec0 + (size_t)c * kRec;
      const float dec = decn;
      float U[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) U[j] = Un[j];
      if (c + 1 < NC) {
        if (vrow) load_u(rec + kRec);
        decn = __ldcg(rec + kRec + kOffDec);
      }
      {  // v' = U - W S_c  (:315-324); TMEM lane = row of [W_hi; W_lo]
        if (ok && !mbar_wait_ns(&sm.m1, c & 1, wns)) ok = false;
        __syncwarp();
        umma::fence_after_sync();
        float d[16], e[16];
        umma::ld_32x32b_x16(tb + lane_base, d);
        umma::ld_32x32b_x16(tb + lane_base + 16, e);
        umma::wait_ld();
        if (!vrow && ok) {  // W_lo rows: W_lo S_hi + W_lo S_lo of token tid - 64
          float4 *x = reinterpret_cast<float4 *>(&sm.X[tid - kC][0]);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            x[q] = make_float4(d[4 * q] + e[4 * q], d[4 * q + 1] + e[4 * q + 1], d[4 * q + 2] + e[4 * q + 2],
                               d[4 * q + 3] + e[4 * q + 3]);
        }
        named_bar_sync(kBarRows, kStateRowThreads);
        if (vrow && ok) {
          const float4 *x = reinterpret_cast<const float4 *>(&sm.X[tid][0]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 xl = x[q];
            d[4 * q] = U[4 * q] - ((d[4 * q] + e[4 * q]) + xl.x);
            d[4 * q + 1] = U[4 * q + 1] - ((d[4 * q + 1] + e[4 * q + 1]) + xl.y);
            d[4 * q + 2] = U[4 * q + 2] - ((d[4 * q + 2] + e[4 * q + 2]) + xl.z);
            d[4 * q + 3] = U[4 * q + 3] - ((d[4 * q + 3] + e[4 * q + 3]) + xl.w);
          }
          store_operand_row(sm.Vb[0], sm.Vb[1], tid, d, lane);
          fence_proxy_async_smem();
          umma::fence_before_sync();
          mbar_arrive(&sm.vready);
        }
      }
      // S <- S e^(gamma_last) + k'^T v'  (:342-350)
      if (ok && !mbar_wait_ns(&sm.m2, c & 1, wns)) ok = false;
      __syncwarp();
      umma::fence_after_sync();
      float d[16], e[16], f[16];
      umma::ld_32x32b_x16(tb + lane_base + kColD2, d);
      umma::ld_32x32b_x16(tb + lane_base + kColD2 + 16, e);
      umma::ld_32x32b_x16(tb + lane_base + kColD2 + 32, f);
      umma::wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) S[j] = S[j] * dec + ((d[j] + e[j]) + f[j]);
      if (c + 1 < NC && ok) {
        store_operand_row(sm.Sb[k >> 6][0], sm.Sb[k >> 6][1], k & 63, S, lane);
        fence_proxy_async_smem();
        umma::fence_before_sync();
        mbar_arrive(&sm.sready);
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *reinterpret_cast<float4 *>(Sg + (size_t)k * kD + col0 + 4 * q) =
          make_float4(S[4 * q], S[4 * q + 1], S[4 * q + 2], S[4 * q + 3]);
  } else if (tid == kStateIssuer) {
    // ---- MMA issue, W copies, publication stores
    const uint64_t pol = l2_policy_evict_first();
    constexpr uint32_t kSlabBytes = (uint32_t)(kC * 64 * sizeof(float));
    auto load_w = [&](int c) {  // the hi half of each k slab
      const float *src = rec0 + (size_t)c * kRec + kOffW;
      mbar_arrive_expect_tx(&sm.wfull[c & 1], 2 * kSlabBytes);
      bulk_g2s(sm.Wb[c & 1], src, kSlabBytes, &sm.wfull[c & 1], pol);
      bulk_g2s(sm.Wb[c & 1] + 2 * kC * 64, src + kC * 64, kSlabBytes, &sm.wfull[c & 1], pol);
    };
    constexpr uint32_t kPrefetch = (kOffKp + kD * kC - kOffU) * sizeof(float);  // U, W, k'^T
    // Chunks [0, w_issued) have had their W copy issued, [0, w_seen) have
    // been observed complete; m1_last / m2_last are the last chunks whose MMA
    // groups were committed.  After a wait that gave up, nothing new is
    // issued and every started copy and MMA is waited for (bounded) before
    // the CTA frees its TMEM and shared memory.
    int w_issued = 1, w_seen = 0, m1_last = -1, m2_last = -1;
    const bool withhold = p.fault != 0;  // test hook: chunk 1's W copy is never issued
    load_w(0);
    if (NC > 1) prefetch_l2_bulk(rec0 + kRec + kOffU, kPrefetch);
    const uint32_t idw = umma::idesc_tf32(128, 2 * kCS, 0, 0), idn = umma::idesc_tf32(128, kCS, 0, 0);
    constexpr uint32_t sbo = (64 / 4) * 128;
    for (int c = 0; c < NC; ++c) {
      const int buf = c & 1;
      float *rec = rec0 + (size_t)c * kRec;
      // S_c is in Sb, and MMA2 of chunk c-1 is complete: W buffer buf ^ 1 is free
      if (ok && !mbar_wait_ns(&sm.sready, c & 1, wns)) ok = false;
      if (!ok) break;
      if (c + 1 < NC && !(withhold && c + 1 == 1)) {
        load_w(c + 1);
        w_issued = c + 2;
      }
      if (c + 2 < NC) {
        prefetch_l2_bulk(rec + 2 * kRec + kOffU, kPrefetch);
        prefetch_l2_bulk(rec + 2 * kRec + kOffDec, 64 * sizeof(float));
      }
      bulk_s2g(rec + kOffSc + 16 * 64 * s, sm.Sb[0][0], 16 * 64 * sizeof(float));
      bulk_s2g(rec + kOffSc + kD * 64 + 16 * 64 * s, sm.Sb[1][0], 16 * 64 * sizeof(float));
      bulk_commit();
      if (ok && !mbar_wait_ns(&sm.wfull[buf], (c >> 1) & 1, wns)) ok = false;
      if (ok) w_seen = c + 1;
      if (ok && !mbar_wait_ns(&sm.wlo, c & 1, wns)) ok = false;
      if (!ok) break;
      bulk_wait_read<1>();  // the v'^T store of chunk c-1 has read Vb
      umma::fence_after_sync();
      // Descriptors advance by adding the byte offset / 16 to the start
      // address field (every operand lies below 228 KB, so it cannot carry).
      const uint64_t dW = umma::smem_desc(sm.Wb[buf], 128, sbo);       // rows 0-63 hi, 64-127 lo
      const uint64_t dSb = umma::smem_desc(&sm.Sb[0][0][0], 128, sbo);  // [hi; lo] rows per k slab
#pragma unroll
      for (int ks = 0; ks < kD / 8; ++ks) {
        const uint64_t ao = (uint64_t)(((ks >> 3) * (2 * kC * 64) + (ks & 7) * 64) * 4 / 16);
        const uint64_t bo = (uint64_t)(((ks >> 3) * (2 * kCS * 64) + (ks & 7) * 64) * 4 / 16);
        umma::mma_tf32(tb, dW + ao, dSb + bo, idw, ks > 0 ? 1u : 0u);
      }
      umma::commit(&sm.m1);
      m1_last = c;
      if (ok && !mbar_wait_ns(&sm.kready, c & 1, wns)) ok = false;
      if (ok && !mbar_wait_ns(&sm.vready, c & 1, wns)) ok = false;
      if (!ok) break;
      bulk_wait_read<0>();  // the S_c^T stores have read Sb before S_{c+1} replaces it
      umma::fence_after_sync();
      const uint64_t dVb = umma::smem_desc(sm.Vb[0], 128, sbo);  // [hi; lo] rows
#pragma unroll
      for (int ks = 0; ks < kC / 8; ++ks) {
        const uint64_t o = (uint64_t)(ks * 64 * 4 / 16);
        mma_tf32_tmem_a(tb + kColD2, tb + kColKh + 8 * ks, dVb + o, idw, ks > 0 ? 1u : 0u);
        mma_tf32_tmem_a(tb + kColD2 + 32, tb + kColKl + 8 * ks, dVb + o, idn, ks > 0 ? 1u : 0u);
      }
      umma::commit(&sm.m2);
      m2_last = c;
      bulk_s2g(rec + kOffVt + 16 * kC * s, sm.Vb[0], 16 * kC * sizeof(float));
      bulk_commit();
    }
    for (int j = w_seen; j < w_issued; ++j) (void)mbar_wait_ns(&sm.wfull[j & 1], (j >> 1) & 1, wns);
    if (m1_last >= 0) (void)mbar_wait_ns(&sm.m1, m1_last & 1, wns);
    if (m2_last >= 0) (void)mbar_wait_ns(&sm.m2, m2_last & 1, wns);
    bulk_wait<0>();  // every published tile is complete before the CTA retires
  } else if (warp >= 5 && warp < kStateKWarp0) {
    // ---- tf32 lo half of each W buffer, once MMA1 of the previous chunk is
    // complete (which keeps this role at most one chunk ahead)
    const int t = tid - 5 * 32;
    for (int c = 0; c < NC; ++c) {
      const int buf = c & 1;
      if (ok && !mbar_wait_ns(&sm.wfull[buf], (c >> 1) & 1, wns)) ok = false;
      if (c > 0 && ok && !mbar_wait_ns(&sm.m1, (c - 1) & 1, wns)) ok = false;
      float4 *w4 = reinterpret_cast<float4 *>(sm.Wb[buf]);
      for (int e = t; ok && e < 2 * kC * 64 / 4; e += kStateLoThreads) {
        const int i = (e >> 10) * (2 * kC * 64 / 4) + (e & 1023);  // float4 of k slab e / 1024
        const float4 v = w4[i];
        w4[i + kC * 64 / 4] =
            make_float4(umma::tf32_lo(v.x), umma::tf32_lo(v.y), umma::tf32_lo(v.z), umma::tf32_lo(v.w));
      }
      fence_proxy_async_smem();
      mbar_arrive(&sm.wlo);
    }
  } else if (warp >= kStateKWarp0) {
    // ---- k'^T rows into TMEM: thread = TMEM lane = k (warp w % 4 owns lanes
    // 32 (w % 4) ..), columns kColKh + t (hi) and kColKl + t (lo)
    const int q = warp & 3, k = 32 * q + lane;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    for (int c = 0; c < NC; ++c) {
      // row k of the blocked [128 k][64 t] tile: 16 float4, t = 4 m .. 4 m + 3
      const float4 *src = reinterpret_cast<const float4 *>(rec0 + (size_t)c * kRec + kOffKp);
      float row[64];
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const float4 v = __ldcg(src + ((k >> 3) * 16 + m) * 8 + (k & 7));
        row[4 * m] = v.x; row[4 * m + 1] = v.y; row[4 * m + 2] = v.z; row[4 * m + 3] = v.w;
      }
      if (c > 0 && ok && !mbar_wait_ns(&sm.m2, (c - 1) & 1, wns)) ok = false;  // MMA2 of chunk c-1 has read k'^T
      // tcgen05.st is warp-collective: the whole warp stores or none of it
      const bool wok = __all_sync(0xffffffffu, ok);
      umma::fence_after_sync();
#pragma unroll
      for (int j = 0; j < 4 && wok; ++j) {
        float hi[16], lo[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          hi[i] = row[16 * j + i];
          lo[i] = umma::tf32_lo(row[16 * j + i]);
        }
        umma::st_32x32b_x16(tb + lane_base + kColKh + 16 * j, hi);
        umma::st_32x32b_x16(tb + lane_base + kColKl + 16 * j, lo);
      }
      umma::wait_st();
      umma::fence_before_sync();
      mbar_arrive(&sm.kready);
    }
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

  umma::fence_before_sync();
  const int failed = __syncthreads_or(ok ? 0 : 1);
  if (failed && tid == 0) {  // a bounded wait gave up: poison the state, flag the status word
    Sg[col0] = __int_as_float(0x7fc00000);
    atomicOr(p.status, Q35_STATUS_WAIT_TIMEOUT);
  }
  if (warp == 4) umma::tmem_dealloc(tb, kTmemCols);
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

  // Thread 0 issues the copies and MMAs: stages [0, l_issued) have been
  // requested, [0, l_seen) seen complete, m_last is the last committed MMA
  // group.  After a wait that gave up it issues nothing more and, before
  // TMEM is freed, waits (bounded) for what it started.
  int l_issued = 1, l_seen = 0, m_last = -1;
#pragma unroll 1
  for (int st = 0; st < 3; ++st) {
    if (ok && !mbar_wait_ns(&sm.barL, st & 1, p.wait_ns)) ok = false;
    if (ok) l_seen = st + 1;
    if (ok) {  // lo terms
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
    // every thread's lo terms are written; a thread whose wait gave up votes the
    // stage's MMAs off
    const int all_ok = __syncthreads_and(ok ? 1 : 0);
    umma::fence_after_sync();
    if (tid == 0 && all_ok) {
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
      m_last = st;
      // the buffers take the next stage once this stage's MMAs have read them
      if (st < 2) {
        if (ok && !mbar_wait_ns(&sm.barM, st & 1, p.wait_ns)) ok = false;
        if (ok) {
          load_stage(st + 1, l2_policy_evict_first());
          l_issued = st + 2;
        }
      }
    }
    if (!all_ok) ok = false;
  }
  // stage 2 (and so every MMA) complete: the barrier's third phase (parity 0);
  // every thread has passed stage 2's barrier, so phases 0 and 1 are done
  if (ok && !mbar_wait_ns(&sm.barM, 0, p.wait_ns)) ok = false;
  if (tid == 0) {
    for (int j = l_seen; j < l_issued; ++j) (void)mbar_wait_ns(&sm.barL, j & 1, p.wait_ns);
    if (m_last >= 0) (void)mbar_wait_ns(&sm.barM, m_last & 1, p.wait_ns);
  }
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
  umma::fence_before_sync();
  const int failed = __syncthreads_or(ok ? 0 : 1);
  if (failed && nt > 0 && (tid & 127) == 0) {  // a bounded wait gave up: poison, flag the status word
    ob[0] = __int_as_float(0x7fc00000);
    atomicOr(p.status, Q35_STATUS_WAIT_TIMEOUT);
  }
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
  return kWsHeader + (size_t)d->batch * d->num_v_heads * NC * kRec * sizeof(float);
}

int gdn_prefill_launch(const q35_gdn_dims *d, int T, const float *mixed_qkv, const float *z, const float *beta,
                       const float *g, const float *conv_w, const float *norm_w, float *conv_state, int has_prev,
                       float *rec_state, int has_init, float *out, void *ws, size_t ws_bytes, cudaStream_t st) {
  const size_t need = gdn_prefill_workspace_bytes(d, T);
  Q35_REQUIRE(ws != nullptr && ws_bytes >= need && (reinterpret_cast<uintptr_t>(ws) & 15u) == 0, Q35_ERR_WORKSPACE,
              "gdn_prefill: workspace missing, unaligned or too small (need " + std::to_string(need) + " bytes)");
  PrefillParams p;
  p.x = mixed_qkv; p.z = z; p.beta = beta; p.g = g; p.conv_w = conv_w; p.norm_w = norm_w;
  p.conv_state = conv_state; p.rec_state = rec_state; p.out = out;
  p.status = static_cast<uint32_t *>(ws);
  p.ws = reinterpret_cast<float *>(static_cast<unsigned char *>(ws) + kWsHeader);
  p.fault = take_fault(kFaultPrefillState) ? 1 : 0;
  p.wait_ns = p.fault ? kFaultWaitLimitNs : kWaitLimitNs;
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
