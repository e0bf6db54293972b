/*
 * q35_oracle.c -- CPU restatement of the reference's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker, never the product).  Each
 * function cites the reference file:line it restates; the op order follows the
 * reference's Burn tensor program, evaluated in f32 with sequential sums.
 * Pinning and the list of restated functions: see q35_oracle.h.
 */
#include "q35_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 1;

void q35o_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
int q35o_get_threads(void) { return g_threads; }

static inline float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
static inline float siluf_(float x) { return x * sigmoidf_(x); }

/* text_modules.rs:134-162 */
void q35o_conv1d_update(int B, int C, int K, const float *x, float *conv_state,
                        const float *w, float *y) {
  const int SL = K - 1;
#pragma omp parallel for num_threads(g_threads) schedule(static)
  for (int64_t bc = 0; bc < (int64_t)B * C; ++bc) {
    const int c = (int)(bc % C);
    float *st = conv_state + bc * SL;
    float win[16];
    /* cat([conv_state, hidden_states], 2) */
    for (int j = 0; j < SL; ++j) win[j] = st[j];
    win[SL] = x[bc];
    /* conv1d, groups = channels, no padding: one output column */
    float acc = 0.0f;
    for (int j = 0; j < K; ++j) acc += w[(int64_t)c * K + j] * win[j];
    y[bc] = siluf_(acc);
    /* new state = last state_len columns of the concatenation */
    for (int j = 0; j < SL; ++j) st[j] = win[j + 1];
  }
}

/* text_modules.rs:164-182 and the cache handling of :531-552 */
void q35o_conv1d_prefill(int B, int T, int C, int K, const float *x,
                         float *conv_state, int has_prev, const float *w,
                         float *y) {
  const int SL = K - 1;
#pragma omp parallel for num_threads(g_threads) schedule(static)
  for (int64_t bc = 0; bc < (int64_t)B * C; ++bc) {
    const int64_t b = bc / C;
    const int c = (int)(bc % C);
    float *st = conv_state + bc * SL;
    float prev[16];
    for (int j = 0; j < SL; ++j) prev[j] = has_prev ? st[j] : 0.0f;
    /* input column i of the (left-padded) sequence: i < 0 -> prev / zeros */
#define XIN(i) ((i) < 0 ? prev[SL + (i)] : x[((b * T) + (i)) * C + c])
    for (int t = 0; t < T; ++t) {
      float acc = 0.0f;
      for (int j = 0; j < K; ++j) acc += w[(int64_t)c * K + j] * XIN(t - SL + j);
      y[((b * T) + t) * C + c] = siluf_(acc);
    }
    /* conv state <- last K-1 input columns (:538-540) */
    float nst[16];
    for (int j = 0; j < SL; ++j) nst[j] = XIN(T - SL + j);
    for (int j = 0; j < SL; ++j) st[j] = nst[j];
#undef XIN
  }
}

/* text_modules.rs:184-187 */
void q35o_l2norm(int64_t rows, int d, float *x, float eps) {
  for (int64_t r = 0; r < rows; ++r) {
    float *p = x + r * d;
    float ss = 0.0f;
    for (int i = 0; i < d; ++i) ss += p[i] * p[i];
    const float inv = 1.0f / sqrtf(ss + eps);
    for (int i = 0; i < d; ++i) p[i] = p[i] * inv;
  }
}

/* text_modules.rs:85-117 */
void q35o_rmsnorm_gated(int64_t rows, int d, const float *x, const float *z,
                        const float *w, float eps, float *y) {
  for (int64_t r = 0; r < rows; ++r) {
    const float *p = x + r * d;
    float ss = 0.0f;
    for (int i = 0; i < d; ++i) ss += p[i] * p[i];
    const float inv = 1.0f / sqrtf(ss / (float)d + eps);
    for (int i = 0; i < d; ++i)
      y[r * d + i] = (w[i] * (p[i] * inv)) * siluf_(z[r * d + i]);
  }
}

/* text_modules.rs:800-809 */
void q35o_rmsnorm(int64_t rows, int d, float *x, const float *w, float eps) {
  for (int64_t r = 0; r < rows; ++r) {
    float *p = x + r * d;
    float ss = 0.0f;
    for (int i = 0; i < d; ++i) ss += p[i] * p[i];
    const float inv = 1.0f / sqrtf(ss / (float)d + eps);
    for (int i = 0; i < d; ++i) p[i] = (p[i] * inv) * (1.0f + w[i]);
  }
}

/* text_modules.rs:30-58, 73-81 */
void q35o_rope_tables(int N, const int64_t *pos, int rot, float theta,
                      float *cos_out, float *sin_out) {
  const int half = rot / 2;
  const float scaling = -logf(theta) / (float)rot;
  for (int n = 0; n < N; ++n) {
    for (int i = 0; i < half; ++i) {
      const float inv_freq = expf((float)(2 * i) * scaling);
      const float f = (float)pos[n] * inv_freq;
      const float c = cosf(f), s = sinf(f);
      cos_out[(int64_t)n * rot + i] = c;
      cos_out[(int64_t)n * rot + half + i] = c;
      sin_out[(int64_t)n * rot + i] = s;
      sin_out[(int64_t)n * rot + half + i] = s;
    }
  }
}

/* text_modules.rs:739-774: x_rot*cos + rotate_half(x_rot)*sin on [0,rot) */
void q35o_apply_rope(int D, int rot, float *x, const float *cos,
                     const float *sin) {
  (void)D;
  const int half = rot / 2;
  float tmp[1024];
  for (int i = 0; i < rot; ++i) {
    const float rh = i < half ? -x[i + half] : x[i - half];
    tmp[i] = x[i] * cos[i] + rh * sin[i];
  }
  for (int i = 0; i < rot; ++i) x[i] = tmp[i];
}

/* kernels.rs:174-247 (mode 0: 8 splits, partial sums summed in split order;
 * softplus threshold tested on the post-softplus value, :238-243) and
 * text_modules.rs:578-595 (mode 1: plain matmul; threshold on a+dt_bias). */
void q35o_gate_proj(int N, int in_dim, int H, const float *x, const float *wb,
                    const float *wa, const float *a_log, const float *dt_bias,
                    float *beta, float *g, int mode) {
  for (int n = 0; n < N; ++n) {
    const float *xr = x + (int64_t)n * in_dim;
    for (int h = 0; h < H; ++h) {
      float bsum = 0.0f, asum = 0.0f;
      if (mode == 0) {
        const int splits = 8, u = 8;
        const int chunk = in_dim / splits;
        for (int s = 0; s < splits; ++s) {
          float pb = 0.0f, pa = 0.0f;
          for (int blk = 0; blk < chunk / u; ++blk)
            for (int j = 0; j < u; ++j) {
              const int row = s * chunk + blk * u + j;
              pb += xr[row] * wb[(int64_t)row * H + h];
              pa += xr[row] * wa[(int64_t)row * H + h];
            }
          bsum += pb;
          asum += pa;
        }
        const float xg = asum + dt_bias[h];
        const float pre = logf(expf(xg) + 1.0f);
        const float sp = pre > 20.0f ? xg : pre;
        beta[(int64_t)n * H + h] = 1.0f / (1.0f + expf(-bsum));
        g[(int64_t)n * H + h] = -expf(a_log[h]) * sp;
      } else {
        for (int row = 0; row < in_dim; ++row) {
          bsum += xr[row] * wb[(int64_t)row * H + h];
          asum += xr[row] * wa[(int64_t)row * H + h];
        }
        const float xg = asum + dt_bias[h];
        const float sp = xg > 20.0f ? xg : logf(expf(xg) + 1.0f);
        beta[(int64_t)n * H + h] = sigmoidf_(bsum);
        g[(int64_t)n * H + h] = -expf(a_log[h]) * sp;
      }
    }
  }
}

/* text_modules.rs:365-443 */
void q35o_recurrent_gdr(int B, int T, int Hk, int Hv, int DK, int DV,
                        const float *q, const float *k, const float *v,
                        const float *g, const float *beta, float *S,
                        float *out) {
  const int rf = Hv / Hk;
  const float scale = powf((float)DK, -0.5f);
#pragma omp parallel for num_threads(g_threads) schedule(dynamic, 1)
  for (int64_t bh = 0; bh < (int64_t)B * Hv; ++bh) {
    const int64_t b = bh / Hv;
    const int h = (int)(bh % Hv), hk = h / rf;
    float *St = S + bh * DK * DV;
    float *qt = (float *)malloc(sizeof(float) * (DK * 2 + DV * 2));
    float *kt = qt + DK, *kv = kt + DK, *delta = kv + DV;
    for (int t = 0; t < T; ++t) {
      const int64_t tok = b * T + t;
      memcpy(qt, q + (tok * Hk + hk) * DK, sizeof(float) * DK);
      memcpy(kt, k + (tok * Hk + hk) * DK, sizeof(float) * DK);
      q35o_l2norm(1, DK, qt, 1e-6f);
      q35o_l2norm(1, DK, kt, 1e-6f);
      for (int i = 0; i < DK; ++i) qt[i] *= scale;
      const float *vt = v + (tok * Hv + h) * DV;
      const float dec = expf(g[tok * Hv + h]);
      const float bt = beta[tok * Hv + h];
      /* S = S * exp(g) */
      for (int64_t i = 0; i < (int64_t)DK * DV; ++i) St[i] *= dec;
      /* kv_mem = sum_k S[k][v] * k[k] */
      for (int j = 0; j < DV; ++j) kv[j] = 0.0f;
      for (int i = 0; i < DK; ++i)
        for (int j = 0; j < DV; ++j) kv[j] += St[(int64_t)i * DV + j] * kt[i];
      /* delta = (v - kv_mem) * beta ; S += k delta^T */
      for (int j = 0; j < DV; ++j) delta[j] = (vt[j] - kv[j]) * bt;
      for (int i = 0; i < DK; ++i)
        for (int j = 0; j < DV; ++j) St[(int64_t)i * DV + j] += kt[i] * delta[j];
      /* out = sum_k S[k][v] * q[k] */
      float *o = out + (tok * Hv + h) * DV;
      for (int j = 0; j < DV; ++j) o[j] = 0.0f;
      for (int i = 0; i < DK; ++i)
        for (int j = 0; j < DV; ++j) o[j] += St[(int64_t)i * DV + j] * qt[i];
    }
    free(qt);
  }
}

/* text_modules.rs:189-363 */
void q35o_chunk_gdr(int B, int T, int Hk, int Hv, int DK, int DV, int C,
                    const float *q, const float *k, const float *v,
                    const float *g, const float *beta, float *S, float *out) {
  const int rf = Hv / Hk;
  const float scale = powf((float)DK, -0.5f);
  const int pad = (C - T % C) % C;
  const int Tp = T + pad, NC = Tp / C;
#pragma omp parallel for num_threads(g_threads) schedule(dynamic, 1)
  for (int64_t bh = 0; bh < (int64_t)B * Hv; ++bh) {
    const int64_t b = bh / Hv;
    const int h = (int)(bh % Hv), hk = h / rf;
    float *St = S + bh * DK * DV;
    /* per-chunk working set */
    float *qc = (float *)calloc((size_t)C * DK, sizeof(float));
    float *kc = (float *)calloc((size_t)C * DK, sizeof(float));
    float *kb = (float *)calloc((size_t)C * DK, sizeof(float));
    float *vb = (float *)calloc((size_t)C * DV, sizeof(float));
    float *gam = (float *)calloc((size_t)C, sizeof(float));
    float *Dm = (float *)calloc((size_t)C * C, sizeof(float));
    float *A = (float *)calloc((size_t)C * C, sizeof(float));
    float *Aqk = (float *)calloc((size_t)C * C, sizeof(float));
    float *row = (float *)calloc((size_t)C, sizeof(float));
    float *U = (float *)calloc((size_t)C * DV, sizeof(float));
    float *W = (float *)calloc((size_t)C * DK, sizeof(float));
    float *vn = (float *)calloc((size_t)C * DV, sizeof(float));
    float *Sn = (float *)calloc((size_t)DK * DV, sizeof(float));
    for (int c = 0; c < NC; ++c) {
      /* load, l2norm (:218-219), scale (:221-222), zero padding (:224-236) */
      float bt[256];
      for (int i = 0; i < C; ++i) {
        const int t = c * C + i;
        if (t < T) {
          const int64_t tok = b * T + t;
          memcpy(qc + (int64_t)i * DK, q + (tok * Hk + hk) * DK, sizeof(float) * DK);
          memcpy(kc + (int64_t)i * DK, k + (tok * Hk + hk) * DK, sizeof(float) * DK);
          q35o_l2norm(1, DK, qc + (int64_t)i * DK, 1e-6f);
          q35o_l2norm(1, DK, kc + (int64_t)i * DK, 1e-6f);
          for (int d = 0; d < DK; ++d) qc[(int64_t)i * DK + d] *= scale;
          bt[i] = beta[tok * Hv + h];
          gam[i] = g[tok * Hv + h];
          const float *vt = v + (tok * Hv + h) * DV;
          for (int d = 0; d < DV; ++d) vb[(int64_t)i * DV + d] = vt[d] * bt[i];
        } else {
          memset(qc + (int64_t)i * DK, 0, sizeof(float) * DK);
          memset(kc + (int64_t)i * DK, 0, sizeof(float) * DK);
          memset(vb + (int64_t)i * DV, 0, sizeof(float) * DV);
          bt[i] = 0.0f;
          gam[i] = 0.0f;
        }
        /* k_beta = key * beta (:247) */
        for (int d = 0; d < DK; ++d) kb[(int64_t)i * DK + d] = kc[(int64_t)i * DK + d] * bt[i];
      }
      /* cum_decay = cumsum(decay) (:255) */
      for (int i = 1; i < C; ++i) gam[i] = gam[i] + gam[i - 1];
      /* pairwise_decay = exp(gi - gj), -inf (-> 0) above the diagonal (:259-265) */
      for (int i = 0; i < C; ++i)
        for (int j = 0; j < C; ++j)
          Dm[i * C + j] = j <= i ? expf(gam[i] - gam[j]) : 0.0f;
      /* ut_system = (k_beta @ key^T) * decay; intra = (q @ k^T) * decay (:269-273) */
      for (int i = 0; i < C; ++i)
        for (int j = 0; j < C; ++j) {
          float s1 = 0.0f, s2 = 0.0f;
          for (int d = 0; d < DK; ++d) {
            s1 += kb[(int64_t)i * DK + d] * kc[(int64_t)j * DK + d];
            s2 += qc[(int64_t)i * DK + d] * kc[(int64_t)j * DK + d];
          }
          A[i * C + j] = s1 * Dm[i * C + j];
          Aqk[i * C + j] = s2 * Dm[i * C + j];
        }
      /* ut_system = -tril(ut_system, -1) (:279) */
      for (int i = 0; i < C; ++i)
        for (int j = 0; j < C; ++j) A[i * C + j] = j < i ? -A[i * C + j] : 0.0f;
      /* row recursion (:280-287): A[i,:i] = row + row @ A[:i,:i] */
      for (int i = 1; i < C; ++i) {
        for (int j = 0; j < i; ++j) row[j] = A[i * C + j];
        for (int j = 0; j < i; ++j) {
          float s = 0.0f;
          for (int m = 0; m < i; ++m) s += row[m] * A[m * C + j];
          A[i * C + j] = row[j] + s;
        }
      }
      /* + I (:289-290) */
      for (int i = 0; i < C; ++i) A[i * C + i] += 1.0f;
      /* new_values = T @ v_beta; k_cumdecay = T @ (k_beta * exp(g)) (:292-293) */
      for (int i = 0; i < C; ++i) {
        for (int d = 0; d < DV; ++d) {
          float s = 0.0f;
          for (int j = 0; j < C; ++j) s += A[i * C + j] * vb[(int64_t)j * DV + d];
          U[(int64_t)i * DV + d] = s;
        }
        for (int d = 0; d < DK; ++d) {
          float s = 0.0f;
          for (int j = 0; j < C; ++j)
            s += A[i * C + j] * (kb[(int64_t)j * DK + d] * expf(gam[j]));
          W[(int64_t)i * DK + d] = s;
        }
      }
      /* query *= exp(cum_decay); key *= exp(last - cum) (:303-311) */
      const float glast = gam[C - 1];
      for (int i = 0; i < C; ++i) {
        const float eq = expf(gam[i]), ek = expf(glast - gam[i]);
        for (int d = 0; d < DK; ++d) {
          qc[(int64_t)i * DK + d] *= eq;
          kc[(int64_t)i * DK + d] *= ek;
        }
      }
      const float cdec = expf(glast);
      /* v_new = new_values - k_cumdecay @ S (:315-324) */
      for (int i = 0; i < C; ++i)
        for (int d = 0; d < DV; ++d) {
          float s = 0.0f;
          for (int j = 0; j < DK; ++j) s += W[(int64_t)i * DK + j] * St[(int64_t)j * DV + d];
          vn[(int64_t)i * DV + d] = U[(int64_t)i * DV + d] - s;
        }
      /* out = (q*exp(g)) @ S + intra @ v_new (:325-341) */
      for (int i = 0; i < C; ++i) {
        const int t = c * C + i;
        for (int d = 0; d < DV; ++d) {
          float s1 = 0.0f, s2 = 0.0f;
          for (int j = 0; j < DK; ++j) s1 += qc[(int64_t)i * DK + j] * St[(int64_t)j * DV + d];
          for (int j = 0; j < C; ++j) s2 += Aqk[i * C + j] * vn[(int64_t)j * DV + d];
          if (t < T) out[((b * T + t) * Hv + h) * DV + d] = s1 + s2;
        }
      }
      /* S = S * exp(g_last) + (key*exp(last-g))^T @ v_new (:342-349) */
      for (int j = 0; j < DK; ++j)
        for (int d = 0; d < DV; ++d) {
          float s = 0.0f;
          for (int i = 0; i < C; ++i) s += kc[(int64_t)i * DK + j] * vn[(int64_t)i * DV + d];
          Sn[(int64_t)j * DV + d] = St[(int64_t)j * DV + d] * cdec + s;
        }
      memcpy(St, Sn, sizeof(float) * DK * DV);
    }
    free(qc); free(kc); free(kb); free(vb); free(gam); free(Dm); free(A);
    free(Aqk); free(row); free(U); free(W); free(vn); free(Sn);
  }
}

/* split of mixed_qkv into q|k|v and reshape (text_modules.rs:554-567) */
static void split_qkv(int64_t N, int Hk, int Hv, int DK, int DV, const float *y,
                      float *q, float *k, float *v) {
  const int kd = Hk * DK, vd = Hv * DV, C = 2 * kd + vd;
  for (int64_t n = 0; n < N; ++n) {
    memcpy(q + n * kd, y + n * C, sizeof(float) * kd);
    memcpy(k + n * kd, y + n * C + kd, sizeof(float) * kd);
    memcpy(v + n * vd, y + n * C + 2 * kd, sizeof(float) * vd);
  }
}

void q35o_gdn_decode(int B, int Hk, int Hv, int DK, int DV, int K,
                     const float *mixed_qkv, const float *z, const float *beta,
                     const float *g, const float *conv_w, const float *norm_w,
                     float *conv_state, float *S, float *out, float eps) {
  const int kd = Hk * DK, vd = Hv * DV, C = 2 * kd + vd;
  float *y = (float *)malloc(sizeof(float) * (size_t)B * C);
  float *q = (float *)malloc(sizeof(float) * (size_t)B * kd);
  float *k = (float *)malloc(sizeof(float) * (size_t)B * kd);
  float *v = (float *)malloc(sizeof(float) * (size_t)B * vd);
  float *core = (float *)malloc(sizeof(float) * (size_t)B * vd);
  q35o_conv1d_update(B, C, K, mixed_qkv, conv_state, conv_w, y);
  split_qkv(B, Hk, Hv, DK, DV, y, q, k, v);
  q35o_recurrent_gdr(B, 1, Hk, Hv, DK, DV, q, k, v, g, beta, S, core);
  q35o_rmsnorm_gated((int64_t)B * Hv, DV, core, z, norm_w, eps, out);
  free(y); free(q); free(k); free(v); free(core);
}

void q35o_gdn_prefill(int B, int T, int Hk, int Hv, int DK, int DV, int K,
                      int chunk, const float *mixed_qkv, const float *z,
                      const float *beta, const float *g, const float *conv_w,
                      const float *norm_w, float *conv_state, int has_prev,
                      float *S, int has_init, float *out, float eps) {
  const int kd = Hk * DK, vd = Hv * DV, C = 2 * kd + vd;
  const int64_t N = (int64_t)B * T;
  float *y = (float *)malloc(sizeof(float) * (size_t)N * C);
  float *q = (float *)malloc(sizeof(float) * (size_t)N * kd);
  float *k = (float *)malloc(sizeof(float) * (size_t)N * kd);
  float *v = (float *)malloc(sizeof(float) * (size_t)N * vd);
  float *core = (float *)malloc(sizeof(float) * (size_t)N * vd);
  q35o_conv1d_prefill(B, T, C, K, mixed_qkv, conv_state, has_prev, conv_w, y);
  split_qkv(N, Hk, Hv, DK, DV, y, q, k, v);
  if (!has_init) memset(S, 0, sizeof(float) * (size_t)B * Hv * DK * DV);
  q35o_chunk_gdr(B, T, Hk, Hv, DK, DV, chunk, q, k, v, g, beta, S, core);
  q35o_rmsnorm_gated(N * Hv, DV, core, z, norm_w, eps, out);
  free(y); free(q); free(k); free(v); free(core);
}

/* Attention core for T query tokens of sequence b at positions
 * lens[b] .. lens[b]+T-1 (text_modules.rs:866-936; causal mask model.rs:59-67). */
static void gqa_core(int B, int T, int Hq, int Hkv, int D, int rot, int64_t cap,
                     const float *q_gate, const float *k_new, const float *v_new,
                     const float *qn_w, const float *kn_w, const float *cos,
                     const float *sin, float *k_cache, float *v_cache,
                     int32_t *lens, float *out, float eps) {
  const int grp = Hq / Hkv;
  const float scale = 1.0f / sqrtf((float)D);
  /* k_norm + RoPE, then cache append (:877-909), every sequence first */
#pragma omp parallel for num_threads(g_threads) schedule(static)
  for (int b = 0; b < B; ++b) {
    const int64_t L0 = lens[b];
    for (int t = 0; t < T; ++t) {
      const int64_t tok = (int64_t)b * T + t;
      for (int kh = 0; kh < Hkv; ++kh) {
        float *kd = k_cache + (((int64_t)b * Hkv + kh) * cap + L0 + t) * D;
        float *vd = v_cache + (((int64_t)b * Hkv + kh) * cap + L0 + t) * D;
        memcpy(kd, k_new + (tok * Hkv + kh) * D, sizeof(float) * D);
        memcpy(vd, v_new + (tok * Hkv + kh) * D, sizeof(float) * D);
        q35o_rmsnorm(1, D, kd, kn_w, eps);
        q35o_apply_rope(D, rot, kd, cos + tok * rot, sin + tok * rot);
      }
    }
  }
  /* attention of every (sequence, token, query head), independently */
#pragma omp parallel for num_threads(g_threads) schedule(dynamic, 1)
  for (int64_t bth = 0; bth < (int64_t)B * T * Hq; ++bth) {
    const int b = (int)(bth / ((int64_t)T * Hq));
    const int64_t th = bth % ((int64_t)T * Hq);
    const int t = (int)(th / Hq), h = (int)(th % Hq), kh = h / grp;
    const int64_t L0 = lens[b];
    const int64_t tok = (int64_t)b * T + t;
    const int64_t Lk = L0 + t + 1; /* causal: keys 0 .. L0+t */
    float *qv = (float *)malloc(sizeof(float) * (D * 2 + (size_t)Lk));
    float *o = qv + D, *sc = o + D;
    const float *qg = q_gate + (tok * Hq + h) * 2 * D;
    memcpy(qv, qg, sizeof(float) * D);
    q35o_rmsnorm(1, D, qv, qn_w, eps);
    q35o_apply_rope(D, rot, qv, cos + tok * rot, sin + tok * rot);
    const float *Kc = k_cache + ((int64_t)b * Hkv + kh) * cap * D;
    const float *Vc = v_cache + ((int64_t)b * Hkv + kh) * cap * D;
    float mx = -INFINITY;
    for (int64_t j = 0; j < Lk; ++j) {
      float s = 0.0f;
      for (int d = 0; d < D; ++d) s += qv[d] * Kc[j * D + d];
      sc[j] = s * scale;
      if (sc[j] > mx) mx = sc[j];
    }
    float den = 0.0f;
    for (int64_t j = 0; j < Lk; ++j) {
      sc[j] = expf(sc[j] - mx);
      den += sc[j];
    }
    for (int d = 0; d < D; ++d) o[d] = 0.0f;
    for (int64_t j = 0; j < Lk; ++j) {
      const float p = sc[j] / den;
      for (int d = 0; d < D; ++d) o[d] += p * Vc[j * D + d];
    }
    /* attn_output * sigmoid(gate) (:936) */
    for (int d = 0; d < D; ++d)
      out[(tok * Hq + h) * D + d] = o[d] * sigmoidf_(qg[D + d]);
    free(qv);
  }
  for (int b = 0; b < B; ++b) lens[b] = (int32_t)(lens[b] + T);
}

void q35o_gqa_decode(int B, int Hq, int Hkv, int D, int rot, int64_t cap,
                     const float *q_gate, const float *k_new,
                     const float *v_new, const float *qn_w, const float *kn_w,
                     const float *cos, const float *sin, float *k_cache,
                     float *v_cache, int32_t *lens, float *out, float eps) {
  gqa_core(B, 1, Hq, Hkv, D, rot, cap, q_gate, k_new, v_new, qn_w, kn_w, cos,
           sin, k_cache, v_cache, lens, out, eps);
}

void q35o_gqa_prefill(int B, int T, int Hq, int Hkv, int D, int rot,
                      int64_t cap, const float *q_gate, const float *k_new,
                      const float *v_new, const float *qn_w, const float *kn_w,
                      const float *cos, const float *sin, float *k_cache,
                      float *v_cache, int32_t *lens, float *out, float eps) {
  gqa_core(B, T, Hq, Hkv, D, rot, cap, q_gate, k_new, v_new, qn_w, kn_w, cos,
           sin, k_cache, v_cache, lens, out, eps);
}

/* kernels.rs:103-165 and the launch arithmetic of :495-537 */
void q35o_q8_gemv(int in_dim, int out_dim, const float *x, const int8_t *wq,
                  const float *scales, float *y, int exact) {
  int splits = 25000 / out_dim;
  int hi = in_dim / 80 > 1 ? in_dim / 80 : 1;
  if (splits < 1) splits = 1;
  if (splits > hi) splits = hi;
  const int chunk = in_dim / splits, u = 8, nsc = out_dim / 64;
  for (int pos = 0; pos < out_dim; ++pos) {
    float acc = 0.0f;
    for (int s = 0; s < splits; ++s) {
      float part = 0.0f;
      const int r0 = s * chunk;
      const int rows = exact ? (s == splits - 1 ? in_dim - r0 : chunk) : (chunk / u) * u;
      for (int i = r0; i < r0 + rows; ++i)
        part += (float)wq[(int64_t)i * out_dim + pos] * x[i] *
                scales[(int64_t)i * nsc + pos / 64];
      acc += part;
    }
    y[pos] = acc;
  }
}
