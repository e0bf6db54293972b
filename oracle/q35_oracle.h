/*
 * q35_oracle.h -- CPU restatement of the reference's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * kernels in qwen-3.5_b200/csrc.  Only tests/, __graft_entry__.smoke() and the
 * CPU-baseline legs of bench.py may load it.  The product path never calls it.
 *
 * What it restates (reference = inventwithdean/Qwen-3.5, Rust/Burn 0.22.1):
 *   src/text_modules.rs:134-162   causal_conv1d_update (decode conv + SiLU)
 *   src/text_modules.rs:164-182   causal_conv1d_fn     (prefill conv + SiLU)
 *   src/text_modules.rs:531-552   prefill conv-state handling
 *   src/text_modules.rs:184-187   l2norm
 *   src/text_modules.rs:189-363   burn_chunk_gated_delta_rule (WY form)
 *   src/text_modules.rs:365-443   burn_recurrent_gated_delta_rule
 *   src/text_modules.rs:85-117    RMSNormGated
 *   src/text_modules.rs:794-809   RMSNorm (1 + w)
 *   src/text_modules.rs:23-82     TextRotaryEmbedding (cos/sin tables)
 *   src/text_modules.rs:739-774   rotate_half / apply_rotary_pos_emb
 *   src/text_modules.rs:776-792   repeat_kv (as GQA head grouping)
 *   src/text_modules.rs:842-936   Attention::forward core (norms, RoPE, cache
 *                                 append, SDPA, sigmoid gate)
 *   src/kernels.rs:174-247        gate_proj_kernel (decode beta / g)
 *   src/text_modules.rs:578-595   prefill beta / g
 *   src/kernels.rs:103-165        q8_gemv_partial_sum (+ sum reduction)
 *
 * Third-party arithmetic on the path (burn 0.22.1, not vendored in the
 * reference): burn::tensor::module::attention with
 * AttentionModuleOptions::default() is restated as standard scaled dot-product
 * attention (scale 1/sqrt(head_dim), max-subtracted softmax); burn conv1d is
 * restated as grouped cross-correlation (no kernel flip).
 *
 * Parity pinning: the reference ships no tests, fixtures or golden vectors and
 * cannot be compiled here (Rust toolchain absent), so this restatement is pinned
 * against (1) the HF transformers Qwen3.5 torch functions that the reference's
 * Burn code is a line-by-line port of (fixtures + generating script in
 * tests/golden/), (2) hand-derived known answers, and (3) the reference's own
 * implied identity chunked-prefill == token-by-token recurrence.  Against the
 * Burn build itself parity is unpinned.
 *
 * All tensors are row-major f32, shapes given per argument.
 */
#ifndef Q35_ORACLE_H
#define Q35_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

void q35o_set_threads(int n);
int q35o_get_threads(void);

/* --- elementwise / small ops --------------------------------------------- */

/* text_modules.rs:134-162.  x [B,C], conv_state [B,C,K-1] (in/out),
 * w [C,K], y [B,C] = silu(sum_j w[c,j]*win[j]), win = [state..., x]. */
void q35o_conv1d_update(int B, int C, int K, const float *x, float *conv_state,
                        const float *w, float *y);

/* text_modules.rs:164-182 with the caller logic of :531-552.
 * x [B,T,C] (token-major, as produced by in_proj_qkv), conv_state [B,C,K-1]
 * (in: previous state if has_prev else ignored/zeros; out: last K-1 inputs of
 * [prev-or-zero, x]), y [B,T,C]. */
void q35o_conv1d_prefill(int B, int T, int C, int K, const float *x,
                         float *conv_state, int has_prev, const float *w,
                         float *y);

/* text_modules.rs:184-187, rows of length d, in place. */
void q35o_l2norm(int64_t rows, int d, float *x, float eps);

/* text_modules.rs:85-117: y = x * 1/sqrt(mean(x^2)+eps) * w * silu(z). */
void q35o_rmsnorm_gated(int64_t rows, int d, const float *x, const float *z,
                        const float *w, float eps, float *y);

/* text_modules.rs:800-809: x <- x * 1/sqrt(mean(x^2)+eps) * (1 + w). */
void q35o_rmsnorm(int64_t rows, int d, float *x, const float *w, float eps);

/* text_modules.rs:23-82 (text positions: the three MRoPE streams are equal,
 * so the interleaved recomposition is the identity).  pos [N] -> cos,sin
 * [N,rot] = cat(f,f) with f[i] = pos * exp(i*2 * (-ln(theta)/rot)). */
void q35o_rope_tables(int N, const int64_t *pos, int rot, float theta,
                      float *cos_out, float *sin_out);

/* text_modules.rs:754-774 on one head vector x[D] (first rot dims rotated). */
void q35o_apply_rope(int D, int rot, float *x, const float *cos,
                     const float *sin);

/* kernels.rs:174-247 (decode, mode 0) or text_modules.rs:578-595 (prefill,
 * mode 1).  x [N,in_dim], wb/wa [in_dim,H], a_log/dt_bias [H] ->
 * beta [N,H], g [N,H]. */
void q35o_gate_proj(int N, int in_dim, int H, const float *x, const float *wb,
                    const float *wa, const float *a_log, const float *dt_bias,
                    float *beta, float *g, int mode);

/* --- gated delta rule ---------------------------------------------------- */

/* text_modules.rs:365-443 (with use_qk_l2norm_in_kernel).
 * q,k [B,T,Hk,DK]; v [B,T,Hv,DV]; g,beta [B,T,Hv]; S [B,Hv,DK,DV] in/out;
 * out [B,T,Hv,DV].  v-head h uses k-head h/(Hv/Hk) (text_modules.rs:597-615). */
void q35o_recurrent_gdr(int B, int T, int Hk, int Hv, int DK, int DV,
                        const float *q, const float *k, const float *v,
                        const float *g, const float *beta, float *S,
                        float *out);

/* text_modules.rs:189-363, same tensor contract, chunk length `chunk`. */
void q35o_chunk_gdr(int B, int T, int Hk, int Hv, int DK, int DV, int chunk,
                    const float *q, const float *k, const float *v,
                    const float *g, const float *beta, float *S, float *out);

/* --- module-level cores (between the input and output projections) ------- */

/* GatedDeltaNet::forward decode branch (text_modules.rs:515-530, 554-567,
 * 627-636, 651-660).  mixed_qkv [B,C] (C = 2*Hk*DK + Hv*DV), z [B,Hv*DV],
 * beta,g [B,Hv], conv_w [C,K], norm_w [DV], conv_state [B,C,K-1] in/out,
 * S [B,Hv,DK,DV] in/out, out [B,Hv*DV]. */
void q35o_gdn_decode(int B, int Hk, int Hv, int DK, int DV, int K,
                     const float *mixed_qkv, const float *z, const float *beta,
                     const float *g, const float *conv_w, const float *norm_w,
                     float *conv_state, float *S, float *out, float eps);

/* GatedDeltaNet::forward chunked branch (text_modules.rs:531-552, 554-567,
 * 637-660).  mixed_qkv [B,T,C], z [B,T,Hv*DV], beta,g [B,T,Hv];
 * conv_state/S in/out with has_prev / has_init flags; out [B,T,Hv*DV]. */
void q35o_gdn_prefill(int B, int T, int Hk, int Hv, int DK, int DV, int K,
                      int chunk, const float *mixed_qkv, const float *z,
                      const float *beta, const float *g, const float *conv_w,
                      const float *norm_w, float *conv_state, int has_prev,
                      float *S, int has_init, float *out, float eps);

/* Attention::forward decode core (text_modules.rs:866-936).
 * q_gate [B,Hq,2D] (per head [q | gate]), k_new/v_new [B,Hkv,D],
 * qn_w/kn_w [D], cos/sin [B,rot], k_cache/v_cache [B,Hkv,cap,D] (the new
 * k/v are written at lens[b]), lens [B] (valid length before the append;
 * incremented), out [B,Hq*D] = attn * sigmoid(gate). */
void q35o_gqa_decode(int B, int Hq, int Hkv, int D, int rot, int64_t cap,
                     const float *q_gate, const float *k_new,
                     const float *v_new, const float *qn_w, const float *kn_w,
                     const float *cos, const float *sin, float *k_cache,
                     float *v_cache, int32_t *lens, float *out, float eps);

/* The same attention over several query tokens of one prompt (prefill core,
 * causal mask of model.rs:59-67 with past_len = lens[b]).  q_gate [B,T,Hq,2D],
 * k_new/v_new [B,T,Hkv,D], cos/sin [B,T,rot], out [B,T,Hq*D]. */
void q35o_gqa_prefill(int B, int T, int Hq, int Hkv, int D, int rot,
                      int64_t cap, const float *q_gate, const float *k_new,
                      const float *v_new, const float *qn_w, const float *kn_w,
                      const float *cos, const float *sin, float *k_cache,
                      float *v_cache, int32_t *lens, float *out, float eps);

/* kernels.rs:103-165: Q8F split-K GEMV as the reference computes it.
 * x [in_dim]; wq [in_dim, out_dim] int8 (packed 4 per u32 in the reference;
 * here one byte each, same values); scales [in_dim, out_dim/64]; y [out_dim].
 * exact=0 reproduces the reference's row coverage (rows past
 * splits*(chunk/8)*8 are skipped); exact=1 covers every row. */
void q35o_q8_gemv(int in_dim, int out_dim, const float *x, const int8_t *wq,
                  const float *scales, float *y, int exact);

#ifdef __cplusplus
}
#endif
#endif
