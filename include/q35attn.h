/*
 * q35attn.h -- C ABI of the B200 (sm_100a) attention hot path for the Qwen3.5
 * hybrid decoder (Gated DeltaNet linear attention + gated GQA full attention).
 *
 * Drop-in boundary: each entry point replaces the tensor program between the
 * input projections and the output projection of one reference module
 * (inventwithdean/Qwen-3.5, src/text_modules.rs).  Plain pointers and sizes
 * only; every pointer argument is a DEVICE pointer unless stated otherwise;
 * `stream` is a cudaStream_t (NULL = legacy default stream).  All tensors are
 * row-major float32 (the reference casts weights to F32 at load, main.rs:166,
 * and keeps state/cache in f32, text_config.rs:112).
 *
 * Ownership: the caller owns every buffer.  Hot-path entry points never
 * allocate; where scratch is needed the caller passes a workspace sized by the
 * matching *_workspace_size query.  State and caches are updated in place.
 *
 * Errors: every entry point returns Q35_OK (0) or a Q35_ERR_* code and never
 * aborts (the reference panics instead, kernels.rs:442,472,580).
 * q35_last_error() returns a thread-local message for the last failure.
 * Conditions only the device can see (a cache that is full) are reported
 * through a status word in the workspace, read with q35_workspace_status().
 *
 * Threading: calls are stream-ordered and asynchronous.  Concurrent calls are
 * safe when they touch disjoint buffers (including disjoint workspaces).
 */
#ifndef Q35ATTN_H
#define Q35ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define Q35_OK 0
#define Q35_ERR_INVALID_ARG 1       /* null pointer, negative size, bad flag */
#define Q35_ERR_UNSUPPORTED 2       /* shape outside the compiled kernel set */
#define Q35_ERR_CAPACITY 3          /* KV cache capacity exceeded (host-visible) */
#define Q35_ERR_WORKSPACE 4         /* workspace missing or too small */
#define Q35_ERR_CUDA 5              /* CUDA runtime error (launch / config) */
#define Q35_ERR_DEVICE 6            /* no usable sm_100 device */

/* Device-side status bits (q35_workspace_status). */
#define Q35_STATUS_CACHE_FULL 0x1u    /* lens[b] >= capacity: step skipped for b */
#define Q35_STATUS_LEN_HINT 0x2u      /* lens[b]+1 > max_len hint: step skipped for b */
#define Q35_STATUS_WAIT_TIMEOUT 0x4u  /* a bounded in-kernel wait gave up */

/* Gated DeltaNet layer shapes (text_config.rs:95-99, text_modules.rs:670-699).
 * Qwen3.5-2B: {B, 16, 16, 128, 128, 4, 1e-6}. */
typedef struct q35_gdn_dims {
  int32_t batch;        /* B: independent sequences */
  int32_t num_k_heads;  /* linear_num_key_heads */
  int32_t num_v_heads;  /* linear_num_value_heads (multiple of num_k_heads) */
  int32_t head_k_dim;   /* linear_key_head_dim   (128 supported) */
  int32_t head_v_dim;   /* linear_value_head_dim (128 supported) */
  int32_t conv_kernel;  /* linear_conv_kernel_dim (2..4 supported) */
  float eps;            /* rms_norm_eps of the gated output norm */
} q35_gdn_dims;

/* Gated GQA full-attention shapes (text_config.rs:65,105-108,121-122).
 * Qwen3.5-2B: {B, 8, 2, 256, 64, cap, 1e-6}. */
typedef struct q35_gqa_dims {
  int32_t batch;         /* B */
  int32_t num_q_heads;   /* num_attention_heads */
  int32_t num_kv_heads;  /* num_key_value_heads (divides num_q_heads, group <= 8) */
  int32_t head_dim;      /* 256 supported */
  int32_t rotary_dim;    /* head_dim * partial_rotary_factor (even, <= head_dim) */
  int32_t reserved;
  int64_t capacity;      /* token capacity of the K/V cache per (sequence, kv head) */
  float eps;             /* rms_norm_eps of q_norm / k_norm */
} q35_gqa_dims;

/* --------------------------------------------------------------------------
 * Gated DeltaNet, one decode step (seq_len == 1, conv state present).
 * Replaces text_modules.rs:515-530 (causal_conv1d_update + SiLU), :554-567
 * (q/k/v split), :597-615 (k-head expansion), :627-636
 * (burn_recurrent_gated_delta_rule, :365-443) and :651-660 (RMSNormGated,
 * :85-117) -- everything between in_proj_* and out_proj of
 * GatedDeltaNet::forward (:483-667).
 *   mixed_qkv  [B, C]      in_proj_qkv output, C = 2*Hk*DK + Hv*DV
 *   z          [B, Hv*DV]  in_proj_z output (gate of the output norm)
 *   beta, g    [B, Hv]     sigmoid(b) and -exp(A_log)*softplus(a+dt_bias)
 *   conv_w     [C, K]      depthwise conv weight (Conv1d [C,1,K] squeezed)
 *   norm_w     [DV]        RMSNormGated weight
 *   conv_state [B, C, K-1] in/out (cache.conv_states[l])
 *   rec_state  [B, Hv, DK, DV] in/out, [head][k][v] (cache.recurrent_states[l])
 *   out        [B, Hv*DV]  input of out_proj
 */
int q35_gdn_decode(const q35_gdn_dims *dims, const float *mixed_qkv,
                   const float *z, const float *beta, const float *g,
                   const float *conv_w, const float *norm_w, float *conv_state,
                   float *rec_state, float *out, void *stream);

/* --------------------------------------------------------------------------
 * Gated DeltaNet chunked prefill (seq_len = T tokens per sequence).
 * Replaces text_modules.rs:531-552 (causal_conv1d_fn, :164-182, with the
 * conv-state capture), :554-615 and :637-660 (burn_chunk_gated_delta_rule,
 * :189-363, chunk 64, then RMSNormGated).
 *   mixed_qkv [B, T, C], z [B, T, Hv*DV], beta/g [B, T, Hv], out [B, T, Hv*DV]
 *   conv_state [B, C, K-1]: read when has_prev_conv (prepended history,
 *              :535-537), always overwritten with the last K-1 inputs.
 *   rec_state  [B, Hv, DK, DV]: initial state when has_init_state, else zero;
 *              overwritten with the final state.
 *   workspace  >= q35_gdn_prefill_workspace_size(dims, T) bytes, 16-byte
 *              aligned.  Its first 256 bytes hold the status word
 *              (Q35_STATUS_WAIT_TIMEOUT when a bounded in-kernel wait gave
 *              up; the state and outputs then hold NaN), read and cleared
 *              with q35_workspace_status.  Zero them once with
 *              q35_workspace_init(workspace, 256, stream) before first use.
 *   mixed_qkv, z, norm_w, rec_state and out must be 16-byte aligned.
 */
size_t q35_gdn_prefill_workspace_size(const q35_gdn_dims *dims, int32_t seq_len);
int q35_gdn_prefill(const q35_gdn_dims *dims, int32_t seq_len,
                    const float *mixed_qkv, const float *z, const float *beta,
                    const float *g, const float *conv_w, const float *norm_w,
                    float *conv_state, int32_t has_prev_conv, float *rec_state,
                    int32_t has_init_state, float *out, void *workspace,
                    size_t workspace_bytes, void *stream);

/* --------------------------------------------------------------------------
 * beta / g gate projection.  mode 0 replaces kernels.rs:174-247
 * (gate_proj_kernel: 8-way split partial sums, softplus threshold tested on
 * the softplus value, called at text_modules.rs:569-576); mode 1 replaces the
 * prefill branch text_modules.rs:578-595 (threshold on a + dt_bias).
 *   x [N, in_dim]; w_b, w_a [in_dim, H] (f32, not quantized, main.rs:205-218);
 *   a_log, dt_bias [H]; beta, g [N, H].
 */
int q35_gdn_gate(int32_t n_rows, int32_t in_dim, int32_t num_heads,
                 const float *x, const float *w_b, const float *w_a,
                 const float *a_log, const float *dt_bias, float *beta,
                 float *g, int32_t mode, void *stream);

/* --------------------------------------------------------------------------
 * Q8F split-K GEMV y = x^T W, the decode projections of both layer types.
 * Replaces q8_gemv_partial_sum_kernel + q8_gemv_sum_reduction_kernel
 * (kernels.rs:103-165; host side :495-537, called from text_modules.rs:498,
 * 505, 662, 856, 877, 886, 939, 1003-1005).
 *   x       [in_dim] f32
 *   w       [in_dim, out_dim/4] u32: byte j (little-endian) of word c is the
 *           int8 weight of column 4c + j
 *   scales  [in_dim, out_dim/64] f32, one per (input row, 64-column block)
 *   y       [out_dim] f32
 *   mode    0: every input row.  1: only the rows the reference's kernel
 *           covers (per split s: rows s*chunk .. s*chunk + (chunk/8)*8 - 1,
 *           chunk = in_dim/splits, splits = clamp(25000/out_dim, 1,
 *           max(in_dim/80, 1)); kernels.rs:119-131, :504).
 * out_dim must be a multiple of 64; w must be 16-byte aligned.  No workspace:
 * the split-K partial sums are added inside a thread-block cluster.
 */
int q35_q8_gemv(int32_t in_dim, int32_t out_dim, const float *x,
                const uint32_t *w, const float *scales, float *y,
                int32_t mode, void *stream);

/* One Q8F projection of a fused GEMV launch (layout as for q35_q8_gemv). */
typedef struct {
  const uint32_t *w;     /* [in_dim, out_dim/4] u32, 16-byte aligned */
  const float *scales;   /* [in_dim, out_dim/64] f32, 16-byte aligned */
  float *y;              /* [out_dim] f32 */
  int32_t out_dim;       /* multiple of 256 */
} q35_q8_segment;

/* Up to four Q8F GEMVs of the same input in one launch, with the decoder's
 * RMSNorm optionally fused in front and the MLP's SwiGLU optionally behind.
 * Replaces, per decoder layer (text_modules.rs:1053-1085), the input or
 * post-attention RMSNorm (:800-809) followed by the projections that read its
 * output: the GatedDeltaNet in_proj_qkvz pair (:498, :505), the attention
 * q/k/v projections (:856, :877, :886) or the MLP up/gate pair (:1003-1005).
 *   x         [in_dim] f32, 16-byte aligned
 *   norm_w    NULL: the segments read x as it is.  Else [in_dim]: the input is
 *             h / sqrt(mean(h^2) + eps) * (1 + norm_w), h = x (+ residual).
 *   residual  NULL or [in_dim] (needs norm_w); sum_out, x_out: NULL or [in_dim]
 *             receive h and the normalised input (need norm_w; must not
 *             alias x or residual).
 *   swiglu    1: exactly two segments (up, gate) of equal out_dim; segment
 *             0's y receives up * silu(gate) and segment 1's y is unused.
 *   mode      row coverage per segment, as for q35_q8_gemv.
 * in_dim % 4 == 0 and at most 8192 with the norm (16384 without).
 */
int q35_q8_gemv_fused(int32_t in_dim, int32_t n_seg, const q35_q8_segment *segs,
                      const float *x, const float *residual, const float *norm_w,
                      float eps, float *sum_out, float *x_out, int32_t swiglu,
                      int32_t mode, void *stream);

/* --------------------------------------------------------------------------
 * Q8F projections of a prompt: y[n_rows, out_dim] = x[n_rows, in_dim] W with
 * W[k][n] = q[k][n] * scales[k][n/64] rounded to f32, the dense weight that
 * Linear::forward multiplies with at seq_len > 1 (text_modules.rs:499-506,
 * 663, 858-888, 941, 1007-1009).  Same weight layout as q35_q8_gemv; the
 * int8 tiles are dequantised in shared memory (no dense copy of W) and the
 * products run on the tensor cores as bf16 hi/lo splits with f32
 * accumulation (relative error near 2^-16 per product).
 *   workspace  >= q35_q8_gemm_workspace_size(n_rows, in_dim) bytes (x split
 *              into its bf16 terms), 16-byte aligned; reused by every call.
 * in_dim % 32 == 0, every out_dim % 256 == 0, x and every w / scales / y
 * 16-byte aligned.  A bounded wait that gives up sets Q35_STATUS_WAIT_TIMEOUT
 * in the device status word (q35_device_status). */
size_t q35_q8_gemm_workspace_size(int32_t n_rows, int32_t in_dim);
int q35_q8_gemm(int32_t n_rows, int32_t in_dim, int32_t out_dim, const float *x,
                const uint32_t *w, const float *scales, float *y,
                void *workspace, size_t workspace_bytes, void *stream);

/* Up to four Q8F projections of the same prompt rows in one launch (the
 * GatedDeltaNet in_proj_qkv / in_proj_z pair, :499-506; attention q / k / v,
 * :858-888), or with swiglu = 1 exactly two (up, gate) of equal out_dim
 * whose result up * silu(gate) goes to segs[0].y (the MLP, :1007-1009;
 * segs[1].y is unused).  Layouts and limits as for q35_q8_gemm. */
int q35_q8_gemm_fused(int32_t n_rows, int32_t in_dim, int32_t n_seg,
                      const q35_q8_segment *segs, const float *x, int32_t swiglu,
                      void *workspace, size_t workspace_bytes, void *stream);

/* --------------------------------------------------------------------------
 * Decoder-stack glue (outside the attention cores; used by the end-to-end
 * hybrid stack).  All tensors f32 unless stated, row-major, device pointers.
 *   q35_q8_embedding: kernels.rs:15-45.  table [vocab, dim/4] u32 (Q8F),
 *     scales [vocab, dim/64]; out [n, dim].  ids outside [0, vocab) give
 *     zero rows.
 *   q35_add_rmsnorm: text_modules.rs:800-809 with the residual add of
 *     :1053-1085: h = x (+ residual if non-NULL), sum_out = h if non-NULL,
 *     out = h / sqrt(mean(h^2) + eps) * (1 + weight).  [n_rows, dim].
 *   q35_silu_mul: out = up * silu(gate) (:999-1011), n elements.
 *   q35_q8_lm_head: kernels.rs:251-291, logits[v] = E[v] . x with the tied
 *     Q8F embedding E [vocab, dim] (dim 2048).
 *   q35_argmax: kernels.rs:298-371; ties resolve to the smallest index.
 *   q35_q8_dequant: the dense f32 weight [rows, cols] of a Q8F matrix (the
 *     prefill Linear::forward operand).
 *   q35_rope_gather: cos/sin [B, rot] of each sequence's decode position
 *     lens[b] from tables [max_pos, rot] (text_modules.rs:30-43 at
 *     position past_len, model.rs:50-56), so a captured decode step needs
 *     no host-side position.
 */
int q35_q8_embedding(int32_t n, int32_t vocab, int32_t dim, const int32_t *ids,
                     const uint32_t *table, const float *scales, float *out,
                     void *stream);
int q35_add_rmsnorm(int32_t n_rows, int32_t dim, const float *x,
                    const float *residual, const float *weight, float eps,
                    float *out, float *sum_out, void *stream);
int q35_silu_mul(int64_t n, const float *gate, const float *up, float *out,
                 void *stream);
int q35_q8_lm_head(int32_t vocab, int32_t dim, const float *x,
                   const uint32_t *table, const float *scales, float *logits,
                   void *stream);
size_t q35_argmax_workspace_size(void);
int q35_argmax(int32_t n, const float *x, int32_t *out_index, void *workspace,
               size_t workspace_bytes, void *stream);
int q35_q8_dequant(int32_t rows, int32_t cols, const uint32_t *w,
                   const float *scales, float *out, void *stream);
int q35_rope_gather(int32_t batch, int32_t rot, int32_t max_pos,
                    const int32_t *lens, const float *table_cos,
                    const float *table_sin, float *cos_out, float *sin_out,
                    void *stream);

/* --------------------------------------------------------------------------
 * Gated GQA, one decode step.  Replaces text_modules.rs:866-936 of
 * Attention::forward (:842-944): q/gate split of q_proj, q_norm/k_norm
 * (RMSNorm 1+w, :800-809), partial RoPE (:754-774), KV-cache append
 * (:899-909, in place instead of cat), repeat_kv (:776-792, as head
 * grouping, no copy), SDPA (burn::tensor::module::attention, scale
 * 1/sqrt(head_dim)) and the sigmoid output gate.
 *   q_gate   [B, Hq, 2*D]   q_proj output: per head [query | gate]
 *   k_new, v_new [B, Hkv, D] k_proj / v_proj outputs (pre-norm, pre-RoPE)
 *   qn_w, kn_w [D]          q_norm / k_norm weights (applied as 1 + w)
 *   cos, sin [B, rotary_dim] rotary tables of the new position
 *   k_cache, v_cache [B, Hkv, capacity, D] in/out (post-norm, post-RoPE keys)
 *   lens [B] int32 in/out   valid tokens per sequence; the new token is
 *                           written at lens[b] and lens[b] is incremented
 *   out [B, Hq*D]           attention output * sigmoid(gate) (o_proj input)
 *   max_len                 host upper bound on lens[b]+1 over the batch
 *                           (sizes the split-K grid; capacity is always safe)
 *   workspace  >= q35_gqa_decode_workspace_size(dims, max_len) bytes, zeroed
 *              once by q35_workspace_init before first use; the kernel leaves
 *              it reusable.  One workspace per concurrently running call.
 */
size_t q35_gqa_decode_workspace_size(const q35_gqa_dims *dims, int64_t max_len);
int q35_workspace_init(void *workspace, size_t workspace_bytes, void *stream);
int q35_gqa_decode(const q35_gqa_dims *dims, int64_t max_len,
                   const float *q_gate, const float *k_new, const float *v_new,
                   const float *qn_w, const float *kn_w, const float *cos,
                   const float *sin, float *k_cache, float *v_cache,
                   int32_t *lens, float *out, void *workspace,
                   size_t workspace_bytes, void *stream);

/* --------------------------------------------------------------------------
 * Gated GQA over a prompt of T tokens (prefill).  Replaces Attention::forward
 * (text_modules.rs:842-944) for seq_len = T: the same per-token steps as
 * q35_gqa_decode, with the causal mask of model.rs:59-67 (prompt token t sees
 * keys 0 .. lens[b] + t).  Appends T keys / values at lens[b] and adds T to
 * lens[b].
 *   q_gate   [B, T, Hq, 2*D]   k_new, v_new [B, T, Hkv, D]
 *   cos, sin [B, T, rotary_dim] (NULL allowed when rotary_dim == 0)
 *   out      [B, T, Hq*D]
 *   max_len  host upper bound on lens[b] + T over the batch (sizes the
 *            workspace; sequences beyond it or beyond the capacity are
 *            skipped and flagged in the workspace status word).
 *   workspace >= q35_gqa_prefill_workspace_size(dims, T, max_len) bytes,
 *            256-byte aligned; its first word is the status word read by
 *            q35_workspace_status.
 * Requires num_q_heads + num_kv_heads <= 32 and head_dim 256.
 */
size_t q35_gqa_prefill_workspace_size(const q35_gqa_dims *dims, int32_t seq_len,
                                      int64_t max_len);
int q35_gqa_prefill(const q35_gqa_dims *dims, int32_t seq_len, int64_t max_len,
                    const float *q_gate, const float *k_new, const float *v_new,
                    const float *qn_w, const float *kn_w, const float *cos,
                    const float *sin, float *k_cache, float *v_cache,
                    int32_t *lens, float *out, void *workspace,
                    size_t workspace_bytes, void *stream);

/* Context-parallel form of q35_gqa_decode for one shard of a KV cache split
 * along its length across GPUs (text_modules.rs:899-928 with the keys
 * partitioned; no reference counterpart for the partitioning itself).
 * Writes, per (sequence, query head), the unnormalised partial
 * partial_out[B, Hq, D+2] = [o (D) | m | l] of the softmax over this shard's
 * keys, m in log2 units (scores * log2(e)), o = sum_j 2^(s_j - m) v_j.
 * k_new / v_new NULL: attend the cached keys [0, lens[b]) only, no append,
 * lens unchanged (every shard but the last).  Non-NULL: append at lens[b] as
 * q35_gqa_decode does and attend [0, lens[b]] (the shard holding the tail).
 * cos / sin are the tables of the token's global position. */
int q35_gqa_decode_partial(const q35_gqa_dims *dims, int64_t max_len,
                           const float *q_gate, const float *k_new,
                           const float *v_new, const float *qn_w,
                           const float *kn_w, const float *cos,
                           const float *sin, float *k_cache, float *v_cache,
                           int32_t *lens, float *partial_out, void *workspace,
                           size_t workspace_bytes, void *stream);

/* Merges n_parts shard partials parts[n_parts, B, Hq, D+2] (as written by
 * q35_gqa_decode_partial, gathered from every shard) into
 * out[B, Hq*D] = (sum o 2^(m-M)) / (sum l 2^(m-M)) * sigmoid(gate), the gate
 * taken from q_gate[B, Hq, 2*D] (text_modules.rs:930-936). */
int q35_gqa_combine_partials(int32_t batch, int32_t num_q_heads,
                             int32_t head_dim, int32_t n_parts,
                             const float *parts, const float *q_gate,
                             float *out, void *stream);

/* --------------------------------------------------------------------------
 * Exchange step of one sequence decoded across the GPUs of a node over peer
 * memory (the single-sequence variant of BASELINE config 4; the reference
 * runs one device and has no counterpart).  Each rank holds a shard:
 * GatedDeltaNet value heads (its outputs, n_gdn floats per sequence, are one
 * slice of out_proj's input, text_modules.rs:651-662) and a length range of
 * the KV cache (its softmax partials [B, Hq, D+2] from
 * q35_gqa_decode_partial, text_modules.rs:899-928).  q35_cp_exchange stores
 * this rank's payload into every peer's receive buffer over NVLink, each
 * value in an 8-byte word tagged with the step's epoch, polls (bounded, 1 s)
 * its own buffer until every rank's words of the step are there, and
 * writes on every rank
 *   gdn_full [B, world * n_gdn]  the GDN outputs in rank order, and
 *   gqa_out  [B, Hq * D]         the merged attention output * sigmoid(gate)
 *                                (gate from q_gate [B, Hq, 2 * D]).
 * Set-up (not on the hot path): q35_cp_create allocates this rank's receive
 * buffer and returns its 64-byte CUDA IPC handle; the caller exchanges the
 * handles (e.g. over its process group) and passes all of them, in rank
 * order, to q35_cp_connect.  Every rank calls q35_cp_exchange the same number
 * of times, in the same order; each call is one kernel and allocates nothing,
 * so the steps can be captured in a CUDA graph.  n_gdn must be even and
 * every buffer 8-byte aligned.  A wait that gives up sets
 * Q35_STATUS_WAIT_TIMEOUT (q35_cp_status) and poisons the outputs with NaN. */
int q35_cp_create(int32_t world, int32_t rank, int32_t batch, int32_t n_gdn,
                  int32_t num_q_heads, int32_t head_dim, void **ctx_out,
                  void *ipc_handle_out);
int q35_cp_connect(void *ctx, const void *ipc_handles);
int q35_cp_exchange(void *ctx, const float *gdn_local, const float *gqa_part,
                    const float *q_gate, float *gdn_full, float *gqa_out,
                    void *stream);
int q35_cp_status(void *ctx, uint32_t *status_out, int32_t clear, void *stream);
/* Tear-down: every rank calls q35_cp_disconnect (unmaps the peers' buffers)
 * with no exchange in flight, the ranks meet at a barrier, then each calls
 * q35_cp_destroy (frees its own buffer). */
int q35_cp_disconnect(void *ctx);
int q35_cp_destroy(void *ctx);

/* q35_gqa_decode for callers that cannot allocate device memory (no entry
 * in the reference: its Burn host always allocates).  Same arguments and
 * semantics minus the workspace: the split-K scratch lives in a fixed 16 MiB
 * array inside the library, held on every GPU that loads it until exit.
 * Calls needing more (q35_gqa_decode_workspace_size > 16 MiB, e.g. 256
 * sequences at 32K context) fail with Q35_ERR_WORKSPACE.  All calls share the
 * array, so calls that overlap on the GPU race; each call first clears the
 * array's counters with a memset on `stream`.  The first call on a device
 * looks up the array's device address and should come before any stream
 * capture.  Every argument check runs before anything is queued on
 * `stream`.  The device-side status word (Q35_STATUS_* bits) lives in the
 * private array and is cleared by the next call, so these callers cannot
 * read it: a skipped sequence (full cache, length hint exceeded, a wait that
 * gave up) shows only as lens[b] left unchanged.  Callers that need the bits
 * use q35_gqa_decode with a workspace and q35_workspace_status. */
int q35_gqa_decode_noalloc(const q35_gqa_dims *dims, int64_t max_len,
                           const float *q_gate, const float *k_new,
                           const float *v_new, const float *qn_w,
                           const float *kn_w, const float *cos,
                           const float *sin, float *k_cache, float *v_cache,
                           int32_t *lens, float *out, void *stream);

/* Reads (and with clear != 0 resets) the device-side status word of a
 * workspace (Q35_STATUS_* bits).  Synchronizes `stream`.  status_out is a
 * HOST pointer. */
int q35_workspace_status(void *workspace, uint32_t *status_out, int32_t clear,
                         void *stream);

/* Test hook: q35_gdn_decode with the kernel schedule forced: split in
 * {1, 2, 4, 8} selects the cluster kernel with that per-head column split,
 * -1 the persistent streaming kernel (the default picks from the batch). */
int q35_gdn_decode_split(const q35_gdn_dims *dims, int32_t split,
                         const float *mixed_qkv, const float *z,
                         const float *beta, const float *g,
                         const float *conv_w, const float *norm_w,
                         float *conv_state, float *rec_state, float *out,
                         void *stream);

/* Reads (and with clear != 0 resets) this device's status word, the
 * Q35_STATUS_* bits of the kernels that take no workspace and report there
 * (q35_q8_gemm(_fused), q35_q8_gemv(_fused), q35_gdn_gate mode 0 and the
 * streaming schedule of q35_gdn_decode).
 * Synchronizes `stream`.  status_out is a HOST pointer. */
int q35_device_status(uint32_t *status_out, int32_t clear, void *stream);

/* Test hook: the next call that reaches the armed site withholds one of its
 * asynchronous copies and bounds its waits at 2 ms, so that a wait runs out
 * and the error path runs (status word set, outputs poisoned, every copy and
 * tensor-core operation already started waited for) without a fault or a
 * hang.  site 1: the q35_gdn_prefill state pass (chunk 1's W operand, needs
 * seq_len > 64); site 2: the q35_gqa_decode producer (the first K tile of the
 * first split); site 3: q35_cp_exchange (this rank stores none of its
 * words, so its own waits run out); 0 disarms.  Arming is global to the
 * process and consumed by one call. */
int q35_test_arm_wait_fault(int32_t site);

/* --------------------------------------------------------------------------
 * Library information. */
const char *q35_last_error(void);       /* thread-local, never NULL */
const char *q35_version(void);
/* Number of kernel launches the library issued on this host thread since
 * the last reset (test/bench bookkeeping; counts every <<<>>>/cudaLaunch). */
uint64_t q35_launch_count(int32_t reset);

#ifdef __cplusplus
}
#endif
#endif /* Q35ATTN_H */
