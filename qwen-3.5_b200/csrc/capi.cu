// capi.cu -- the extern "C" boundary of libq35attn (declared in
// include/q35attn.h): argument validation, error reporting, workspace
// management and dispatch to the sm_100a kernels.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"

namespace q35 {

// kernels (defined in the other translation units)
int gdn_decode_launch(const q35_gdn_dims *d, const float *mixed_qkv, const float *z, const float *beta,
                      const float *g, const float *conv_w, const float *norm_w, float *conv_state,
                      float *rec_state, float *out, cudaStream_t st, int force_split);
int gdn_gate_launch(int N, int in_dim, int H, const float *x, const float *wb, const float *wa, const float *a_log,
                    const float *dt_bias, float *beta, float *g, int mode, cudaStream_t st);
size_t gqa_workspace_bytes(int B, int Hq, int Hkv, long long max_len, int sms);
int gqa_decode_launch(const q35_gqa_dims *d, long long max_len, const float *q_gate, const float *k_new,
                      const float *v_new, const float *qn_w, const float *kn_w, const float *cos,
                      const float *sin, float *k_cache, float *v_cache, int32_t *lens, float *out,
                      void *ws, size_t ws_bytes, cudaStream_t st, float *part_out);
size_t gqa_prefill_workspace_bytes(int B, int T, int Hq, int Hkv, long long max_len);
int gqa_prefill_launch(const q35_gqa_dims *d, int T, long long max_len, const float *q_gate, const float *k_new,
                       const float *v_new, const float *qn_w, const float *kn_w, const float *cos,
                       const float *sin, float *k_cache, float *v_cache, int32_t *lens, float *out, void *ws,
                       size_t ws_bytes, cudaStream_t st);
int q8_embedding_launch(int n, int vocab, int dim, const int32_t *ids, const uint32_t *table, const float *scales,
                        float *out, cudaStream_t st);
int add_rmsnorm_launch(int n, int dim, const float *x, const float *residual, const float *w, float eps, float *out,
                       float *sum_out, cudaStream_t st);
int silu_mul_launch(size_t n, const float *gate, const float *up, float *out, cudaStream_t st);
int q8_lm_head_launch(int vocab, int dim, const float *x, const uint32_t *table, const float *scales, float *logits,
                      cudaStream_t st);
size_t argmax_workspace_bytes();
int argmax_launch(int n, const float *x, int32_t *out, void *ws, cudaStream_t st);
int q8_dequant_launch(int rows, int cols, const uint32_t *w, const float *scales, float *out, cudaStream_t st);
int rope_gather_launch(int B, int rot, int max_pos, const int32_t *lens, const float *tc, const float *ts, float *oc,
                       float *os, cudaStream_t st);
int gqa_combine_launch(int B, int Hq, int n_parts, const float *parts, const float *q_gate, float *out,
                       cudaStream_t st);
size_t gdn_prefill_workspace_bytes(const q35_gdn_dims *d, int T);
int gqa_decode_check_args(const q35_gqa_dims *dims, int64_t max_len, const float *q_gate, const float *k_new,
                          const float *v_new, const float *qn_w, const float *kn_w, const float *cos,
                          const float *sin, const float *k_cache, const float *v_cache, const int32_t *lens,
                          const float *out);
size_t q8_gemm_workspace_bytes(int T, int K);
int q8_gemm_launch(int T, int K, int n_seg, const q35_q8_segment *segs, const float *x, int swiglu, void *ws,
                   size_t ws_bytes, cudaStream_t st);
int q8_gemv_launch(int in_dim, int out_dim, const float *x, const uint32_t *w, const float *scales, float *y,
                   int mode, cudaStream_t st);
int q8_gemv_fused_launch(int in_dim, int n_seg, const q35_q8_segment *segs, const float *x, const float *residual,
                         const float *norm_w, float eps, float *sum_out, float *x_out, int swiglu, int mode,
                         cudaStream_t st);
int gdn_prefill_launch(const q35_gdn_dims *d, int T, const float *mixed_qkv, const float *z, const float *beta,
                       const float *g, const float *conv_w, const float *norm_w, float *conv_state, int has_prev,
                       float *rec_state, int has_init, float *out, void *ws, size_t ws_bytes, cudaStream_t st);

namespace {
thread_local std::string g_last_error = "";
std::atomic<uint64_t> g_launches{0};
std::mutex g_sm_mu;
int g_sm_count[64] = {0};
int g_sm_major[64] = {0};
}  // namespace

void set_error(const std::string &msg) { g_last_error = msg; }

namespace {
std::atomic<int> g_fault_site{kFaultNone};
}  // namespace

// Status word of the kernels that take no workspace (Q35_STATUS_* bits), one
// per device; kernels receive its device address as an argument.
__device__ uint32_t g_device_status;

namespace {
std::mutex g_status_mu;
uint32_t *g_status_ptr[64] = {nullptr};
}  // namespace

uint32_t *device_status_word() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_status_mu);
  if (g_status_ptr[dev] == nullptr) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
    g_status_ptr[dev] = static_cast<uint32_t *>(p);
  }
  return g_status_ptr[dev];
}

bool take_fault(int site) {
  int s = site;
  return site != kFaultNone && g_fault_site.compare_exchange_strong(s, kFaultNone);
}

bool pdl_enabled() {
  static const bool on = [] {
    const char *v = std::getenv("Q35_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int fail(int code, const std::string &msg) {
  set_error(msg);
  return code;
}

int check_cuda(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return Q35_OK;
  return fail(Q35_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

void note_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

static int query_device(int *sms, int *major) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
  std::lock_guard<std::mutex> lk(g_sm_mu);
  if (g_sm_count[dev] == 0) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return -1;
    g_sm_count[dev] = prop.multiProcessorCount;
    g_sm_major[dev] = prop.major;
  }
  *sms = g_sm_count[dev];
  *major = g_sm_major[dev];
  return 0;
}

int device_sm_count() {
  int sms = 148, major = 10;
  if (query_device(&sms, &major) != 0) return 148;
  return sms;
}

int require_sm100() {
  int sms = 0, major = 0;
  if (query_device(&sms, &major) != 0) return fail(Q35_ERR_DEVICE, "no CUDA device available");
  if (major != 10) return fail(Q35_ERR_DEVICE, "libq35attn is built for sm_100a (B200); device major " +
                                                   std::to_string(major));
  return Q35_OK;
}

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int check_gdn_dims(const q35_gdn_dims *d) {
  Q35_REQUIRE(d != nullptr, Q35_ERR_INVALID_ARG, "dims is NULL");
  Q35_REQUIRE(d->batch >= 0 && d->num_k_heads > 0 && d->num_v_heads > 0, Q35_ERR_INVALID_ARG,
              "gdn dims: batch must be >= 0 and head counts > 0");
  Q35_REQUIRE(d->num_v_heads % d->num_k_heads == 0, Q35_ERR_INVALID_ARG,
              "gdn dims: num_v_heads must be a multiple of num_k_heads");
  Q35_REQUIRE(d->head_k_dim == 128 && d->head_v_dim == 128, Q35_ERR_UNSUPPORTED,
              "gdn dims: head_k_dim = head_v_dim = 128 is the compiled configuration");
  Q35_REQUIRE(d->conv_kernel >= 2 && d->conv_kernel <= 4, Q35_ERR_UNSUPPORTED, "gdn dims: conv_kernel must be 2..4");
  Q35_REQUIRE(d->eps >= 0.0f, Q35_ERR_INVALID_ARG, "gdn dims: eps must be >= 0");
  Q35_REQUIRE(d->batch <= 65535 && d->num_v_heads <= 65535, Q35_ERR_UNSUPPORTED, "gdn dims: batch / heads too large");
  return Q35_OK;
}

static int check_gqa_dims(const q35_gqa_dims *d) {
  Q35_REQUIRE(d != nullptr, Q35_ERR_INVALID_ARG, "dims is NULL");
  Q35_REQUIRE(d->batch >= 0 && d->num_q_heads > 0 && d->num_kv_heads > 0, Q35_ERR_INVALID_ARG,
              "gqa dims: batch must be >= 0 and head counts > 0");
  Q35_REQUIRE(d->num_q_heads % d->num_kv_heads == 0, Q35_ERR_INVALID_ARG,
              "gqa dims: num_q_heads must be a multiple of num_kv_heads");
  const int G = d->num_q_heads / d->num_kv_heads;
  Q35_REQUIRE(G == 1 || G == 2 || G == 4 || G == 8, Q35_ERR_UNSUPPORTED, "gqa dims: group size must be 1, 2, 4 or 8");
  Q35_REQUIRE(d->head_dim == 256, Q35_ERR_UNSUPPORTED, "gqa dims: head_dim = 256 is the compiled configuration");
  Q35_REQUIRE(d->rotary_dim >= 0 && d->rotary_dim <= d->head_dim && d->rotary_dim % 2 == 0, Q35_ERR_INVALID_ARG,
              "gqa dims: rotary_dim must be even and <= head_dim");
  Q35_REQUIRE(d->capacity > 0 && d->capacity < (1LL << 31), Q35_ERR_INVALID_ARG,
              "gqa dims: capacity must be in [1, 2^31)");
  Q35_REQUIRE(d->batch <= 65535 && d->num_kv_heads <= 65535, Q35_ERR_UNSUPPORTED, "gqa dims: batch / heads too large");
  Q35_REQUIRE(d->eps >= 0.0f, Q35_ERR_INVALID_ARG, "gqa dims: eps must be >= 0");
  return Q35_OK;
}

}  // namespace q35

using namespace q35;

#define Q35_PTR(p) Q35_REQUIRE((p) != nullptr, Q35_ERR_INVALID_ARG, #p " is NULL")
#define Q35_PTR16(p) \
  Q35_REQUIRE((p) != nullptr && aligned16(p), Q35_ERR_INVALID_ARG, #p " must be a non-NULL 16-byte aligned pointer")

// Every check q35_gqa_decode makes before it touches the device (shapes,
// max_len against the capacity, pointer alignment, the device itself), so a
// caller can validate a call before queueing anything on its stream.
int q35::gqa_decode_check_args(const q35_gqa_dims *dims, int64_t max_len, const float *q_gate, const float *k_new,
                          const float *v_new, const float *qn_w, const float *kn_w, const float *cos,
                          const float *sin, const float *k_cache, const float *v_cache, const int32_t *lens,
                          const float *out) {
  if (int rc = check_gqa_dims(dims)) return rc;
  Q35_REQUIRE(max_len > 0, Q35_ERR_INVALID_ARG, "gqa_decode: max_len must be > 0");
  Q35_REQUIRE(max_len <= dims->capacity, Q35_ERR_CAPACITY, "gqa_decode: max_len exceeds the cache capacity");
  if (dims->batch == 0) return Q35_OK;
  Q35_PTR16(q_gate); Q35_PTR16(k_new); Q35_PTR16(v_new); Q35_PTR16(qn_w); Q35_PTR16(kn_w);
  if (dims->rotary_dim > 0) {
    Q35_PTR(cos);
    Q35_PTR(sin);
  }
  Q35_PTR16(k_cache); Q35_PTR16(v_cache); Q35_PTR(lens); Q35_PTR(out);
  return require_sm100();
}

extern "C" {

const char *q35_last_error(void) { return g_last_error.c_str(); }

const char *q35_version(void) { return "q35attn 0.1.0 (sm_100a)"; }

uint64_t q35_launch_count(int32_t reset) {
  return reset ? g_launches.exchange(0) : g_launches.load();
}

size_t q35_q8_gemm_workspace_size(int32_t n_rows, int32_t in_dim) {
  if (n_rows <= 0 || in_dim <= 0 || in_dim % 32 != 0) return 0;
  return q8_gemm_workspace_bytes(n_rows, in_dim);
}

int q35_q8_gemm(int32_t n_rows, int32_t in_dim, int32_t out_dim, const float *x, const uint32_t *w,
                const float *scales, float *y, void *workspace, size_t workspace_bytes, void *stream) {
  Q35_REQUIRE(n_rows >= 0 && in_dim > 0 && out_dim > 0, Q35_ERR_INVALID_ARG, "q8_gemm: bad sizes");
  if (n_rows == 0) return Q35_OK;
  Q35_PTR16(x); Q35_PTR16(w); Q35_PTR16(scales); Q35_PTR16(y);
  if (int rc = require_sm100()) return rc;
  const q35_q8_segment seg = {w, scales, y, out_dim};
  return q8_gemm_launch(n_rows, in_dim, 1, &seg, x, 0, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int q35_q8_gemm_fused(int32_t n_rows, int32_t in_dim, int32_t n_seg, const q35_q8_segment *segs, const float *x,
                      int32_t swiglu, void *workspace, size_t workspace_bytes, void *stream) {
  Q35_REQUIRE(n_rows >= 0 && in_dim > 0, Q35_ERR_INVALID_ARG, "q8_gemm_fused: bad sizes");
  Q35_REQUIRE(swiglu == 0 || swiglu == 1, Q35_ERR_INVALID_ARG, "q8_gemm_fused: swiglu must be 0 or 1");
  Q35_PTR(segs);
  if (n_rows == 0) return Q35_OK;
  Q35_PTR16(x);
  if (int rc = require_sm100()) return rc;
  return q8_gemm_launch(n_rows, in_dim, n_seg, segs, x, swiglu, workspace, workspace_bytes,
                        static_cast<cudaStream_t>(stream));
}

int q35_device_status(uint32_t *status_out, int32_t clear, void *stream) {
  Q35_PTR(status_out);
  if (int rc = require_sm100()) return rc;
  uint32_t *w = device_status_word();
  Q35_REQUIRE(w != nullptr, Q35_ERR_CUDA, "device_status: status word unavailable");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t v = 0;
  if (int rc = check_cuda(cudaMemcpyAsync(&v, w, sizeof(v), cudaMemcpyDeviceToHost, st), "device status read"))
    return rc;
  if (int rc = check_cuda(cudaStreamSynchronize(st), "device status sync")) return rc;
  *status_out = v;
  if (clear) return check_cuda(cudaMemsetAsync(w, 0, sizeof(uint32_t), st), "device status clear");
  return Q35_OK;
}

int q35_test_arm_wait_fault(int32_t site) {
  Q35_REQUIRE(site >= kFaultNone && site <= kFaultCpExchange, Q35_ERR_INVALID_ARG,
              "test_arm_wait_fault: unknown site");
  g_fault_site.store(site);
  return Q35_OK;
}

int q35_gdn_decode(const q35_gdn_dims *dims, const float *mixed_qkv, const float *z, const float *beta,
                   const float *g, const float *conv_w, const float *norm_w, float *conv_state, float *rec_state,
                   float *out, void *stream) {
  if (int rc = check_gdn_dims(dims)) return rc;
  if (dims->batch == 0) return Q35_OK;
  Q35_PTR(mixed_qkv); Q35_PTR(z); Q35_PTR(beta); Q35_PTR(g); Q35_PTR(conv_w); Q35_PTR(norm_w);
  Q35_PTR(conv_state); Q35_PTR(out);
  Q35_PTR16(rec_state);
  if (int rc = require_sm100()) return rc;
  return gdn_decode_launch(dims, mixed_qkv, z, beta, g, conv_w, norm_w, conv_state, rec_state, out,
                           static_cast<cudaStream_t>(stream), 0);
}

/* Test hook: same as q35_gdn_decode with the column split forced (1,2,4,8). */
int q35_gdn_decode_split(const q35_gdn_dims *dims, int32_t split, const float *mixed_qkv, const float *z,
                         const float *beta, const float *g, const float *conv_w, const float *norm_w,
                         float *conv_state, float *rec_state, float *out, void *stream) {
  if (int rc = check_gdn_dims(dims)) return rc;
  Q35_REQUIRE(split == -1 || split == 1 || split == 2 || split == 4 || split == 8, Q35_ERR_INVALID_ARG,
              "split must be -1 (streaming kernel) or 1, 2, 4, 8");
  if (dims->batch == 0) return Q35_OK;
  Q35_PTR(mixed_qkv); Q35_PTR(z); Q35_PTR(beta); Q35_PTR(g); Q35_PTR(conv_w); Q35_PTR(norm_w);
  Q35_PTR(conv_state); Q35_PTR(out);
  Q35_PTR16(rec_state);
  if (int rc = require_sm100()) return rc;
  return gdn_decode_launch(dims, mixed_qkv, z, beta, g, conv_w, norm_w, conv_state, rec_state, out,
                           static_cast<cudaStream_t>(stream), split);
}

int q35_gdn_gate(int32_t n_rows, int32_t in_dim, int32_t num_heads, const float *x, const float *w_b,
                 const float *w_a, const float *a_log, const float *dt_bias, float *beta, float *g, int32_t mode,
                 void *stream) {
  Q35_REQUIRE(n_rows >= 0 && in_dim > 0 && num_heads > 0, Q35_ERR_INVALID_ARG, "gdn_gate: bad sizes");
  Q35_REQUIRE(mode == 0 || mode == 1, Q35_ERR_INVALID_ARG, "gdn_gate: mode must be 0 or 1");
  if (n_rows == 0) return Q35_OK;
  Q35_PTR(x); Q35_PTR(w_b); Q35_PTR(w_a); Q35_PTR(a_log); Q35_PTR(dt_bias); Q35_PTR(beta); Q35_PTR(g);
  if (int rc = require_sm100()) return rc;
  return gdn_gate_launch(n_rows, in_dim, num_heads, x, w_b, w_a, a_log, dt_bias, beta, g, mode,
                         static_cast<cudaStream_t>(stream));
}

int q35_q8_gemv(int32_t in_dim, int32_t out_dim, const float *x, const uint32_t *w, const float *scales, float *y,
                int32_t mode, void *stream) {
  Q35_REQUIRE(in_dim > 0 && out_dim > 0, Q35_ERR_INVALID_ARG, "q8_gemv: in_dim and out_dim must be > 0");
  Q35_REQUIRE(out_dim % 64 == 0, Q35_ERR_UNSUPPORTED, "q8_gemv: out_dim must be a multiple of 64 (Q8F block)");
  Q35_REQUIRE(mode == 0 || mode == 1, Q35_ERR_INVALID_ARG, "q8_gemv: mode must be 0 or 1");
  Q35_PTR(x); Q35_PTR16(w); Q35_PTR(scales); Q35_PTR(y);
  if (int rc = require_sm100()) return rc;
  return q8_gemv_launch(in_dim, out_dim, x, w, scales, y, mode, static_cast<cudaStream_t>(stream));
}

int q35_q8_gemv_fused(int32_t in_dim, int32_t n_seg, const q35_q8_segment *segs, const float *x,
                      const float *residual, const float *norm_w, float eps, float *sum_out, float *x_out,
                      int32_t swiglu, int32_t mode, void *stream) {
  Q35_REQUIRE(in_dim > 0, Q35_ERR_INVALID_ARG, "q8_gemv_fused: in_dim must be > 0");
  Q35_REQUIRE(mode == 0 || mode == 1, Q35_ERR_INVALID_ARG, "q8_gemv_fused: mode must be 0 or 1");
  Q35_REQUIRE(swiglu == 0 || swiglu == 1, Q35_ERR_INVALID_ARG, "q8_gemv_fused: swiglu must be 0 or 1");
  Q35_REQUIRE(n_seg >= 1 && n_seg <= 4, Q35_ERR_INVALID_ARG, "q8_gemv_fused: 1 to 4 segments");
  Q35_PTR(segs); Q35_PTR16(x);
  Q35_REQUIRE(!swiglu || (n_seg == 2 && segs[0].out_dim == segs[1].out_dim), Q35_ERR_INVALID_ARG,
              "q8_gemv_fused: swiglu takes two segments (up, gate) of equal out_dim");
  Q35_REQUIRE(in_dim % 4 == 0 && in_dim <= (norm_w ? 8192 : 16384), Q35_ERR_UNSUPPORTED,
              "q8_gemv_fused: in_dim must be a multiple of 4, at most 8192 with the norm (16384 without)");
  Q35_REQUIRE(norm_w != nullptr || (residual == nullptr && sum_out == nullptr && x_out == nullptr), Q35_ERR_INVALID_ARG,
              "q8_gemv_fused: residual / sum_out / x_out need norm_w");
  if (residual) Q35_PTR16(residual);
  if (norm_w) Q35_PTR16(norm_w);
  for (int k = 0; k < n_seg; ++k) {
    Q35_REQUIRE(segs[k].out_dim > 0 && segs[k].out_dim % 256 == 0, Q35_ERR_UNSUPPORTED,
                "q8_gemv_fused: every out_dim must be a positive multiple of 256");
    Q35_PTR16(segs[k].w); Q35_PTR16(segs[k].scales); Q35_PTR(segs[k].y);
  }
  const void *outs[2] = {sum_out, x_out};
  for (const void *o : outs)
    Q35_REQUIRE(o == nullptr || (o != x && o != residual), Q35_ERR_INVALID_ARG,
                "q8_gemv_fused: sum_out / x_out must not alias x or residual");
  if (int rc = require_sm100()) return rc;
  return q8_gemv_fused_launch(in_dim, n_seg, segs, x, residual, norm_w, eps, sum_out, x_out, swiglu, mode,
                              static_cast<cudaStream_t>(stream));
}

size_t q35_gqa_prefill_workspace_size(const q35_gqa_dims *dims, int32_t seq_len, int64_t max_len) {
  if (check_gqa_dims(dims) != Q35_OK || seq_len <= 0 || max_len < seq_len) return 0;
  return gqa_prefill_workspace_bytes(dims->batch, seq_len, dims->num_q_heads, dims->num_kv_heads, max_len);
}

int q35_gqa_prefill(const q35_gqa_dims *dims, int32_t seq_len, int64_t max_len, const float *q_gate,
                    const float *k_new, const float *v_new, const float *qn_w, const float *kn_w, const float *cos,
                    const float *sin, float *k_cache, float *v_cache, int32_t *lens, float *out, void *workspace,
                    size_t workspace_bytes, void *stream) {
  if (int rc = check_gqa_dims(dims)) return rc;
  Q35_REQUIRE(seq_len >= 0, Q35_ERR_INVALID_ARG, "gqa_prefill: seq_len must be >= 0");
  if (dims->batch == 0 || seq_len == 0) return Q35_OK;
  Q35_REQUIRE(max_len >= seq_len && max_len <= dims->capacity, Q35_ERR_INVALID_ARG,
              "gqa_prefill: max_len must be in [seq_len, capacity]");
  Q35_REQUIRE(dims->num_q_heads + dims->num_kv_heads <= 32, Q35_ERR_UNSUPPORTED,
              "gqa_prefill: num_q_heads + num_kv_heads must be <= 32");
  Q35_PTR16(q_gate); Q35_PTR16(k_new); Q35_PTR16(v_new); Q35_PTR16(qn_w); Q35_PTR16(kn_w);
  Q35_PTR16(k_cache); Q35_PTR16(v_cache); Q35_PTR(lens); Q35_PTR16(out);
  if (dims->rotary_dim > 0) {
    Q35_PTR(cos); Q35_PTR(sin);
  }
  if (int rc = require_sm100()) return rc;
  return gqa_prefill_launch(dims, seq_len, max_len, q_gate, k_new, v_new, qn_w, kn_w, cos, sin, k_cache, v_cache,
                            lens, out, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int q35_q8_embedding(int32_t n, int32_t vocab, int32_t dim, const int32_t *ids, const uint32_t *table,
                     const float *scales, float *out, void *stream) {
  Q35_REQUIRE(n >= 0 && vocab > 0 && dim > 0 && dim % 64 == 0, Q35_ERR_INVALID_ARG,
              "q8_embedding: n >= 0, vocab > 0, dim a multiple of 64");
  if (n == 0) return Q35_OK;
  Q35_PTR(ids); Q35_PTR(table); Q35_PTR(scales); Q35_PTR16(out);
  if (int rc = require_sm100()) return rc;
  return q8_embedding_launch(n, vocab, dim, ids, table, scales, out, static_cast<cudaStream_t>(stream));
}

int q35_add_rmsnorm(int32_t n_rows, int32_t dim, const float *x, const float *residual, const float *weight,
                    float eps, float *out, float *sum_out, void *stream) {
  Q35_REQUIRE(n_rows >= 0 && dim > 0 && eps >= 0.0f, Q35_ERR_INVALID_ARG, "add_rmsnorm: bad sizes");
  if (n_rows == 0) return Q35_OK;
  Q35_PTR(x); Q35_PTR(weight); Q35_PTR(out);
  if (int rc = require_sm100()) return rc;
  return add_rmsnorm_launch(n_rows, dim, x, residual, weight, eps, out, sum_out, static_cast<cudaStream_t>(stream));
}

int q35_silu_mul(int64_t n, const float *gate, const float *up, float *out, void *stream) {
  Q35_REQUIRE(n >= 0, Q35_ERR_INVALID_ARG, "silu_mul: n must be >= 0");
  if (n == 0) return Q35_OK;
  Q35_PTR(gate); Q35_PTR(up); Q35_PTR(out);
  if (int rc = require_sm100()) return rc;
  return silu_mul_launch((size_t)n, gate, up, out, static_cast<cudaStream_t>(stream));
}

int q35_q8_lm_head(int32_t vocab, int32_t dim, const float *x, const uint32_t *table, const float *scales,
                   float *logits, void *stream) {
  Q35_REQUIRE(vocab > 0, Q35_ERR_INVALID_ARG, "q8_lm_head: vocab must be > 0");
  Q35_PTR16(x); Q35_PTR16(table); Q35_PTR(scales); Q35_PTR(logits);
  if (int rc = require_sm100()) return rc;
  return q8_lm_head_launch(vocab, dim, x, table, scales, logits, static_cast<cudaStream_t>(stream));
}

size_t q35_argmax_workspace_size(void) { return argmax_workspace_bytes(); }

int q35_argmax(int32_t n, const float *x, int32_t *out_index, void *workspace, size_t workspace_bytes,
               void *stream) {
  Q35_REQUIRE(n > 0, Q35_ERR_INVALID_ARG, "argmax: n must be > 0");
  Q35_PTR(x); Q35_PTR(out_index); Q35_PTR(workspace);
  Q35_REQUIRE(workspace_bytes >= argmax_workspace_bytes(), Q35_ERR_WORKSPACE, "argmax: workspace too small");
  if (int rc = require_sm100()) return rc;
  return argmax_launch(n, x, out_index, workspace, static_cast<cudaStream_t>(stream));
}

int q35_q8_dequant(int32_t rows, int32_t cols, const uint32_t *w, const float *scales, float *out, void *stream) {
  Q35_REQUIRE(rows >= 0 && cols > 0 && cols % 64 == 0, Q35_ERR_INVALID_ARG,
              "q8_dequant: rows >= 0, cols a multiple of 64");
  if (rows == 0) return Q35_OK;
  Q35_PTR(w); Q35_PTR(scales); Q35_PTR16(out);
  if (int rc = require_sm100()) return rc;
  return q8_dequant_launch(rows, cols, w, scales, out, static_cast<cudaStream_t>(stream));
}

int q35_rope_gather(int32_t batch, int32_t rot, int32_t max_pos, const int32_t *lens, const float *table_cos,
                    const float *table_sin, float *cos_out, float *sin_out, void *stream) {
  Q35_REQUIRE(batch >= 0 && rot >= 0 && rot <= 1024 && max_pos > 0, Q35_ERR_INVALID_ARG, "rope_gather: bad sizes");
  if (batch == 0 || rot == 0) return Q35_OK;
  Q35_PTR(lens); Q35_PTR(table_cos); Q35_PTR(table_sin); Q35_PTR(cos_out); Q35_PTR(sin_out);
  if (int rc = require_sm100()) return rc;
  return rope_gather_launch(batch, rot, max_pos, lens, table_cos, table_sin, cos_out, sin_out,
                            static_cast<cudaStream_t>(stream));
}

size_t q35_gqa_decode_workspace_size(const q35_gqa_dims *dims, int64_t max_len) {
  if (check_gqa_dims(dims) != Q35_OK || max_len <= 0) return 0;
  return gqa_workspace_bytes(dims->batch, dims->num_q_heads, dims->num_kv_heads, max_len, device_sm_count());
}

int q35_workspace_init(void *workspace, size_t workspace_bytes, void *stream) {
  Q35_PTR(workspace);
  return check_cuda(cudaMemsetAsync(workspace, 0, workspace_bytes, static_cast<cudaStream_t>(stream)),
                    "workspace init");
}

int q35_gqa_decode(const q35_gqa_dims *dims, int64_t max_len, const float *q_gate, const float *k_new,
                   const float *v_new, const float *qn_w, const float *kn_w, const float *cos, const float *sin,
                   float *k_cache, float *v_cache, int32_t *lens, float *out, void *workspace,
                   size_t workspace_bytes, void *stream) {
  if (int rc = gqa_decode_check_args(dims, max_len, q_gate, k_new, v_new, qn_w, kn_w, cos, sin, k_cache, v_cache,
                                     lens, out))
    return rc;
  if (dims->batch == 0) return Q35_OK;
  return gqa_decode_launch(dims, max_len, q_gate, k_new, v_new, qn_w, kn_w, cos, sin, k_cache, v_cache, lens, out,
                           workspace, workspace_bytes, static_cast<cudaStream_t>(stream), nullptr);
}

int q35_gqa_decode_partial(const q35_gqa_dims *dims, int64_t max_len, const float *q_gate, const float *k_new,
                           const float *v_new, const float *qn_w, const float *kn_w, const float *cos,
                           const float *sin, float *k_cache, float *v_cache, int32_t *lens, float *partial_out,
                           void *workspace, size_t workspace_bytes, void *stream) {
  if (int rc = check_gqa_dims(dims)) return rc;
  Q35_REQUIRE(max_len > 0, Q35_ERR_INVALID_ARG, "gqa_decode_partial: max_len must be > 0");
  Q35_REQUIRE(max_len <= dims->capacity, Q35_ERR_CAPACITY, "gqa_decode_partial: max_len exceeds the capacity");
  Q35_REQUIRE((k_new == nullptr) == (v_new == nullptr), Q35_ERR_INVALID_ARG,
              "gqa_decode_partial: k_new and v_new must both be set (append) or both be NULL");
  if (dims->batch == 0) return Q35_OK;
  Q35_PTR16(q_gate); Q35_PTR16(qn_w);
  if (k_new != nullptr) {
    Q35_PTR16(k_new); Q35_PTR16(v_new); Q35_PTR16(kn_w);
  }
  if (dims->rotary_dim > 0) {
    Q35_PTR(cos);
    Q35_PTR(sin);
  }
  Q35_PTR16(k_cache); Q35_PTR16(v_cache); Q35_PTR(lens); Q35_PTR(partial_out);
  if (int rc = require_sm100()) return rc;
  return gqa_decode_launch(dims, max_len, q_gate, k_new, v_new, qn_w, kn_w, cos, sin, k_cache, v_cache, lens,
                           nullptr, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), partial_out);
}

int q35_gqa_combine_partials(int32_t batch, int32_t num_q_heads, int32_t head_dim, int32_t n_parts,
                             const float *parts, const float *q_gate, float *out, void *stream) {
  Q35_REQUIRE(batch >= 0 && num_q_heads > 0 && n_parts > 0, Q35_ERR_INVALID_ARG, "gqa_combine: bad sizes");
  Q35_REQUIRE(head_dim == 256, Q35_ERR_UNSUPPORTED, "gqa_combine: head_dim = 256 is the compiled configuration");
  if (batch == 0) return Q35_OK;
  Q35_PTR(parts); Q35_PTR(q_gate); Q35_PTR(out);
  if (int rc = require_sm100()) return rc;
  return gqa_combine_launch(batch, num_q_heads, n_parts, parts, q_gate, out, static_cast<cudaStream_t>(stream));
}

int q35_workspace_status(void *workspace, uint32_t *status_out, int32_t clear, void *stream) {
  Q35_PTR(workspace);
  Q35_PTR(status_out);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t v = 0;
  if (int rc = check_cuda(cudaMemcpyAsync(&v, workspace, sizeof(v), cudaMemcpyDeviceToHost, st), "status read"))
    return rc;
  if (int rc = check_cuda(cudaStreamSynchronize(st), "status sync")) return rc;
  *status_out = v;
  if (clear) return check_cuda(cudaMemsetAsync(workspace, 0, sizeof(uint32_t), st), "status clear");
  return Q35_OK;
}

size_t q35_gdn_prefill_workspace_size(const q35_gdn_dims *dims, int32_t seq_len) {
  if (check_gdn_dims(dims) != Q35_OK || seq_len <= 0) return 0;
  return gdn_prefill_workspace_bytes(dims, seq_len);
}

int q35_gdn_prefill(const q35_gdn_dims *dims, int32_t seq_len, const float *mixed_qkv, const float *z,
                    const float *beta, const float *g, const float *conv_w, const float *norm_w, float *conv_state,
                    int32_t has_prev_conv, float *rec_state, int32_t has_init_state, float *out, void *workspace,
                    size_t workspace_bytes, void *stream) {
  if (int rc = check_gdn_dims(dims)) return rc;
  Q35_REQUIRE(seq_len >= 0, Q35_ERR_INVALID_ARG, "gdn_prefill: seq_len must be >= 0");
  Q35_REQUIRE(has_prev_conv == 0 || has_prev_conv == 1, Q35_ERR_INVALID_ARG, "has_prev_conv must be 0 or 1");
  Q35_REQUIRE(has_init_state == 0 || has_init_state == 1, Q35_ERR_INVALID_ARG, "has_init_state must be 0 or 1");
  if (dims->batch == 0 || seq_len == 0) return Q35_OK;
  Q35_PTR(beta); Q35_PTR(g); Q35_PTR(conv_w); Q35_PTR(conv_state);
  Q35_PTR16(mixed_qkv); Q35_PTR16(z); Q35_PTR16(norm_w); Q35_PTR16(out); Q35_PTR16(rec_state);
  if (int rc = require_sm100()) return rc;
  return gdn_prefill_launch(dims, seq_len, mixed_qkv, z, beta, g, conv_w, norm_w, conv_state, has_prev_conv,
                            rec_state, has_init_state, out, workspace, workspace_bytes,
                            static_cast<cudaStream_t>(stream));
}

}  // extern "C"
