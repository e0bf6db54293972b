// q35_modules.cpp -- the C++ host layer of q35_modules.hpp: argument checks,
// cache-slot bookkeeping and the prefill / decode dispatch of the reference's
// modules, on top of the C ABI.
#include "q35_modules.hpp"

#include <cuda_runtime.h>

#include <utility>

namespace q35 {
namespace host {

Error::Error(int code, const std::string &msg) : std::runtime_error(msg), code_(code) {}

void check(int rc) {
  if (rc != Q35_OK) throw Error(rc, std::string("q35attn: ") + q35_last_error());
}

static void check_cuda(cudaError_t e, const char *what) {
  if (e != cudaSuccess) throw Error(Q35_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

static void require(bool ok, int code, const std::string &msg) {
  if (!ok) throw Error(code, msg);
}

// ---------------------------------------------------------------- DeviceBuffer
DeviceBuffer::DeviceBuffer(size_t bytes) { reserve(bytes); }
DeviceBuffer::~DeviceBuffer() {
  if (ptr_) cudaFree(ptr_);
}
DeviceBuffer::DeviceBuffer(DeviceBuffer &&o) noexcept : ptr_(o.ptr_), bytes_(o.bytes_) {
  o.ptr_ = nullptr;
  o.bytes_ = 0;
}
DeviceBuffer &DeviceBuffer::operator=(DeviceBuffer &&o) noexcept {
  if (this != &o) {
    if (ptr_) cudaFree(ptr_);
    ptr_ = o.ptr_;
    bytes_ = o.bytes_;
    o.ptr_ = nullptr;
    o.bytes_ = 0;
  }
  return *this;
}
void DeviceBuffer::reserve(size_t bytes) {
  if (bytes <= bytes_) return;
  if (ptr_) check_cuda(cudaFree(ptr_), "cudaFree");
  ptr_ = nullptr;
  bytes_ = 0;
  check_cuda(cudaMalloc(&ptr_, bytes), "cudaMalloc");
  bytes_ = bytes;
}

// ---------------------------------------------------------------- Cache
Cache::Cache(const TextConfig &cfg, int num_layers, int batch, int64_t max_len)
    : cfg_(cfg), batch_(batch), max_len_(max_len), slots_((size_t)(num_layers > 0 ? num_layers : 0)) {
  require(num_layers > 0 && batch > 0 && max_len > 0, Q35_ERR_INVALID_ARG,
          "Cache: num_layers, batch and max_len must be > 0");
}

Cache::Slot &Cache::slot(int layer) {
  require(layer >= 0 && layer < (int)slots_.size(), Q35_ERR_INVALID_ARG, "Cache: layer index out of range");
  return slots_[(size_t)layer];
}
const Cache::Slot &Cache::slot(int layer) const {
  require(layer >= 0 && layer < (int)slots_.size(), Q35_ERR_INVALID_ARG, "Cache: layer index out of range");
  return slots_[(size_t)layer];
}

bool Cache::has_conv_state(int layer) const { return slot(layer).conv_set; }
bool Cache::has_recurrent_state(int layer) const { return slot(layer).rec_set; }
bool Cache::has_kv(int layer) const { return slot(layer).kv_set; }

float *Cache::conv_state(int layer) {
  Slot &s = slot(layer);
  s.conv.reserve((size_t)batch_ * cfg_.conv_dim() * (cfg_.linear_conv_kernel_dim - 1) * sizeof(float));
  return s.conv.as<float>();
}
float *Cache::recurrent_state(int layer) {
  Slot &s = slot(layer);
  s.rec.reserve((size_t)batch_ * cfg_.linear_num_value_heads * cfg_.linear_key_head_dim *
                cfg_.linear_value_head_dim * sizeof(float));
  return s.rec.as<float>();
}
float *Cache::key_states(int layer) {
  Slot &s = slot(layer);
  s.k.reserve((size_t)batch_ * cfg_.num_key_value_heads * (size_t)max_len_ * cfg_.head_dim * sizeof(float));
  return s.k.as<float>();
}
float *Cache::value_states(int layer) {
  Slot &s = slot(layer);
  s.v.reserve((size_t)batch_ * cfg_.num_key_value_heads * (size_t)max_len_ * cfg_.head_dim * sizeof(float));
  return s.v.as<float>();
}
int32_t *Cache::lengths(int layer) {
  Slot &s = slot(layer);
  const bool fresh = s.lens.data() == nullptr;
  s.lens.reserve((size_t)batch_ * sizeof(int32_t));
  if (fresh) check_cuda(cudaMemset(s.lens.data(), 0, (size_t)batch_ * sizeof(int32_t)), "cudaMemset");
  return s.lens.as<int32_t>();
}
std::vector<int32_t> Cache::host_lengths(int layer, void *stream) {
  std::vector<int32_t> h((size_t)batch_);
  int32_t *d = lengths(layer);
  auto st = static_cast<cudaStream_t>(stream);
  check_cuda(cudaMemcpyAsync(h.data(), d, h.size() * sizeof(int32_t), cudaMemcpyDeviceToHost, st), "cudaMemcpy");
  check_cuda(cudaStreamSynchronize(st), "cudaStreamSynchronize");
  return h;
}

// ---------------------------------------------------------------- GatedDeltaNetCore
GatedDeltaNetCore::GatedDeltaNetCore(const TextConfig &cfg, int layer_idx, const float *conv_w,
                                     const float *norm_w)
    : cfg_(cfg), layer_(layer_idx), conv_w_(conv_w), norm_w_(norm_w) {
  require(conv_w != nullptr && norm_w != nullptr, Q35_ERR_INVALID_ARG,
          "GatedDeltaNetCore: conv_w and norm_w are required");
}

q35_gdn_dims GatedDeltaNetCore::dims(int batch) const {
  q35_gdn_dims d;
  d.batch = batch;
  d.num_k_heads = cfg_.linear_num_key_heads;
  d.num_v_heads = cfg_.linear_num_value_heads;
  d.head_k_dim = cfg_.linear_key_head_dim;
  d.head_v_dim = cfg_.linear_value_head_dim;
  d.conv_kernel = cfg_.linear_conv_kernel_dim;
  d.eps = cfg_.rms_norm_eps;
  return d;
}

void GatedDeltaNetCore::forward(const float *mixed_qkv, const float *z, const float *beta, const float *g, int batch,
                                int seq_len, Cache *cache, float *out, void *stream) {
  require(batch > 0 && seq_len > 0, Q35_ERR_INVALID_ARG, "GatedDeltaNet: batch and seq_len must be > 0");
  require(cache == nullptr || cache->batch() == batch, Q35_ERR_INVALID_ARG,
          "GatedDeltaNet: cache batch does not match");
  const q35_gdn_dims d = dims(batch);
  // use_precomputed_states = the layer's conv state is cached (:511-513)
  const bool precomputed = cache != nullptr && cache->has_conv_state(layer_);
  float *conv, *rec;
  if (cache) {
    conv = cache->conv_state(layer_);
    rec = cache->recurrent_state(layer_);
  } else {  // cache: None -- the states live only for this call
    scratch_conv_.reserve((size_t)batch * cfg_.conv_dim() * (cfg_.linear_conv_kernel_dim - 1) * sizeof(float));
    scratch_rec_.reserve((size_t)batch * cfg_.linear_num_value_heads * cfg_.linear_key_head_dim *
                         cfg_.linear_value_head_dim * sizeof(float));
    conv = scratch_conv_.as<float>();
    rec = scratch_rec_.as<float>();
  }
  if (precomputed && seq_len == 1) {  // causal_conv1d_update + burn_recurrent_gated_delta_rule (:515-530, 627-636)
    check(q35_gdn_decode(&d, mixed_qkv, z, beta, g, conv_w_, norm_w_, conv, rec, out, stream));
  } else {  // causal_conv1d_fn + burn_chunk_gated_delta_rule (:531-552, 637-646)
    const int has_init = precomputed && cache->has_recurrent_state(layer_);
    const size_t need = q35_gdn_prefill_workspace_size(&d, seq_len);
    require(need > 0, Q35_ERR_INVALID_ARG, "GatedDeltaNet: invalid shape for the chunked path");
    const size_t had = ws_.bytes();
    ws_.reserve(need);
    if (ws_.bytes() != had) check(q35_workspace_init(ws_.data(), 256, stream));  // a fresh status word
    check(q35_gdn_prefill(&d, seq_len, mixed_qkv, z, beta, g, conv_w_, norm_w_, conv, precomputed ? 1 : 0, rec,
                          has_init, out, ws_.data(), ws_.bytes(), stream));
  }
  if (cache) {  // the layer's slots now hold this call's final states (:538-540, 650-652)
    Cache::Slot &s = cache->slot(layer_);
    s.conv_set = true;
    s.rec_set = true;
  }
}

// ---------------------------------------------------------------- AttentionCore
AttentionCore::AttentionCore(const TextConfig &cfg, int layer_idx, const float *q_norm_w, const float *k_norm_w)
    : cfg_(cfg), layer_(layer_idx), qn_w_(q_norm_w), kn_w_(k_norm_w) {
  require(q_norm_w != nullptr && k_norm_w != nullptr, Q35_ERR_INVALID_ARG,
          "AttentionCore: q_norm and k_norm weights are required");
}

q35_gqa_dims AttentionCore::dims(int batch, int64_t capacity) const {
  q35_gqa_dims d;
  d.batch = batch;
  d.num_q_heads = cfg_.num_attention_heads;
  d.num_kv_heads = cfg_.num_key_value_heads;
  d.head_dim = cfg_.head_dim;
  d.rotary_dim = cfg_.rotary_dim;
  d.reserved = 0;
  d.capacity = capacity;
  d.eps = cfg_.rms_norm_eps;
  return d;
}

void AttentionCore::forward(const float *q_gate, const float *k_new, const float *v_new, const float *cos,
                            const float *sin, int batch, int seq_len, Cache &cache, float *out, void *stream) {
  require(batch > 0 && seq_len > 0, Q35_ERR_INVALID_ARG, "Attention: batch and seq_len must be > 0");
  require(cache.batch() == batch, Q35_ERR_INVALID_ARG, "Attention: cache batch does not match");
  const int64_t cap = cache.max_len();
  const q35_gqa_dims d = dims(batch, cap);
  float *K = cache.key_states(layer_), *V = cache.value_states(layer_);
  int32_t *lens = cache.lengths(layer_);
  if (seq_len == 1) {  // one new token against the cached keys (:899-936)
    if (decode_ws_len_ != cap || decode_ws_batch_ != batch) {
      const size_t need = q35_gqa_decode_workspace_size(&d, cap);
      require(need > 0, Q35_ERR_INVALID_ARG, "Attention: invalid shape for decode");
      decode_ws_ = DeviceBuffer(need);  // fresh: the counters must start zeroed
      check(q35_workspace_init(decode_ws_.data(), need, stream));
      decode_ws_len_ = cap;
      decode_ws_batch_ = batch;
    }
    check(q35_gqa_decode(&d, cap, q_gate, k_new, v_new, qn_w_, kn_w_, cos, sin, K, V, lens, out, decode_ws_.data(),
                         decode_ws_.bytes(), stream));
  } else {  // the prompt, causal over the cached keys and itself (mask of model.rs:59-67)
    const size_t need = q35_gqa_prefill_workspace_size(&d, seq_len, cap);
    require(need > 0, Q35_ERR_INVALID_ARG, "Attention: invalid shape for prefill");
    prefill_ws_.reserve(need);
    check(q35_gqa_prefill(&d, seq_len, cap, q_gate, k_new, v_new, qn_w_, kn_w_, cos, sin, K, V, lens, out,
                          prefill_ws_.data(), prefill_ws_.bytes(), stream));
  }
  cache.slot(layer_).kv_set = true;
}

void AttentionCore::check_status(void *stream) {
  if (decode_ws_.data() == nullptr) return;
  uint32_t status = 0;
  check(q35_workspace_status(decode_ws_.data(), &status, 1, stream));
  if (status & Q35_STATUS_CACHE_FULL) throw Error(Q35_ERR_CAPACITY, "Attention: KV cache full, a decode step was skipped");
  if (status & Q35_STATUS_LEN_HINT)
    throw Error(Q35_ERR_CAPACITY, "Attention: length beyond the planned maximum, a decode step was skipped");
  if (status) throw Error(Q35_ERR_CUDA, "Attention: decode reported device status " + std::to_string(status));
}

}  // namespace host
}  // namespace q35
