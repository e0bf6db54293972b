// q35_modules.hpp -- C++ host layer above the C ABI (include/q35attn.h),
// mirroring the attention modules of inventwithdean/Qwen-3.5
// src/text_modules.rs between their projections:
//
//   Cache             text_modules.rs:445-461 (per-layer conv / recurrent /
//                     key / value slots, empty until a layer's first forward)
//   GatedDeltaNetCore GatedDeltaNet::forward (:484-667) from mixed_qkv, z,
//                     beta, g to the RMSNormGated output: causal conv1d update
//                     (decode) or conv1d fn (prefill), q/k/v split and head
//                     expansion, l2norm, the recurrent gated delta rule when
//                     seq_len == 1 and the layer's conv state is cached, the
//                     chunked rule (chunk 64) otherwise, RMSNormGated.
//   AttentionCore     Attention::forward (:842-944) from the q_proj output
//                     (query | gate per head), k and v to the gated output:
//                     q/k RMSNorm, partial RoPE, the KV-cache append, GQA
//                     attention (causal over the cache), sigmoid gate.
//
// All tensors are f32 device pointers in the reference's layouts (row-major,
// batch first).  Where the reference panics, these classes throw
// q35::host::Error carrying the library's status code and message.  Calls are
// stream-ordered; a Cache and a core object must not be used from two
// threads at once.
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "q35attn.h"

namespace q35 {
namespace host {

class Error : public std::runtime_error {
 public:
  Error(int code, const std::string &msg);
  int code() const { return code_; }

 private:
  int code_;
};

// Throws Error with q35_last_error() when rc != Q35_OK.
void check(int rc);

// The text_config.rs fields this path uses (defaults: the 2B model,
// text_config.rs:65-122).
struct TextConfig {
  int hidden_size = 2048;
  int linear_num_key_heads = 16;
  int linear_num_value_heads = 16;
  int linear_key_head_dim = 128;
  int linear_value_head_dim = 128;
  int linear_conv_kernel_dim = 4;
  int num_attention_heads = 8;
  int num_key_value_heads = 2;
  int head_dim = 256;
  int rotary_dim = 64;  // partial_rotary_factor 0.25 of head_dim
  float rms_norm_eps = 1e-6f;

  int conv_dim() const {
    return 2 * linear_num_key_heads * linear_key_head_dim + linear_num_value_heads * linear_value_head_dim;
  }
};

// Owning device allocation (cudaMalloc), move-only.
class DeviceBuffer {
 public:
  DeviceBuffer() = default;
  explicit DeviceBuffer(size_t bytes);
  ~DeviceBuffer();
  DeviceBuffer(DeviceBuffer &&o) noexcept;
  DeviceBuffer &operator=(DeviceBuffer &&o) noexcept;
  DeviceBuffer(const DeviceBuffer &) = delete;
  DeviceBuffer &operator=(const DeviceBuffer &) = delete;
  void *data() const { return ptr_; }
  size_t bytes() const { return bytes_; }
  template <class T>
  T *as() const {
    return static_cast<T *>(ptr_);
  }
  // Ensures at least `bytes`; the contents are not kept when it grows.
  void reserve(size_t bytes);

 private:
  void *ptr_ = nullptr;
  size_t bytes_ = 0;
};

// Cache::new(num_layers) (text_modules.rs:452-460).  The key/value slots of an
// attention layer hold `max_len` tokens per sequence (the reference
// concatenates; here the cache is preallocated and appended in place).
class Cache {
 public:
  Cache(const TextConfig &cfg, int num_layers, int batch, int64_t max_len);

  int num_layers() const { return (int)slots_.size(); }
  int batch() const { return batch_; }
  int64_t max_len() const { return max_len_; }
  // conv_states[layer].is_some() -- decides the decode branch (:511-515)
  bool has_conv_state(int layer) const;
  bool has_recurrent_state(int layer) const;
  bool has_kv(int layer) const;

  // Device views of a layer's slots (allocated on first use).
  float *conv_state(int layer);       // [batch, conv_dim, K-1]
  float *recurrent_state(int layer);  // [batch, Hv, dk, dv]
  float *key_states(int layer);       // [batch, Hkv, max_len, head_dim]
  float *value_states(int layer);     // [batch, Hkv, max_len, head_dim]
  int32_t *lengths(int layer);        // [batch] tokens cached per sequence
  // Copies the per-sequence cached lengths of an attention layer to the host.
  std::vector<int32_t> host_lengths(int layer, void *stream = nullptr);

 private:
  friend class GatedDeltaNetCore;
  friend class AttentionCore;
  struct Slot {
    DeviceBuffer conv, rec, k, v, lens;
    bool conv_set = false, rec_set = false, kv_set = false;
  };
  Slot &slot(int layer);
  const Slot &slot(int layer) const;
  TextConfig cfg_;
  int batch_;
  int64_t max_len_;
  std::vector<Slot> slots_;
};

class GatedDeltaNetCore {
 public:
  // conv_w [conv_dim, K] and norm_w [dv] are device pointers owned by the caller.
  GatedDeltaNetCore(const TextConfig &cfg, int layer_idx, const float *conv_w, const float *norm_w);

  // mixed_qkv [B, T, conv_dim], z [B, T, Hv * dv], beta and g [B, T, Hv];
  // out [B, T, Hv * dv].  cache == nullptr is the reference's `cache: None`:
  // no state is read or kept (the chunked rule from zero state).
  void forward(const float *mixed_qkv, const float *z, const float *beta, const float *g, int batch, int seq_len,
               Cache *cache, float *out, void *stream);

 private:
  q35_gdn_dims dims(int batch) const;
  TextConfig cfg_;
  int layer_;
  const float *conv_w_, *norm_w_;
  DeviceBuffer ws_, scratch_conv_, scratch_rec_;
};

class AttentionCore {
 public:
  // q_norm_w, k_norm_w [head_dim] (used as 1 + w) are device pointers owned by the caller.
  AttentionCore(const TextConfig &cfg, int layer_idx, const float *q_norm_w, const float *k_norm_w);

  // q_gate [B, T, Hq, 2 * head_dim] (per head: query | gate, :866-874),
  // k_new and v_new [B, T, Hkv, head_dim] (before norm / RoPE), cos and sin
  // [B, T, rotary_dim] for positions lens[b] .. lens[b] + T - 1; out [B, T, Hq *
  // head_dim].  The new keys and values are appended to the cache.
  void forward(const float *q_gate, const float *k_new, const float *v_new, const float *cos, const float *sin,
               int batch, int seq_len, Cache &cache, float *out, void *stream);

  // Reads and clears the device status of the decode steps issued so far
  // (synchronises `stream`): throws Error(Q35_ERR_CAPACITY) if a step was
  // skipped because a sequence's cache was full -- where the reference would
  // panic on the concatenation -- and Error(Q35_ERR_CUDA) on a device wait
  // that gave up.  Kept out of forward() so decode steps stay capturable.
  void check_status(void *stream);

 private:
  q35_gqa_dims dims(int batch, int64_t capacity) const;
  TextConfig cfg_;
  int layer_;
  const float *qn_w_, *kn_w_;
  DeviceBuffer decode_ws_, prefill_ws_;
  int64_t decode_ws_len_ = -1;
  int decode_ws_batch_ = -1;
};

}  // namespace host
}  // namespace q35
