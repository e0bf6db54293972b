// gqa_decode_noalloc.cu -- q35_gqa_decode for callers that cannot allocate.
//
// Some hosts of this library cannot hand it a workspace: an inference engine
// that reserves all device memory once at start-up and forbids cudaMalloc
// while serving (an allocation there can synchronize the device and fragment
// the reserved pool), or a thin FFI binding whose host language has no device
// allocator of its own.  This entry point runs the same split-K flash-decode
// kernel as q35_gqa_decode, but its scratch (split partials, arrival counters,
// status word) lives in a fixed array inside the library instead of a
// caller-provided workspace.
//
// Properties the caller must know:
//  * the array is kNoAllocScratchBytes (16 MiB) per GPU, reserved on every GPU
//    that loads the library until the process exits;
//  * a call needs q35_gqa_decode_workspace_size(dims, max_len) bytes of it and
//    is rejected with Q35_ERR_WORKSPACE when that is larger;
//  * every call uses the same array: calls whose kernels overlap on the GPU
//    (different streams, or several host threads) race and corrupt each
//    other's results;
//  * the first call on a device resolves the array's device address
//    (cudaGetSymbolAddress) with that device current; make that first call
//    before any stream capture;
//  * the counters and status word must start at zero, so each call clears
//    them with an asynchronous memset on `stream` before the launch (the array
//    otherwise keeps the previous call's contents);
//  * the device-side status word (Q35_STATUS_* bits: a full cache, a length
//    hint exceeded, a bounded wait that gave up) lives in the private array
//    and is cleared by the next call, so it cannot be read by the caller.  A
//    skipped sequence shows only as lens[b] left unchanged.  Callers that need
//    the status bits use q35_gqa_decode with a workspace and
//    q35_workspace_status.
#include <mutex>

#include "common.cuh"

namespace q35 {

size_t gqa_workspace_counter_bytes(int B, int Hq, int Hkv, long long max_len, int sms);
int gqa_decode_check_args(const q35_gqa_dims *dims, int64_t max_len, const float *q_gate, const float *k_new,
                          const float *v_new, const float *qn_w, const float *kn_w, const float *cos,
                          const float *sin, const float *k_cache, const float *v_cache, const int32_t *lens,
                          const float *out);
int gqa_decode_launch(const q35_gqa_dims *d, long long max_len, const float *q_gate, const float *k_new,
                      const float *v_new, const float *qn_w, const float *kn_w, const float *cos,
                      const float *sin, float *k_cache, float *v_cache, int32_t *lens, float *out,
                      void *ws, size_t ws_bytes, cudaStream_t st, float *part_out);

namespace {

constexpr size_t kNoAllocScratchBytes = 16u << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void *g_scratch_ptr[64] = {nullptr};  // device address of g_noalloc_scratch, per device

// Device address of the scratch array on the current device (resolved once
// per device; the host-side symbol itself is not a device address).
int scratch_for_current_device(void **out) {
  int dev = -1;
  if (int rc = check_cuda(cudaGetDevice(&dev), "noalloc: cudaGetDevice")) return rc;
  Q35_REQUIRE(dev >= 0 && dev < 64, Q35_ERR_DEVICE, "noalloc: device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void *p = nullptr;
    if (int rc = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch), "noalloc: cudaGetSymbolAddress"))
      return rc;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return Q35_OK;
}

}  // namespace
}  // namespace q35

using namespace q35;

extern "C" int q35_gqa_decode_noalloc(const q35_gqa_dims *dims, int64_t max_len, const float *q_gate,
                                      const float *k_new, const float *v_new, const float *qn_w, const float *kn_w,
                                      const float *cos, const float *sin, float *k_cache, float *v_cache,
                                      int32_t *lens, float *out, void *stream) {
  // Every argument check runs before anything is queued on `stream`, so a
  // rejected call leaves the stream (or a graph being captured) untouched and
  // does not clear the counters of a call still running elsewhere.
  if (int rc = gqa_decode_check_args(dims, max_len, q_gate, k_new, v_new, qn_w, kn_w, cos, sin, k_cache, v_cache,
                                     lens, out))
    return rc;
  if (dims->batch == 0) return Q35_OK;
  const int sms = device_sm_count();
  const size_t need = q35_gqa_decode_workspace_size(dims, max_len);
  Q35_REQUIRE(need <= kNoAllocScratchBytes, Q35_ERR_WORKSPACE,
              "gqa_decode_noalloc: this call needs " + std::to_string(need) +
                  " bytes of scratch, above the fixed " + std::to_string(kNoAllocScratchBytes) +
                  "-byte array; use q35_gqa_decode with a workspace");
  void *scratch = nullptr;
  if (int rc = scratch_for_current_device(&scratch)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // status word + split / group / pair / sequence counters must start at zero
  const size_t counters = gqa_workspace_counter_bytes(dims->batch, dims->num_q_heads, dims->num_kv_heads, max_len,
                                                      sms);
  if (int rc = check_cuda(cudaMemsetAsync(scratch, 0, counters, st), "gqa_decode_noalloc: clear counters"))
    return rc;
  return gqa_decode_launch(dims, max_len, q_gate, k_new, v_new, qn_w, kn_w, cos, sin, k_cache, v_cache, lens, out,
                           scratch, kNoAllocScratchBytes, st, nullptr);
}
