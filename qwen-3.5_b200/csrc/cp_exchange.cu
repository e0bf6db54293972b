// cp_exchange.cu -- the exchange step of one long sequence decoded across the
// GPUs of a node (BASELINE config 4's single-sequence variant), over peer
// memory instead of collectives.
//
// Each rank holds a shard of the work of text_modules.rs:
//   * GatedDeltaNet (:483-667), heads-parallel: rank r computes the outputs of
//     its value heads, n_gdn floats per sequence (the input of out_proj is the
//     concatenation over ranks, in rank order);
//   * Attention (:899-928) with the KV cache split along its length: rank r
//     computes, per query head, the unnormalised softmax partial
//     [o (D) | m (log2 units) | l] over its keys (q35_gqa_decode_partial).
// q35_cp_exchange gives every rank the full GDN output and the merged, gated
// attention output in one kernel:
//   1. the CTA stores this rank's payload (GDN outputs + partials) straight
//      into slot [rank] of every peer's receive buffer (plain peer stores over
//      NVLink; no multicast), then, after a system-scope fence, publishes the
//      step's epoch in each peer's flag array (release);
//   2. thread 0 waits (bounded) until every rank's flag in its own array holds
//      the epoch (acquire);
//   3. the CTA merges the partials of every rank (the flash-decode combine of
//      the split keys, then sigmoid(gate)) and concatenates the GDN outputs.
// The receive buffer has two halves selected by the epoch's parity: a rank can
// only start step e+1 after every rank posted step e, so the half of step e-1
// that a fast rank overwrites is no longer read.  The epoch is a counter in
// this rank's own buffer, advanced by the kernel, so captured steps replay.
// A wait that gives up (a rank never arrived within 1 s) sets
// Q35_STATUS_WAIT_TIMEOUT in the context's status word and poisons the outputs
// with NaN; the epochs of the ranks then disagree, so the caller treats the
// context as broken (tears it down and creates a new one).
//
// The receive buffers are allocated once (q35_cp_create) and mapped by the
// peers through CUDA IPC handles (q35_cp_connect); the exchange itself
// allocates nothing.
#include <cstring>
#include <string>

#include "common.cuh"

namespace q35 {
namespace {

constexpr int kCpMaxWorld = 8;
constexpr int kCpThreads = 512;
constexpr int kD = 256;
constexpr uint64_t kCpWaitNs = 1000000000ull;  // 1 s

struct CpCtx {
  int world, rank, batch, n_gdn, hq;
  size_t payload;          // floats per rank per half
  unsigned char *base;     // this rank's buffer (cudaMalloc)
  size_t bytes;
  unsigned char *peer[kCpMaxWorld];  // every rank's buffer as mapped here (peer[rank] = base)
  bool connected;
};

// Buffer layout: [2 halves][world][payload] floats, then (256-byte aligned)
// flags[world] u32, epoch u32, status u32.
size_t cp_flags_offset(const CpCtx &c) {
  const size_t data = 2 * (size_t)c.world * c.payload * sizeof(float);
  return (data + 255) / 256 * 256;
}

struct CpParams {
  float *peer_data[kCpMaxWorld];     // peers' receive buffers (data region)
  uint32_t *peer_flags[kCpMaxWorld];  // peers' flag arrays
  float *my_data;
  uint32_t *my_flags, *epoch, *status;
  const float *gdn_local, *gqa_part, *q_gate;
  float *gdn_full, *gqa_out;
  int world, rank, batch, n_gdn, hq;
  long long payload;
  uint64_t wait_ns;
  int fault;  // test hook: publish no arrival flags
};

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kCpThreads) cp_exchange_kernel(const CpParams p) {
  pdl_entry();
  __shared__ uint32_t s_epoch;
  __shared__ int s_ok;
  const int tid = threadIdx.x;
  if (tid == 0) {
    s_epoch = *p.epoch + 1u;
    *p.epoch = s_epoch;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int half = (int)(epoch & 1u);
  const long long pay = p.payload;
  const long long ng = (long long)p.batch * p.n_gdn;      // GDN floats of this rank
  const long long np = (long long)p.batch * p.hq * (kD + 2);  // partial floats
  // 1. payload -> slot [rank] of every rank's buffer (float4 when aligned)
  for (int r = 0; r < p.world; ++r) {
    float *dst = p.peer_data[r] + ((long long)half * p.world + p.rank) * pay;
    for (long long i = tid; i < ng; i += kCpThreads) dst[i] = p.gdn_local[i];
    for (long long i = tid; i < np; i += kCpThreads) dst[ng + i] = p.gqa_part[i];
  }
  __threadfence_system();
  __syncthreads();
  if (tid == 0) {
    if (!p.fault)
      for (int r = 0; r < p.world; ++r) st_release_sys(p.peer_flags[r] + p.rank, epoch);
    // 2. every rank's payload of this epoch is in our buffer
    bool ok = true;
    const uint64_t t0 = globaltimer_ns();
    for (int r = 0; r < p.world && ok; ++r) {
      while ((int)(ld_acquire_sys(p.my_flags + r) - epoch) < 0) {
        if (globaltimer_ns() - t0 > p.wait_ns) {
          ok = false;
          atomicOr(p.status, Q35_STATUS_WAIT_TIMEOUT);
          break;
        }
      }
    }
    s_ok = ok ? 1 : 0;
  }
  __syncthreads();
  const bool ok = s_ok != 0;
  const float *mine = p.my_data + (long long)half * p.world * pay;
  // 3a. GDN outputs, rank order: gdn_full[b][r * n_gdn + j]
  const long long gtot = (long long)p.world * ng;
  for (long long i = tid; i < gtot; i += kCpThreads) {
    const int b = (int)(i / ((long long)p.world * p.n_gdn));
    const long long rem = i % ((long long)p.world * p.n_gdn);
    const int r = (int)(rem / p.n_gdn), j = (int)(rem % p.n_gdn);
    p.gdn_full[i] = ok ? __ldcv(mine + (long long)r * pay + (long long)b * p.n_gdn + j) : __int_as_float(0x7fc00000);
  }
  // 3b. merge the partials of every rank per (sequence, head, dim)
  const long long otot = (long long)p.batch * p.hq * kD;
  for (long long i = tid; i < otot; i += kCpThreads) {
    const int d = (int)(i % kD);
    const long long bh = i / kD;  // b * hq + h
    float M = -INFINITY;
    for (int r = 0; r < p.world; ++r)
      M = fmaxf(M, __ldcv(mine + (long long)r * pay + ng + bh * (kD + 2) + kD));
    float L = 0.0f, O = 0.0f;
    for (int r = 0; r < p.world; ++r) {
      const float *pr = mine + (long long)r * pay + ng + bh * (kD + 2);
      const float m = __ldcv(pr + kD);
      const float w = m == -INFINITY ? 0.0f : exp2f(m - M);  // a shard without keys adds nothing
      L = fmaf(__ldcv(pr + kD + 1), w, L);
      O = fmaf(__ldcv(pr + d), w, O);
    }
    const float gate = p.q_gate[bh * 2 * kD + kD + d];
    p.gqa_out[i] = ok ? (O / L) * sigmoidf_dev(gate) : __int_as_float(0x7fc00000);
  }
}

}  // namespace
}  // namespace q35

using namespace q35;

extern "C" {

int q35_cp_create(int32_t world, int32_t rank, int32_t batch, int32_t n_gdn, int32_t num_q_heads,
                  int32_t head_dim, void **ctx_out, void *ipc_handle_out) {
  Q35_REQUIRE(ctx_out != nullptr && ipc_handle_out != nullptr, Q35_ERR_INVALID_ARG, "cp_create: NULL output");
  Q35_REQUIRE(world >= 1 && world <= kCpMaxWorld && rank >= 0 && rank < world, Q35_ERR_INVALID_ARG,
              "cp_create: world must be 1..8 and rank in [0, world)");
  Q35_REQUIRE(batch >= 1 && n_gdn >= 0 && num_q_heads >= 1, Q35_ERR_INVALID_ARG, "cp_create: bad sizes");
  Q35_REQUIRE(head_dim == kD, Q35_ERR_UNSUPPORTED, "cp_create: head_dim = 256 is the compiled configuration");
  if (int rc = require_sm100()) return rc;
  CpCtx *c = new CpCtx();
  c->world = world;
  c->rank = rank;
  c->batch = batch;
  c->n_gdn = n_gdn;
  c->hq = num_q_heads;
  c->payload = (size_t)batch * n_gdn + (size_t)batch * num_q_heads * (kD + 2);
  c->bytes = cp_flags_offset(*c) + 256;
  if (cudaMalloc(&c->base, c->bytes) != cudaSuccess) {
    delete c;
    return fail(Q35_ERR_CUDA, "cp_create: cudaMalloc of the receive buffer failed");
  }
  if (int rc = check_cuda(cudaMemset(c->base, 0, c->bytes), "cp_create: clear")) {
    cudaFree(c->base);
    delete c;
    return rc;
  }
  cudaIpcMemHandle_t h;
  if (int rc = check_cuda(cudaIpcGetMemHandle(&h, c->base), "cp_create: cudaIpcGetMemHandle")) {
    cudaFree(c->base);
    delete c;
    return rc;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  std::memcpy(ipc_handle_out, &h, 64);
  for (int r = 0; r < kCpMaxWorld; ++r) c->peer[r] = nullptr;
  c->peer[rank] = c->base;
  c->connected = world == 1;
  *ctx_out = c;
  return Q35_OK;
}

int q35_cp_connect(void *ctx, const void *ipc_handles) {
  Q35_REQUIRE(ctx != nullptr && ipc_handles != nullptr, Q35_ERR_INVALID_ARG, "cp_connect: NULL argument");
  CpCtx *c = static_cast<CpCtx *>(ctx);
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank || c->peer[r] != nullptr) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const unsigned char *>(ipc_handles) + 64 * r, 64);
    void *p = nullptr;
    if (int rc = check_cuda(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess),
                            "cp_connect: cudaIpcOpenMemHandle"))
      return rc;
    c->peer[r] = static_cast<unsigned char *>(p);
  }
  c->connected = true;
  return Q35_OK;
}

int q35_cp_exchange(void *ctx, const float *gdn_local, const float *gqa_part, const float *q_gate, float *gdn_full,
                    float *gqa_out, void *stream) {
  Q35_REQUIRE(ctx != nullptr, Q35_ERR_INVALID_ARG, "cp_exchange: ctx is NULL");
  CpCtx *c = static_cast<CpCtx *>(ctx);
  Q35_REQUIRE(c->connected, Q35_ERR_INVALID_ARG, "cp_exchange: q35_cp_connect has not run");
  Q35_REQUIRE(gqa_part != nullptr && q_gate != nullptr && gqa_out != nullptr, Q35_ERR_INVALID_ARG,
              "cp_exchange: NULL pointer");
  Q35_REQUIRE(c->n_gdn == 0 || (gdn_local != nullptr && gdn_full != nullptr), Q35_ERR_INVALID_ARG,
              "cp_exchange: NULL GDN pointer");
  CpParams p = {};
  const size_t fo = cp_flags_offset(*c);
  for (int r = 0; r < c->world; ++r) {
    p.peer_data[r] = reinterpret_cast<float *>(c->peer[r]);
    p.peer_flags[r] = reinterpret_cast<uint32_t *>(c->peer[r] + fo);
  }
  p.my_data = reinterpret_cast<float *>(c->base);
  p.my_flags = reinterpret_cast<uint32_t *>(c->base + fo);
  p.epoch = p.my_flags + c->world;
  p.status = p.epoch + 1;
  p.gdn_local = gdn_local;
  p.gqa_part = gqa_part;
  p.q_gate = q_gate;
  p.gdn_full = gdn_full;
  p.gqa_out = gqa_out;
  p.world = c->world;
  p.rank = c->rank;
  p.batch = c->batch;
  p.n_gdn = c->n_gdn;
  p.hq = c->hq;
  p.payload = (long long)c->payload;
  p.fault = take_fault(kFaultCpExchange) ? 1 : 0;
  p.wait_ns = p.fault ? kFaultWaitLimitNs : kCpWaitNs;
  note_launch();
  (void)launch_kernel(cp_exchange_kernel, dim3(1), dim3(kCpThreads), 0, static_cast<cudaStream_t>(stream), 1, 1, p);
  return check_cuda(cudaGetLastError(), "cp_exchange launch");
}

int q35_cp_status(void *ctx, uint32_t *status_out, int32_t clear, void *stream) {
  Q35_REQUIRE(ctx != nullptr && status_out != nullptr, Q35_ERR_INVALID_ARG, "cp_status: NULL argument");
  CpCtx *c = static_cast<CpCtx *>(ctx);
  uint32_t *w = reinterpret_cast<uint32_t *>(c->base + cp_flags_offset(*c)) + c->world + 1;
  return q35_workspace_status(w, status_out, clear, stream);
}

int q35_cp_disconnect(void *ctx) {
  Q35_REQUIRE(ctx != nullptr, Q35_ERR_INVALID_ARG, "cp_disconnect: ctx is NULL");
  CpCtx *c = static_cast<CpCtx *>(ctx);
  for (int r = 0; r < c->world; ++r)
    if (r != c->rank && c->peer[r] != nullptr) {
      (void)cudaIpcCloseMemHandle(c->peer[r]);
      c->peer[r] = nullptr;
    }
  c->connected = c->world == 1;
  return Q35_OK;
}

int q35_cp_destroy(void *ctx) {
  if (ctx == nullptr) return Q35_OK;
  CpCtx *c = static_cast<CpCtx *>(ctx);
  (void)q35_cp_disconnect(ctx);
  (void)cudaFree(c->base);
  delete c;
  return Q35_OK;
}

}  // extern "C"
