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
// attention output in one kernel, with no fence and no separate flag: every
// 4-byte value travels in an 8-byte word together with the step's epoch
// (value bits low, epoch high), written by one 8-byte access, so a reader that
// sees the epoch in a word also sees that word's value.
//   1. the CTAs store this rank's payload (GDN outputs + partials) as such
//      words straight into slot [rank] of every rank's receive buffer (plain
//      16-byte peer stores over NVLink, one GPU after the other);
//   2. each thread polls (bounded) the words it needs in its own buffer until
//      they carry the epoch, then merges: the flash-decode combine of every
//      rank's partial, times sigmoid(gate), and the GDN outputs in rank order.
// No CTA waits for another CTA of its own grid: the work is spread so that a
// thread has about one (pair of values, destination) to send and one pair to
// receive.
// The receive buffer has two halves selected by the epoch's parity: a rank can
// only start step e+1 after it read every rank's step-e words, and every rank
// wrote those only after finishing step e-1, so the half of step e-1 that a
// fast rank overwrites is no longer read.  Each CTA keeps its own epoch
// counter in this rank's buffer (all advance once per call, so they agree),
// and the kernel advances it, so captured steps replay.
// A wait that gives up (a rank's words did not arrive within 1 s) sets
// Q35_STATUS_WAIT_TIMEOUT in the context's status word and writes NaN for the
// outputs it could not form; the epochs of the ranks may then disagree, so the
// caller treats the context as broken (tears it down and creates a new one).
//
// The receive buffers are allocated once (q35_cp_create) and mapped by the
// peers through CUDA IPC handles (q35_cp_connect); the exchange itself
// allocates nothing.
#include <algorithm>
#include <cstring>
#include <string>

#include "common.cuh"

namespace q35 {
namespace {

constexpr int kCpMaxWorld = 8;
constexpr int kCpThreads = 256;
constexpr int kCpMaxBlocks = 32;
constexpr int kD = 256;
constexpr uint64_t kCpWaitNs = 1000000000ull;  // 1 s

struct CpCtx {
  int world, rank, batch, n_gdn, hq;
  size_t payload;          // values per rank per half (even)
  int blocks;              // CTAs of the exchange grid
  unsigned char *base;     // this rank's buffer (cudaMalloc)
  size_t bytes;
  unsigned char *peer[kCpMaxWorld];  // every rank's buffer as mapped here (peer[rank] = base)
  bool connected;
};

// Buffer layout: [2 halves][world][payload] 8-byte words, then (256-byte
// aligned) the status u32 followed by one epoch u32 per CTA.
size_t cp_ctrl_offset(const CpCtx &c) {
  const size_t data = 2 * (size_t)c.world * c.payload * sizeof(uint64_t);
  return (data + 255) / 256 * 256;
}

struct CpParams {
  uint64_t *peer_data[kCpMaxWorld];  // every rank's receive buffer (data region)
  const uint64_t *my_data;
  uint32_t *status, *epochs;
  const float *gdn_local, *gqa_part, *q_gate;
  float *gdn_full, *gqa_out;
  int world, rank, batch, n_gdn, hq;
  long long payload;
  uint64_t wait_ns;
  int fault;  // test hook: store nothing, so every wait runs out
};

__device__ __forceinline__ void st_words2(uint64_t *p, float2 v, uint32_t e) {
  const uint64_t hi = (uint64_t)e << 32;
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(hi | __float_as_uint(v.x)),
               "l"(hi | __float_as_uint(v.y))
               : "memory");
}

// Two adjacent words, polled until both carry epoch e; false (and zeros) once
// the deadline t0 + limit has passed.  Each 8-byte element of the access is
// single-copy atomic, and each is checked, so both values belong to epoch e.
__device__ __forceinline__ bool ld_words2(const uint64_t *p, uint32_t e, uint64_t t0, uint64_t limit, float2 &v) {
  uint64_t w0, w1;
  for (;;) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(p) : "memory");
    if ((uint32_t)(w0 >> 32) == e && (uint32_t)(w1 >> 32) == e) break;
    if (globaltimer_ns() - t0 > limit) {
      v = make_float2(0.0f, 0.0f);
      return false;
    }
  }
  v = make_float2(__uint_as_float((uint32_t)w0), __uint_as_float((uint32_t)w1));
  return true;
}

__global__ void __launch_bounds__(kCpThreads) cp_exchange_kernel(const CpParams p) {
  pdl_entry();
  __shared__ uint32_t s_epoch;
  const int tid = threadIdx.x;
  if (tid == 0) {
    s_epoch = p.epochs[blockIdx.x] + 1u;
    p.epochs[blockIdx.x] = s_epoch;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int half = (int)(epoch & 1u);
  const long long pay = p.payload;
  const long long ng = (long long)p.batch * p.n_gdn;          // GDN values of this rank
  const long long np = (long long)p.batch * p.hq * (kD + 2);  // partial values
  const long long gt = (long long)blockIdx.x * kCpThreads + tid, nthr = (long long)gridDim.x * kCpThreads;
  const float nan = __int_as_float(0x7fc00000);
  // 1. payload -> slot [rank] of every rank's buffer, two values per 16-byte store
  if (!p.fault) {
    const float2 *g2 = reinterpret_cast<const float2 *>(p.gdn_local);
    const float2 *q2 = reinterpret_cast<const float2 *>(p.gqa_part);
    const long long ng2 = ng >> 1, n2 = (ng + np) >> 1;
    const long long slot = ((long long)half * p.world + p.rank) * pay;
    for (long long j = gt; j < n2 * p.world; j += nthr) {  // one (pair, destination) per thread step
      const long long i = j % n2;
      const int r = (p.rank + 1 + (int)(j / n2)) % p.world;  // peers first, this rank's own slot last
      const float2 v = i < ng2 ? g2[i] : q2[i - ng2];
      st_words2(p.peer_data[r] + slot + 2 * i, v, epoch);
    }
  }
  // 2. receive from this rank's own buffer as the words arrive: first the
  // merged attention pairs, then the GDN pairs, one task space over the grid
  const uint64_t *mine = p.my_data + (long long)half * p.world * pay;
  const uint64_t t0 = globaltimer_ns();
  bool ok = true;
  const long long n_merge = (long long)p.batch * p.hq * (kD / 2);
  const long long row = (long long)p.world * p.n_gdn;
  const long long n_tasks = n_merge + (long long)p.batch * row / 2;
  for (long long t = gt; t < n_tasks; t += nthr) {
    if (t < n_merge) {
      const long long i = 2 * t;
      const int d = (int)(i % kD);
      const long long bh = i / kD;  // b * hq + h
      float2 ml[kCpMaxWorld], o[kCpMaxWorld];
      bool got = true;
      float M = -INFINITY;
#pragma unroll
      for (int r = 0; r < kCpMaxWorld; ++r) {
        if (r < p.world) {
          const uint64_t *pr = mine + r * pay + ng + bh * (kD + 2);
          got &= ld_words2(pr + kD, epoch, t0, p.wait_ns, ml[r]);
          got &= ld_words2(pr + d, epoch, t0, p.wait_ns, o[r]);
          M = fmaxf(M, ml[r].x);
        }
      }
      float L = 0.0f, O0 = 0.0f, O1 = 0.0f;
#pragma unroll
      for (int r = 0; r < kCpMaxWorld; ++r) {
        if (r < p.world) {
          const float w = ml[r].x == -INFINITY ? 0.0f : exp2f(ml[r].x - M);  // a shard without keys adds nothing
          L = fmaf(ml[r].y, w, L);
          O0 = fmaf(o[r].x, w, O0);
          O1 = fmaf(o[r].y, w, O1);
        }
      }
      ok &= got;
      const float2 gate = *reinterpret_cast<const float2 *>(p.q_gate + bh * 2 * kD + kD + d);
      *reinterpret_cast<float2 *>(p.gqa_out + i) =
          got ? make_float2((O0 / L) * sigmoidf_dev(gate.x), (O1 / L) * sigmoidf_dev(gate.y)) : make_float2(nan, nan);
    } else {
      // GDN outputs in rank order: gdn_full[b][r * n_gdn + j]
      const long long i = 2 * (t - n_merge);
      const long long b = i / row, rem = i % row;
      const int r = (int)(rem / p.n_gdn);
      const long long j = rem % p.n_gdn;
      float2 v;
      const bool got = ld_words2(mine + r * pay + b * p.n_gdn + j, epoch, t0, p.wait_ns, v);
      ok &= got;
      *reinterpret_cast<float2 *>(p.gdn_full + i) = got ? v : make_float2(nan, nan);
    }
  }
  if (!ok) atomicOr(p.status, Q35_STATUS_WAIT_TIMEOUT);
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
  Q35_REQUIRE(n_gdn % 2 == 0, Q35_ERR_UNSUPPORTED, "cp_create: the GDN values per sequence must be even");
  if (int rc = require_sm100()) return rc;
  CpCtx *c = new CpCtx();
  c->world = world;
  c->rank = rank;
  c->batch = batch;
  c->n_gdn = n_gdn;
  c->hq = num_q_heads;
  c->payload = (size_t)batch * n_gdn + (size_t)batch * num_q_heads * (kD + 2);
  {
    // about one pair of values per thread to send (to every rank) and to receive
    const long long pairs = std::max<long long>((long long)c->payload / 2 * world,
                                                (long long)batch * num_q_heads * (kD / 2) +
                                                    (long long)batch * world * n_gdn / 2);
    c->blocks = (int)std::min<long long>(kCpMaxBlocks, std::max<long long>(1, (pairs + kCpThreads - 1) / kCpThreads));
  }
  c->bytes = cp_ctrl_offset(*c) + 256;
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
  Q35_REQUIRE(((reinterpret_cast<uintptr_t>(gdn_local) | reinterpret_cast<uintptr_t>(gqa_part) |
                reinterpret_cast<uintptr_t>(q_gate) | reinterpret_cast<uintptr_t>(gdn_full) |
                reinterpret_cast<uintptr_t>(gqa_out)) & 7u) == 0,
              Q35_ERR_INVALID_ARG, "cp_exchange: every buffer must be 8-byte aligned");
  CpParams p = {};
  for (int r = 0; r < c->world; ++r) p.peer_data[r] = reinterpret_cast<uint64_t *>(c->peer[r]);
  p.my_data = reinterpret_cast<const uint64_t *>(c->base);
  p.status = reinterpret_cast<uint32_t *>(c->base + cp_ctrl_offset(*c));
  p.epochs = p.status + 1;
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
  (void)launch_kernel(cp_exchange_kernel, dim3(c->blocks), dim3(kCpThreads), 0, static_cast<cudaStream_t>(stream), 1,
                      1, p);
  return check_cuda(cudaGetLastError(), "cp_exchange launch");
}

int q35_cp_status(void *ctx, uint32_t *status_out, int32_t clear, void *stream) {
  Q35_REQUIRE(ctx != nullptr && status_out != nullptr, Q35_ERR_INVALID_ARG, "cp_status: NULL argument");
  CpCtx *c = static_cast<CpCtx *>(ctx);
  uint32_t *w = reinterpret_cast<uint32_t *>(c->base + cp_ctrl_offset(*c));
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
