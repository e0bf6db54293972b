// common.cuh -- shared helpers for the sm_100a kernels of libq35attn:
// error plumbing, launch bookkeeping, and thin inline-PTX wrappers for
// mbarriers, bulk (TMA) copies, cluster/DSMEM access and proxy fences.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "q35attn.h"

namespace q35 {

// ---------------------------------------------------------------- host side
void set_error(const std::string &msg);
int fail(int code, const std::string &msg);
int check_cuda(cudaError_t e, const char *what);
void note_launch(int n = 1);
int device_sm_count();
int require_sm100();

// Programmatic dependent launch on every library launch unless the
// environment sets Q35_PDL=0.
bool pdl_enabled();

// Device address of this device's status word for kernels that take no
// workspace (read with q35_device_status); nullptr when it cannot be resolved.
uint32_t *device_status_word();

// cudaLaunchKernelEx with the PDL attribute (and a cluster shape when
// cluster_x * cluster_y > 1).  launch_kernel_serial is the same launch in
// plain stream order: the GQA flash-decode measured 8-10 % slower at batch 1
// with its successor scheduled early, so it keeps the plain order.
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel_impl(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                               cudaStream_t st, unsigned cluster_x, unsigned cluster_y, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  unsigned na = 0;
  if (pdl && pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (cluster_x * cluster_y > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = cluster_x;
    attr[na].val.clusterDim.y = cluster_y;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                          unsigned cluster_x, unsigned cluster_y, Args... args) {
  return launch_kernel_impl(true, kernel, grid, block, smem, st, cluster_x, cluster_y, args...);
}
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel_serial(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                 unsigned cluster_x, unsigned cluster_y, Args... args) {
  return launch_kernel_impl(false, kernel, grid, block, smem, st, cluster_x, cluster_y, args...);
}

#define Q35_REQUIRE(cond, code, msg)          \
  do {                                        \
    if (!(cond)) return ::q35::fail(code, msg); \
  } while (0)

// ---------------------------------------------------------------- device side
constexpr float kLog2e = 1.4426950408889634f;

// Iteration bound for every in-kernel spin: ~2^24 polls of try_wait (each
// poll itself suspends for a hardware-defined interval) is seconds, far beyond
// any legitimate wait, and short enough to return control to the host.
constexpr uint32_t kSpinLimit = 1u << 24;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wall-clock bound of one wait: try_wait may suspend the thread for a
// hardware-defined interval per poll, so the poll count alone does not bound
// the time.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// Bounded wait on an mbarrier phase.  Returns false (and leaves the phase
// incomplete) after limit_ns or kSpinLimit polls, whichever comes first.
__device__ __forceinline__ bool mbar_wait_ns(uint64_t *bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
  return false;
}
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  return mbar_wait_ns(bar, parity, kWaitLimitNs);
}

// Test hook (q35_test_arm_wait_fault): the next launch of the armed site
// withholds one asynchronous copy and waits with this short limit, so that a
// bounded wait runs out and the error path is exercised without a fault.
constexpr uint64_t kFaultWaitLimitNs = 2000000ull;  // 2 ms
enum FaultSite : int { kFaultNone = 0, kFaultPrefillState = 1, kFaultGqaDecode = 2, kFaultCpExchange = 3 };
// Returns the armed site once (and disarms it) when it equals `site`.
bool take_fault(int site);

// Bulk (non-tensor) TMA copy global -> shared, completing `bytes` of
// transaction count on `bar`.  src/dst 16-byte aligned, bytes % 16 == 0.
// The L2 policy marks the streamed lines evict-first.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// The same copy without an L2 policy.
__device__ __forceinline__ void bulk_g2s_nohint(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Orders this thread's generic-proxy global writes before later async-proxy
// (TMA) accesses of the same addresses.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Named barrier helpers (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float sigmoidf_dev(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float siluf_dev(float x) { return x * sigmoidf_dev(x); }

__device__ __forceinline__ float4 f4_fma(float s, float4 a, float4 c) {
  return make_float4(fmaf(s, a.x, c.x), fmaf(s, a.y, c.y), fmaf(s, a.z, c.z), fmaf(s, a.w, c.w));
}

// Packed pairs of f32 (low word = first element) and the sm_100 f32x2 ops.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// Bytes 2h and 2h + 1 of w (signed int8) as an exact f32 pair: a byte permute
// puts q + 128 into the low mantissa byte of 2^23 (0x4B0000XX), and one
// packed subtraction of 2^23 + 128 leaves q in both lanes.
__device__ __forceinline__ uint64_t s8_pair(uint32_t w, int h) {
  const uint32_t u = w ^ 0x80808080u;
  const uint64_t m = f2_pack(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540u | (2 * h))),
                             __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540u | (2 * h + 1))));
  return f2_sub(m, 0x4B0000804B000080ull);
}

}  // namespace q35

namespace q35 {

// Bulk (non-tensor) TMA store shared -> global, tracked by the issuing
// thread's bulk async-group.  Both addresses 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_s2g(void *dst, const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N of this thread's committed bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (bulk copy) reads of them.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

}  // namespace q35

namespace q35 {

// Ampere-style asynchronous 16-byte global -> shared copy (L2 only), grouped
// with commit / wait_group.
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
// 16-byte copy that reads src_bytes (0 or 16) bytes and zero-fills the rest.
__device__ __forceinline__ void cp_async16_zfill(void *smem_dst, const void *gmem_src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void *smem_dst, const void *gmem_src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Programmatic dependent launch.  Every kernel of the library starts with
// pdl_entry(): wait until the previous grid in the stream has completed and
// its memory is visible (a no-op when the launch had no PDL attribute), then
// let the next grid be scheduled; so in a captured sequence of launches the
// next kernel is launched and made resident while this one drains.
__device__ __forceinline__ void pdl_entry() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// L2 prefetch of `bytes` (a multiple of 16) from a 16-byte aligned global
// address; no completion to wait for.
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Thread-block cluster helpers (DSMEM).
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Split cluster barrier: arrive (no memory ordering) early, wait (acquire) later.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// Shared::cluster address of `local` in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t dsmem_addr(const void *local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  return remote;
}
// Asynchronous store of one float into another CTA's shared memory; its 4
// bytes count against that CTA's mbarrier (complete_tx).
__device__ __forceinline__ void st_async_f32(uint32_t remote_addr, float v, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(remote_addr),
               "f"(v), "r"(remote_bar)
               : "memory");
}
// The float at the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ float ld_dsmem_f32(const float *local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

__device__ __forceinline__ float dot4(float4 a, float4 b, float acc) {
  acc = fmaf(a.x, b.x, acc);
  acc = fmaf(a.y, b.y, acc);
  acc = fmaf(a.z, b.z, acc);
  return fmaf(a.w, b.w, acc);
}

}  // namespace q35
