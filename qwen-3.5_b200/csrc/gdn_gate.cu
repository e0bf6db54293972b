// gdn_gate.cu -- beta / g gate projection of the Gated DeltaNet layer.
//
// mode 0 restates kernels.rs:174-247 (gate_proj_kernel, used at decode,
// text_modules.rs:569-576): 8 row splits summed sequentially in blocks of 8,
// partial sums added in split order, softplus threshold tested on the
// softplus value.  Each (split, which, head) partial is accumulated row by row
// in the reference's order and the partials are added in split order, so the
// f32 result is the reference's.  B200 layout: one 8-CTA cluster per input
// row, CTA s = split s.  Its rows of w_b and w_a (contiguous, H floats per
// row) are staged into shared memory with coalesced 16-byte loads before the
// grid-dependency wait (the weights never depend on the previous kernel, so
// the copy overlaps it); one warp-pair then runs the 2H sequential chains from
// shared memory, and ranks 1-7 push their partials into rank 0's shared
// memory with st.async (complete_tx on rank 0's mbarrier) and exit; rank 0
// adds the 8 partials in split order.  Shapes whose split does not fit shared memory use the one-CTA
// kernel (one thread per partial, straight from global memory).
// mode 1 restates the prefill branch text_modules.rs:578-595 (matmul, sigmoid,
// softplus with the threshold on a + dt_bias): one warp per row.
#include "common.cuh"

namespace q35 {
namespace {

constexpr int kSplits = 8;

__global__ void gate_decode_kernel(int in_dim, int H, const float *__restrict__ x, const float *__restrict__ wb,
                                   const float *__restrict__ wa, const float *__restrict__ a_log,
                                   const float *__restrict__ dt_bias, float *__restrict__ beta,
                                   float *__restrict__ g) {
  pdl_entry();
  extern __shared__ float partial[];  // [kSplits][2H]
  const int n = blockIdx.x;
  const int u = threadIdx.x;  // 0 .. 2*H*kSplits-1
  const int h = u % H;
  const int split = u / (2 * H);
  const bool is_beta = ((u / H) % 2) == 0;
  const int chunk = in_dim / kSplits;
  const int row0 = split * chunk;
  const float *xr = x + (size_t)n * in_dim;
  const float *w = is_beta ? wb : wa;
  float acc = 0.0f;
  for (int blk = 0; blk < chunk / 8; ++blk)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int row = row0 + blk * 8 + j;
      acc += xr[row] * w[(size_t)row * H + h];
    }
  partial[split * 2 * H + h + (is_beta ? 0 : H)] = acc;
  __syncthreads();
  if (split == 0) {
    float sum = 0.0f;
    for (int i = 0; i < kSplits; ++i) sum += partial[i * 2 * H + h + (is_beta ? 0 : H)];
    if (is_beta) {
      beta[(size_t)n * H + h] = 1.0f / (1.0f + expf(-sum));
    } else {
      const float xg = sum + dt_bias[h];
      const float pre = logf(expf(xg) + 1.0f);
      const float sp = pre > 20.0f ? xg : pre;
      g[(size_t)n * H + h] = -expf(a_log[h]) * sp;
    }
  }
}

// Copies n floats global -> shared with all threads (16-byte loads when both
// ends are 16-byte aligned and n % 4 == 0).
__device__ __forceinline__ void stage_f32(float *dst, const float *src, int n) {
  if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) == 0 && (n & 3) == 0) {
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
    float4 *d4 = reinterpret_cast<float4 *>(dst);
#pragma unroll 8
    for (int i = threadIdx.x; i < n / 4; i += blockDim.x) d4[i] = __ldg(s4 + i);
  } else {
#pragma unroll 8
    for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = __ldg(src + i);
  }
}

constexpr int kGateThreads = 256;

__global__ void __launch_bounds__(kGateThreads) gate_decode_cluster_kernel(
    int in_dim, int H, const float *__restrict__ x, const float *__restrict__ wb, const float *__restrict__ wa,
    const float *__restrict__ a_log, const float *__restrict__ dt_bias, float *__restrict__ beta,
    float *__restrict__ g, uint32_t *status) {
  extern __shared__ __align__(16) float gsm[];
  const int n = blockIdx.y;
  const int split = (int)cluster_ctarank();
  const int chunk = in_dim / kSplits;
  const int rows = (chunk / 8) * 8;  // rows the reference walks per split (kernels.rs:190-199)
  const int row0 = split * chunk;
  const int wrow = (rows * H + 3) & ~3;  // 16-byte aligned sub-buffers
  float *wbs = gsm, *was = gsm + wrow, *xs = gsm + 2 * wrow, *recv = xs + ((rows + 3) & ~3);  // recv [8][2H]
  __shared__ uint64_t redbar;
  if (split == 0 && threadIdx.x == 0) {  // rank 0 expects 7 ranks x 2H partials
    mbar_init(&redbar, 1);
    mbar_arrive_expect_tx(&redbar, (uint32_t)((kSplits - 1) * 2 * H * sizeof(float)));
    fence_mbar_init();
  }
  cluster_arrive_relaxed();  // waited on before the push: rank 0's barrier is initialised
  stage_f32(wbs, wb + (size_t)row0 * H, rows * H);
  stage_f32(was, wa + (size_t)row0 * H, rows * H);
  pdl_entry();  // x is the previous kernel's output
  stage_f32(xs, x + (size_t)n * in_dim + row0, rows);
  __syncthreads();
  const int u = threadIdx.x;
  float acc = 0.0f;
  if (u < 2 * H) {
    const int h = u % H;
    const float *w = u < H ? wbs : was;
#pragma unroll 8
    for (int r = 0; r < rows; ++r) acc += xs[r] * w[r * H + h];
  }
  cluster_wait();
  if (split != 0) {  // push this split's partials to rank 0 and leave
    if (u < 2 * H)
      st_async_f32(dsmem_addr(&recv[(split - 1) * 2 * H + u], 0), acc, dsmem_addr(&redbar, 0));
    return;
  }
  if (u < 2 * H) {
    const bool got = mbar_wait(&redbar, 0);
    float sum = 0.0f + acc;  // split order: 0, 1, ..., 7
    for (int i = 1; i < kSplits; ++i) sum += recv[(i - 1) * 2 * H + u];
    if (!got) {  // a bounded wait gave up: poison, flag the device status word
      sum = __int_as_float(0x7fc00000);
      if (status != nullptr) atomicOr(status, Q35_STATUS_WAIT_TIMEOUT);
    }
    const int h = u % H;
    if (u < H) {
      beta[(size_t)n * H + h] = 1.0f / (1.0f + expf(-sum));
    } else {
      const float xg = sum + dt_bias[h];
      const float pre = logf(expf(xg) + 1.0f);
      const float sp = pre > 20.0f ? xg : pre;
      g[(size_t)n * H + h] = -expf(a_log[h]) * sp;
    }
  }
}

size_t gate_cluster_smem(int in_dim, int H) {
  const int rows = (in_dim / kSplits / 8) * 8;
  return ((size_t)2 * ((rows * H + 3) & ~3) + ((rows + 3) & ~3) + (kSplits - 1) * 2 * H) * sizeof(float);
}

// Prefill (mode 1), 2H in {32, 64, 128}: a CTA of 256 threads takes R = 256 / (2H)
// rows; thread (r, o) accumulates output o (o < H: the b head o, else the a head
// o - H) of row r.  The in_dim axis is walked in chunks of KC whose [w_b | w_a]
// rows and x values are staged in shared memory once for all R rows, so the
// weights are read once per CTA instead of once per row.  Lanes read
// consecutive weight columns (conflict-free) and one broadcast x value.
template <int H>
__global__ void __launch_bounds__(256) gate_prefill_kernel(int N, int in_dim, const float *__restrict__ x,
                                                           const float *__restrict__ wb,
                                                           const float *__restrict__ wa,
                                                           const float *__restrict__ a_log,
                                                           const float *__restrict__ dt_bias,
                                                           float *__restrict__ beta, float *__restrict__ g) {
  constexpr int O = 2 * H, R = 256 / O, KC = H == 64 ? 64 : 128;
  constexpr int WP = KC * O / 256, XP = (R * KC + 255) / 256;  // weight / x elements per thread per chunk
  __shared__ float ws[KC][O];
  __shared__ float xs[R][KC];
  pdl_entry();
  const int tid = threadIdx.x, r = tid / O, o = tid % O;
  const int row0 = blockIdx.x * R;
  // chunk loads go to registers first, all in flight at once, and the next
  // chunk's are requested before this chunk's products
  float wr[WP], xr[XP];
#define Q35_GATE_LOAD(K0)                                                                                          \
  do {                                                                                                              \
    _Pragma("unroll") for (int i = 0; i < WP; ++i) {                                                                \
      const int e = tid + 256 * i, k = (K0) + e / O, c = e % O;                                                     \
      wr[i] = k < in_dim ? (c < H ? __ldg(wb + (size_t)k * H + c) : __ldg(wa + (size_t)k * H + (c - H))) : 0.0f;    \
    }                                                                                                               \
    _Pragma("unroll") for (int i = 0; i < XP; ++i) {                                                                \
      const int e = tid + 256 * i, rr = e / KC, k = (K0) + e % KC;                                                  \
      xr[i] = (e < R * KC && row0 + rr < N && k < in_dim) ? __ldg(x + (size_t)(row0 + rr) * in_dim + k) : 0.0f;    \
    }                                                                                                               \
  } while (0)
  float acc = 0.0f;
  Q35_GATE_LOAD(0);
  for (int k0 = 0; k0 < in_dim; k0 += KC) {
#pragma unroll
    for (int i = 0; i < WP; ++i) (&ws[0][0])[tid + 256 * i] = wr[i];
#pragma unroll
    for (int i = 0; i < XP; ++i)
      if (tid + 256 * i < R * KC) (&xs[0][0])[tid + 256 * i] = xr[i];
    __syncthreads();
    if (k0 + KC < in_dim) Q35_GATE_LOAD(k0 + KC);
#pragma unroll 16
    for (int k = 0; k < KC; ++k) acc = fmaf(xs[r][k], ws[k][o], acc);
    __syncthreads();
  }
#undef Q35_GATE_LOAD
  const int row = row0 + r;
  if (row < N) {
    if (o < H) {
      beta[(size_t)row * H + o] = sigmoidf_dev(acc);
    } else {
      const int h = o - H;
      const float xg = acc + dt_bias[h];
      const float sp = xg > 20.0f ? xg : logf(expf(xg) + 1.0f);
      g[(size_t)row * H + h] = -expf(a_log[h]) * sp;
    }
  }
}

// Any other head count: one warp per row, one head at a time.
__global__ void gate_prefill_any_kernel(int N, int in_dim, int H, const float *__restrict__ x,
                                        const float *__restrict__ wb, const float *__restrict__ wa,
                                        const float *__restrict__ a_log, const float *__restrict__ dt_bias,
                                        float *__restrict__ beta, float *__restrict__ g) {
  pdl_entry();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= N) return;
  const float *xr = x + (size_t)warp * in_dim;
  for (int h = 0; h < H; ++h) {
    float ab = 0.0f, aa = 0.0f;
    for (int row = lane; row < in_dim; row += 32) {
      const float xv = xr[row];
      ab = fmaf(xv, wb[(size_t)row * H + h], ab);
      aa = fmaf(xv, wa[(size_t)row * H + h], aa);
    }
    ab = warp_sum(ab);
    aa = warp_sum(aa);
    if (lane == 0) {
      const float xg = aa + dt_bias[h];
      const float sp = xg > 20.0f ? xg : logf(expf(xg) + 1.0f);
      beta[(size_t)warp * H + h] = sigmoidf_dev(ab);
      g[(size_t)warp * H + h] = -expf(a_log[h]) * sp;
    }
  }
}

}  // namespace

int gdn_gate_launch(int N, int in_dim, int H, const float *x, const float *wb, const float *wa, const float *a_log,
                    const float *dt_bias, float *beta, float *g, int mode, cudaStream_t st) {
  if (N == 0) return Q35_OK;
  if (mode == 0) {
    Q35_REQUIRE(2 * H * kSplits <= 1024, Q35_ERR_UNSUPPORTED, "gdn_gate: num_heads must be <= 64 for mode 0");
    const size_t smem = gate_cluster_smem(in_dim, H);
    if (N <= 65535 && smem <= 200 * 1024 && in_dim >= kSplits * 8) {
      cudaError_t e = cudaFuncSetAttribute(gate_decode_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem);
      if (e != cudaSuccess) return check_cuda(e, "gdn_gate attributes");
      note_launch();
      (void)launch_kernel(gate_decode_cluster_kernel, dim3(kSplits, N), dim3(kGateThreads), smem, st, kSplits, 1,
                          in_dim, H, x, wb, wa, a_log, dt_bias, beta, g, device_status_word());
      return check_cuda(cudaGetLastError(), "gdn_gate launch");
    }
    note_launch();
    (void)launch_kernel(gate_decode_kernel, dim3(N), dim3(2 * H * kSplits), kSplits * 2 * H * sizeof(float), st, 1, 1, in_dim, H, x, wb, wa, a_log,
                                                                                      dt_bias, beta, g);
    return check_cuda(cudaGetLastError(), "gdn_gate launch");
  }
  note_launch();
  switch (H) {
    case 16: (void)launch_kernel(gate_prefill_kernel<16>, dim3((N + 7) / 8), dim3(256), 0, st, 1, 1, N, in_dim, x, wb, wa, a_log, dt_bias, beta, g); break;
    case 32: (void)launch_kernel(gate_prefill_kernel<32>, dim3((N + 3) / 4), dim3(256), 0, st, 1, 1, N, in_dim, x, wb, wa, a_log, dt_bias, beta, g); break;
    case 64: (void)launch_kernel(gate_prefill_kernel<64>, dim3((N + 1) / 2), dim3(256), 0, st, 1, 1, N, in_dim, x, wb, wa, a_log, dt_bias, beta, g); break;
    default: {
      const int threads = 256, rows_per_cta = threads / 32;
      const int grid = (N + rows_per_cta - 1) / rows_per_cta;
      (void)launch_kernel(gate_prefill_any_kernel, dim3(grid), dim3(threads), 0, st, 1, 1, N, in_dim, H, x, wb, wa, a_log, dt_bias, beta, g);
      break;
    }
  }
  return check_cuda(cudaGetLastError(), "gdn_gate launch");
}

}  // namespace q35
