// gdn_gate.cu -- beta / g gate projection of the Gated DeltaNet layer.
//
// mode 0 restates kernels.rs:174-247 (gate_proj_kernel, used at decode,
// text_modules.rs:569-576): 8 row splits summed sequentially in blocks of 8,
// partial sums added in split order, softplus threshold tested on the
// softplus value.  One CTA per input row; thread (split, which, head) owns one
// partial exactly like the reference's unit layout, so the f32 summation order
// is the reference's.
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

template <int H>
__global__ void gate_prefill_kernel(int N, int in_dim, const float *__restrict__ x, const float *__restrict__ wb,
                                    const float *__restrict__ wa, const float *__restrict__ a_log,
                                    const float *__restrict__ dt_bias, float *__restrict__ beta,
                                    float *__restrict__ g) {
  pdl_entry();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= N) return;
  const float *xr = x + (size_t)warp * in_dim;
  float ab[H], aa[H];
#pragma unroll
  for (int h = 0; h < H; ++h) ab[h] = aa[h] = 0.0f;
  for (int row = lane; row < in_dim; row += 32) {
    const float xv = xr[row];
#pragma unroll
    for (int h = 0; h < H; ++h) {
      ab[h] = fmaf(xv, wb[(size_t)row * H + h], ab[h]);
      aa[h] = fmaf(xv, wa[(size_t)row * H + h], aa[h]);
    }
  }
#pragma unroll
  for (int h = 0; h < H; ++h) {
    ab[h] = warp_sum(ab[h]);
    aa[h] = warp_sum(aa[h]);
  }
  if (lane < H) {
    float bsum = 0.f, asum = 0.f;
#pragma unroll
    for (int h = 0; h < H; ++h)
      if (h == lane) { bsum = ab[h]; asum = aa[h]; }
    const float xg = asum + dt_bias[lane];
    const float sp = xg > 20.0f ? xg : logf(expf(xg) + 1.0f);
    beta[(size_t)warp * H + lane] = sigmoidf_dev(bsum);
    g[(size_t)warp * H + lane] = -expf(a_log[lane]) * sp;
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
    note_launch();
    (void)launch_kernel(gate_decode_kernel, dim3(N), dim3(2 * H * kSplits), kSplits * 2 * H * sizeof(float), st, 1, 1, in_dim, H, x, wb, wa, a_log,
                                                                                      dt_bias, beta, g);
    return check_cuda(cudaGetLastError(), "gdn_gate launch");
  }
  const int threads = 256, rows_per_cta = threads / 32;
  const int grid = (N + rows_per_cta - 1) / rows_per_cta;
  note_launch();
  switch (H) {
    case 16: (void)launch_kernel(gate_prefill_kernel<16>, dim3(grid), dim3(threads), 0, st, 1, 1, N, in_dim, x, wb, wa, a_log, dt_bias, beta, g); break;
    case 32: (void)launch_kernel(gate_prefill_kernel<32>, dim3(grid), dim3(threads), 0, st, 1, 1, N, in_dim, x, wb, wa, a_log, dt_bias, beta, g); break;
    case 48: (void)launch_kernel(gate_prefill_kernel<48>, dim3(grid), dim3(threads), 0, st, 1, 1, N, in_dim, x, wb, wa, a_log, dt_bias, beta, g); break;
    case 64: (void)launch_kernel(gate_prefill_kernel<64>, dim3(grid), dim3(threads), 0, st, 1, 1, N, in_dim, x, wb, wa, a_log, dt_bias, beta, g); break;
    default:
      (void)launch_kernel(gate_prefill_any_kernel, dim3(grid), dim3(threads), 0, st, 1, 1, N, in_dim, H, x, wb, wa, a_log, dt_bias, beta, g);
      break;
  }
  return check_cuda(cudaGetLastError(), "gdn_gate launch");
}

}  // namespace q35
