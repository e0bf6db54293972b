// stack.cu -- the decoder-stack glue around the attention cores, for the
// end-to-end hybrid stack (embedding, RMSNorm with the residual add, SwiGLU,
// tied-embedding lm_head, argmax, Q8F dequantisation for the prefill
// projections).
//
//   q8_embedding : kernels.rs:15-45 (q8_embedding_lookup_kernel), model.rs:47-48
//   add_rmsnorm  : text_modules.rs:800-809 (RMSNorm, weight used as 1 + w)
//                  with the residual adds of DecoderLayer::forward :1053-1085
//   silu_mul     : text_modules.rs:999-1011 (MLP: up * silu(gate))
//   q8_lm_head   : kernels.rs:251-291 (q8_lm_head_kernel), model.rs:126
//   argmax       : kernels.rs:298-371 (two-stage argmax), main.rs:131
//   rope_gather  : text_modules.rs:30-43 at the decode position (model.rs:50-56)
//   q8_dequant   : the weight Linear::forward multiplies at prefill
//                  (text_modules.rs:499, 506, 663, 858, 879, 888, 941, 1007-1009)
//
// All are HBM streams; the lm_head (508 MB of int8 weights per token) is the
// only large one: a warp takes one vocabulary row per step (2 KB, 64 bytes per
// lane, one scale per lane), 4 rows in flight, x held in registers.
#include <algorithm>

#include "common.cuh"

namespace q35 {
namespace {

__device__ __forceinline__ float s8(uint32_t v, int j) { return (float)((int32_t)(v << (24 - 8 * j)) >> 24); }

// ------------------------------------------------------------- embedding
// out[i][c] = int8(table[id_i][c]) * scales[id_i][c / 64]; ids outside
// [0, vocab) give a zero row instead of an out-of-range read
__global__ void q8_embedding_kernel(int n, int vocab, int dim, const int32_t *ids, const uint32_t *table,
                                    const float *scales, float *out) {
  pdl_entry();
  const int i = blockIdx.y;
  const int w = blockIdx.x * blockDim.x + threadIdx.x;  // word index in the row
  if (i >= n || w >= dim / 4) return;
  const int64_t id = ids[i];
  if (id < 0 || id >= vocab) {
    *reinterpret_cast<float4 *>(out + (size_t)i * dim + 4 * w) = make_float4(0.f, 0.f, 0.f, 0.f);
    return;
  }
  const uint32_t word = table[id * (dim / 4) + w];
  const float sc = scales[id * (dim / 64) + (4 * w) / 64];
  *reinterpret_cast<float4 *>(out + (size_t)i * dim + 4 * w) =
      make_float4(s8(word, 0) * sc, s8(word, 1) * sc, s8(word, 2) * sc, s8(word, 3) * sc);
}

// ------------------------------------------------------------- add + RMSNorm
// h = x (+ residual); sum_out = h (optional); out = h / sqrt(mean(h^2) + eps) * (1 + w)
// One CTA of 256 threads per row.
// dim <= 16 * 256: every element is loaded into a register before anything is
// stored (one memory round trip, and in-place use -- sum_out == residual, out
// == x -- is safe because each thread stores only the elements it loaded).
constexpr int kNormRegs = 16;

__global__ void __launch_bounds__(256) add_rmsnorm_reg_kernel(int dim, const float *x, const float *residual,
                                                              const float *w, float eps, float *out,
                                                              float *sum_out) {
  __shared__ float red[8];
  const size_t row = blockIdx.x;
  const float *xr = x + row * dim;
  const float *rr = residual ? residual + row * dim : nullptr;
  float wv[kNormRegs];
#pragma unroll
  for (int j = 0; j < kNormRegs; ++j) {
    const int c = threadIdx.x + j * 256;
    wv[j] = c < dim ? __ldg(w + c) : 0.0f;  // the norm weight is not the previous kernel's output
  }
  pdl_entry();
  float hv[kNormRegs];
#pragma unroll
  for (int j = 0; j < kNormRegs; ++j) {
    const int c = threadIdx.x + j * 256;
    hv[j] = c < dim ? xr[c] + (rr ? rr[c] : 0.0f) : 0.0f;
  }
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < kNormRegs; ++j) ss = fmaf(hv[j], hv[j], ss);
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float inv = 1.0f / sqrtf(tot / (float)dim + eps);
#pragma unroll
  for (int j = 0; j < kNormRegs; ++j) {
    const int c = threadIdx.x + j * 256;
    if (c < dim) {
      if (sum_out) sum_out[row * dim + c] = hv[j];
      out[row * dim + c] = (hv[j] * inv) * (1.0f + wv[j]);
    }
  }
}

__global__ void add_rmsnorm_kernel(int dim, const float *x, const float *residual, const float *w, float eps,
                                   float *out, float *sum_out) {
  pdl_entry();
  __shared__ float red[8];
  const size_t row = blockIdx.x;
  const float *xr = x + row * dim;
  const float *rr = residual ? residual + row * dim : nullptr;
  float ss = 0.0f;
  for (int c = threadIdx.x; c < dim; c += blockDim.x) {
    float h = xr[c];
    if (rr) h = h + rr[c];
    if (sum_out) sum_out[row * dim + c] = h;
    ss = fmaf(h, h, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
  const float inv = 1.0f / sqrtf(tot / (float)dim + eps);
  // sum_out may alias residual (h += x in place): read the stored sum back
  // (each thread revisits exactly the elements it wrote)
  for (int c = threadIdx.x; c < dim; c += blockDim.x) {
    float h;
    if (sum_out) {
      h = sum_out[row * dim + c];
    } else {
      h = xr[c];
      if (rr) h = h + rr[c];
    }
    out[row * dim + c] = (h * inv) * (1.0f + w[c]);
  }
}

// ------------------------------------------------------------- SwiGLU
__global__ void silu_mul_kernel(size_t n, const float *gate, const float *up, float *out) {
  pdl_entry();
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = up[i] * siluf_dev(gate[i]);
}

// ------------------------------------------------------------- lm_head
// logits[v] = sum_c int8(E[v][c]) * x[c] * scales[v][c / 64]; dim == 2048:
// lane l owns columns 64 l .. 64 l + 63 (four 16-byte loads, one scale).
constexpr int kHeadDim = 2048;
// rows in flight per warp; 2 rows leave room for 2 CTAs per SM (vocab 248,320,
// conversion instruction: 97.9 us against 99.5 us for 4 rows at 1 CTA per SM,
// 102.2 us for 8 rows; with the packed f32x2 form below 92.4 us)
constexpr int kHeadRows = 2;
__global__ void __launch_bounds__(256, 2) q8_lm_head_kernel(int vocab, const float *x, const uint4 *table,
                                                         const float *scales, float *logits) {
  pdl_entry();
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nwarps = (gridDim.x * blockDim.x) >> 5;
  float xv[64];
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const float4 v = *reinterpret_cast<const float4 *>(x + 64 * lane + 4 * k);
    xv[4 * k] = v.x;
    xv[4 * k + 1] = v.y;
    xv[4 * k + 2] = v.z;
    xv[4 * k + 3] = v.w;
  }
  for (int r0 = gw * kHeadRows; r0 < vocab; r0 += nwarps * kHeadRows) {
    uint4 q[kHeadRows][4];
    float sc[kHeadRows];
#pragma unroll
    for (int u = 0; u < kHeadRows; ++u) {
      const int r = min(r0 + u, vocab - 1);
      const uint4 *row = table + (size_t)r * (kHeadDim / 16) + 4 * lane;
#pragma unroll
      for (int k = 0; k < 4; ++k) q[u][k] = __ldg(row + k);
      sc[u] = __ldg(scales + (size_t)r * (kHeadDim / 64) + lane);
    }
#pragma unroll
    for (int u = 0; u < kHeadRows; ++u) {
      // one packed f32x2 accumulator: its low half sums the even columns of
      // this thread's 64, its high half the odd ones (exact int8 via s8_pair)
      uint64_t a2 = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t wv[4] = {q[u][k].x, q[u][k].y, q[u][k].z, q[u][k].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float *xj = xv + 16 * k + 4 * j;
          a2 = f2_fma(s8_pair(wv[j], 0), f2_pack(xj[0], xj[1]), a2);
          a2 = f2_fma(s8_pair(wv[j], 1), f2_pack(xj[2], xj[3]), a2);
        }
      }
      float even, odd;
      f2_unpack(a2, even, odd);
      const float acc = warp_sum((even + odd) * sc[u]);  // lane l's 64 columns share scale l
      if (lane == 0 && r0 + u < vocab) logits[r0 + u] = acc;
    }
  }
}

// ------------------------------------------------------------- argmax
// Stage 1: each CTA reduces a contiguous chunk to (max, index); stage 2: one
// CTA reduces the partials.  Ties resolve to the smallest index.
__device__ __forceinline__ void better(float &m, int &i, float v, int j) {
  if (v > m || (v == m && j < i)) {
    m = v;
    i = j;
  }
}
__device__ __forceinline__ void block_argmax(float &m, int &i) {
  __shared__ float sm[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float mv = __shfl_xor_sync(0xffffffffu, m, o);
    const int iv = __shfl_xor_sync(0xffffffffu, i, o);
    better(m, i, mv, iv);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sm[warp] = m;
    si[warp] = i;
  }
  __syncthreads();
  if (warp == 0) {
    m = lane < (int)(blockDim.x >> 5) ? sm[lane] : -INFINITY;
    i = lane < (int)(blockDim.x >> 5) ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float mv = __shfl_xor_sync(0xffffffffu, m, o);
      const int iv = __shfl_xor_sync(0xffffffffu, i, o);
      better(m, i, mv, iv);
    }
  }
}
__global__ void argmax_stage1(int n, const float *x, float *pm, int *pi) {
  pdl_entry();
  const int chunk = (n + gridDim.x - 1) / gridDim.x;
  const int a = blockIdx.x * chunk, e = min(n, a + chunk);
  float m = -INFINITY;
  int idx = 0x7fffffff;
  for (int j = a + threadIdx.x; j < e; j += blockDim.x) better(m, idx, x[j], j);
  block_argmax(m, idx);
  if (threadIdx.x == 0) {
    pm[blockIdx.x] = m;
    pi[blockIdx.x] = idx;
  }
}
__global__ void argmax_stage2(int np, const float *pm, const int *pi, int32_t *out) {
  pdl_entry();
  float m = -INFINITY;
  int idx = 0x7fffffff;
  for (int j = threadIdx.x; j < np; j += blockDim.x) better(m, idx, pm[j], pi[j]);
  block_argmax(m, idx);
  if (threadIdx.x == 0) out[0] = idx;
}

// ------------------------------------------------------------- RoPE rows
// cos/sin of the decode position of every sequence: out[b] = table[lens[b]]
// (TextRotaryEmbedding::forward, text_modules.rs:30-43, at position_ids =
// past_len, model.rs:50-56); positions past the table give cos 1, sin 0.
__global__ void rope_gather_kernel(int B, int rot, int max_pos, const int32_t *lens, const float *tc,
                                   const float *ts, float *oc, float *os) {
  pdl_entry();
  const int b = blockIdx.x, i = threadIdx.x;
  if (b >= B || i >= rot) return;
  const int pos = lens[b];
  const bool in = pos >= 0 && pos < max_pos;
  oc[b * rot + i] = in ? tc[(size_t)pos * rot + i] : 1.0f;
  os[b * rot + i] = in ? ts[(size_t)pos * rot + i] : 0.0f;
}

// ------------------------------------------------------------- dequant
// out[r][c] = int8(w[r][c]) * scales[r][c / 64], f32 [rows, cols]
__global__ void q8_dequant_kernel(int rows, int cols, const uint32_t *w, const float *scales, float *out) {
  pdl_entry();
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;  // word index
  const size_t nw = (size_t)rows * (cols / 4);
  if (i >= nw) return;
  const size_t r = i / (cols / 4), c = 4 * (i % (cols / 4));
  const uint32_t word = w[i];
  const float sc = scales[r * (cols / 64) + c / 64];
  *reinterpret_cast<float4 *>(out + r * cols + c) =
      make_float4(s8(word, 0) * sc, s8(word, 1) * sc, s8(word, 2) * sc, s8(word, 3) * sc);
}

}  // namespace

int q8_embedding_launch(int n, int vocab, int dim, const int32_t *ids, const uint32_t *table, const float *scales,
                        float *out, cudaStream_t st) {
  note_launch();
  (void)launch_kernel(q8_embedding_kernel, dim3((dim / 4 + 255) / 256, n), dim3(256), 0, st, 1, 1, n, vocab, dim, ids, table, scales, out);
  return check_cuda(cudaGetLastError(), "q8_embedding launch");
}

int add_rmsnorm_launch(int n, int dim, const float *x, const float *residual, const float *w, float eps, float *out,
                       float *sum_out, cudaStream_t st) {
  note_launch();
  if (dim <= kNormRegs * 256)
    (void)launch_kernel(add_rmsnorm_reg_kernel, dim3(n), dim3(256), 0, st, 1, 1, dim, x, residual, w, eps, out,
                        sum_out);
  else
    (void)launch_kernel(add_rmsnorm_kernel, dim3(n), dim3(256), 0, st, 1, 1, dim, x, residual, w, eps, out, sum_out);
  return check_cuda(cudaGetLastError(), "add_rmsnorm launch");
}

int silu_mul_launch(size_t n, const float *gate, const float *up, float *out, cudaStream_t st) {
  note_launch();
  (void)launch_kernel(silu_mul_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, 1, 1, n, gate, up, out);
  return check_cuda(cudaGetLastError(), "silu_mul launch");
}

int q8_lm_head_launch(int vocab, int dim, const float *x, const uint32_t *table, const float *scales, float *logits,
                      cudaStream_t st) {
  Q35_REQUIRE(dim == kHeadDim, Q35_ERR_UNSUPPORTED, "q8_lm_head: hidden size 2048 is the compiled configuration");
  note_launch();
  const int blocks = 4 * device_sm_count();
  (void)launch_kernel(q8_lm_head_kernel, dim3(blocks), dim3(256), 0, st, 1, 1, vocab, x, reinterpret_cast<const uint4 *>(table), scales, logits);
  return check_cuda(cudaGetLastError(), "q8_lm_head launch");
}

size_t argmax_workspace_bytes() { return 2 * 1024 * sizeof(float); }

int argmax_launch(int n, const float *x, int32_t *out, void *ws, cudaStream_t st) {
  const int np = std::min(1024, std::max(1, (n + 255) / 256));
  float *pm = static_cast<float *>(ws);
  int *pi = reinterpret_cast<int *>(pm + 1024);
  note_launch(2);
  (void)launch_kernel(argmax_stage1, dim3(np), dim3(256), 0, st, 1, 1, n, x, pm, pi);
  (void)launch_kernel(argmax_stage2, dim3(1), dim3(1024), 0, st, 1, 1, np, pm, pi, out);
  return check_cuda(cudaGetLastError(), "argmax launch");
}

int rope_gather_launch(int B, int rot, int max_pos, const int32_t *lens, const float *tc, const float *ts, float *oc,
                       float *os, cudaStream_t st) {
  note_launch();
  (void)launch_kernel(rope_gather_kernel, dim3(B), dim3(rot), 0, st, 1, 1, B, rot, max_pos, lens, tc, ts, oc, os);
  return check_cuda(cudaGetLastError(), "rope_gather launch");
}

int q8_dequant_launch(int rows, int cols, const uint32_t *w, const float *scales, float *out, cudaStream_t st) {
  const size_t nw = (size_t)rows * (cols / 4);
  note_launch();
  (void)launch_kernel(q8_dequant_kernel, dim3((unsigned)((nw + 255) / 256)), dim3(256), 0, st, 1, 1, rows, cols, w, scales, out);
  return check_cuda(cudaGetLastError(), "q8_dequant launch");
}

}  // namespace q35
