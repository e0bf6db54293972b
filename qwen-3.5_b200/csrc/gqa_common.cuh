// gqa_common.cuh -- device helpers shared by the gated-GQA decode and prefill
// kernels (head_dim 256, text_config.rs:105).
#pragma once

#include "common.cuh"

namespace q35 {
namespace gqa {

constexpr int kHeadDim = 256;

// RMSNorm(1+w) + partial RoPE of one head vector held as 8 floats per lane
// (dims 4*lane..4*lane+3 and 128+4*lane..128+4*lane+3); `tmp` is a 256-float
// shared scratch for the rotate-half partner exchange.  Returns the result in
// x0/x1 (same layout).
__device__ __forceinline__ void norm_rope(float4 &x0, float4 &x1, const float *w, const float *cs,
                                          const float *sn, int rot, float eps, float *tmp, int lane) {
  float ss = x0.x * x0.x + x0.y * x0.y + x0.z * x0.z + x0.w * x0.w;
  ss += x1.x * x1.x + x1.y * x1.y + x1.z * x1.z + x1.w * x1.w;
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / (float)kHeadDim + eps);
  const float4 w0 = *reinterpret_cast<const float4 *>(w + 4 * lane);
  const float4 w1 = *reinterpret_cast<const float4 *>(w + 128 + 4 * lane);
  x0 = make_float4((x0.x * inv) * (1.0f + w0.x), (x0.y * inv) * (1.0f + w0.y), (x0.z * inv) * (1.0f + w0.z),
                   (x0.w * inv) * (1.0f + w0.w));
  x1 = make_float4((x1.x * inv) * (1.0f + w1.x), (x1.y * inv) * (1.0f + w1.y), (x1.z * inv) * (1.0f + w1.z),
                   (x1.w * inv) * (1.0f + w1.w));
  *reinterpret_cast<float4 *>(tmp + 4 * lane) = x0;
  *reinterpret_cast<float4 *>(tmp + 128 + 4 * lane) = x1;
  __syncwarp();
  const int half = rot >> 1;
  float r[8];
  const float xin[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int d = (e < 4 ? 4 * lane : 128 + 4 * lane) + (e & 3);
    if (d < rot) {
      const float rh = d < half ? -tmp[d + half] : tmp[d - half];
      r[e] = xin[e] * cs[d] + rh * sn[d];
    } else {
      r[e] = xin[e];
    }
  }
  __syncwarp();
  x0 = make_float4(r[0], r[1], r[2], r[3]);
  x1 = make_float4(r[4], r[5], r[6], r[7]);
}

}  // namespace gqa
}  // namespace q35
