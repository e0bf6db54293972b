// q35_host_parity.cpp -- parity of the C++ host layer (q35_modules.hpp) against
// the CPU oracle (oracle/q35_oracle.h), the way the reference's modules are
// driven: a layer's first forward is the chunked path (the prompt) and fills
// the cache, later single-token forwards decode from it, and a further prompt
// continues from the cached state.  Test infrastructure: built and run by
// tests/test_host_cpp_gpu.py.  Exit status 0 when every tensor is within
// max|x - ref| / max|ref| <= 1e-3; one line per check on stdout.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <random>
#include <vector>

#include "q35_modules.hpp"
#include "q35_oracle.h"

using q35::host::AttentionCore;
using q35::host::Cache;
using q35::host::Error;
using q35::host::GatedDeltaNetCore;
using q35::host::TextConfig;

static int g_fail = 0;

static void cuda_ok(cudaError_t e) {
  if (e != cudaSuccess) {
    std::fprintf(stderr, "CUDA: %s\n", cudaGetErrorString(e));
    std::exit(2);
  }
}

struct Dev {
  float *p = nullptr;
  size_t n = 0;
  explicit Dev(const std::vector<float> &h) : n(h.size()) {
    cuda_ok(cudaMalloc(&p, n * sizeof(float)));
    cuda_ok(cudaMemcpy(p, h.data(), n * sizeof(float), cudaMemcpyHostToDevice));
  }
  explicit Dev(size_t count) : n(count) { cuda_ok(cudaMalloc(&p, n * sizeof(float))); }
  ~Dev() { cudaFree(p); }
  std::vector<float> host() const {
    std::vector<float> h(n);
    cuda_ok(cudaMemcpy(h.data(), p, n * sizeof(float), cudaMemcpyDeviceToHost));
    return h;
  }
};

static std::vector<float> randn(std::mt19937 &rng, size_t n, float scale = 1.0f) {
  std::normal_distribution<float> d(0.0f, scale);
  std::vector<float> v(n);
  for (auto &x : v) x = d(rng);
  return v;
}

static void expect(const char *what, const std::vector<float> &got, const std::vector<float> &ref) {
  double num = 0.0, den = 0.0;
  for (size_t i = 0; i < ref.size(); ++i) {
    num = std::fmax(num, std::fabs((double)got[i] - ref[i]));
    den = std::fmax(den, std::fabs((double)ref[i]));
  }
  const double e = num / (den > 0 ? den : 1.0);
  const bool ok = e <= 1e-3 && std::isfinite(e);
  std::printf("%-44s max rel err %.3e %s\n", what, e, ok ? "ok" : "FAIL");
  if (!ok) ++g_fail;
}

static void gated_delta_net(const TextConfig &cfg, cudaStream_t st) {
  std::mt19937 rng(1);
  const int B = 2, Hk = cfg.linear_num_key_heads, Hv = cfg.linear_num_value_heads, DK = cfg.linear_key_head_dim,
            DV = cfg.linear_value_head_dim, K = cfg.linear_conv_kernel_dim, C = cfg.conv_dim();
  const std::vector<float> conv_w = randn(rng, (size_t)C * K, 0.5f), norm_w = randn(rng, DV, 0.1f);
  std::vector<float> norm1(norm_w);
  for (auto &w : norm1) w += 1.0f;
  Dev d_conv_w(conv_w), d_norm_w(norm1);
  GatedDeltaNetCore core(cfg, 3, d_conv_w.p, d_norm_w.p);
  Cache cache(cfg, 24, B, 256);
  std::vector<float> ost((size_t)B * C * (K - 1), 0.0f), oS((size_t)B * Hv * DK * DV, 0.0f);
  auto gates = [&](int T, std::vector<float> &beta, std::vector<float> &g) {
    beta = randn(rng, (size_t)B * T * Hv);
    g = randn(rng, (size_t)B * T * Hv);
    for (auto &b : beta) b = 1.0f / (1.0f + std::exp(-b));
    for (auto &x : g) x = -std::log1p(std::exp(x));
  };
  auto step = [&](int T, const char *label) {  // one forward of the layer, on the host layer and on the oracle
    const std::vector<float> x = randn(rng, (size_t)B * T * C), z = randn(rng, (size_t)B * T * Hv * DV);
    std::vector<float> beta, g;
    gates(T, beta, g);
    Dev dx(x), dz(z), db(beta), dg(g), dout((size_t)B * T * Hv * DV);
    const bool decode = T == 1 && cache.has_conv_state(3);
    const bool had_state = cache.has_conv_state(3);
    core.forward(dx.p, dz.p, db.p, dg.p, B, T, &cache, dout.p, st);
    std::vector<float> ref((size_t)B * T * Hv * DV);
    if (decode)
      q35o_gdn_decode(B, Hk, Hv, DK, DV, K, x.data(), z.data(), beta.data(), g.data(), conv_w.data(), norm1.data(),
                      ost.data(), oS.data(), ref.data(), cfg.rms_norm_eps);
    else
      q35o_gdn_prefill(B, T, Hk, Hv, DK, DV, K, 64, x.data(), z.data(), beta.data(), g.data(), conv_w.data(),
                       norm1.data(), ost.data(), had_state, oS.data(), had_state, ref.data(), cfg.rms_norm_eps);
    cuda_ok(cudaStreamSynchronize(st));
    expect(label, dout.host(), ref);
  };
  step(70, "GatedDeltaNet prompt T=70 (chunked, no state)");
  for (int i = 0; i < 3; ++i) step(1, "GatedDeltaNet decode step (recurrent)");
  step(5, "GatedDeltaNet prompt T=5 on the cached state");
  step(1, "GatedDeltaNet decode step after it");
  std::vector<float> S((size_t)B * Hv * DK * DV), cst((size_t)B * C * (K - 1));
  cuda_ok(cudaMemcpy(S.data(), cache.recurrent_state(3), S.size() * 4, cudaMemcpyDeviceToHost));
  cuda_ok(cudaMemcpy(cst.data(), cache.conv_state(3), cst.size() * 4, cudaMemcpyDeviceToHost));
  expect("GatedDeltaNet recurrent state in the cache", S, oS);
  expect("GatedDeltaNet conv state in the cache", cst, ost);

  // cache: None -- the chunked rule from zero state, nothing kept
  {
    const int T = 3;
    const std::vector<float> x = randn(rng, (size_t)B * T * C), z = randn(rng, (size_t)B * T * Hv * DV);
    std::vector<float> beta, g;
    gates(T, beta, g);
    Dev dx(x), dz(z), db(beta), dg(g), dout((size_t)B * T * Hv * DV);
    core.forward(dx.p, dz.p, db.p, dg.p, B, T, nullptr, dout.p, st);
    std::vector<float> ref((size_t)B * T * Hv * DV), st0((size_t)B * C * (K - 1), 0.0f),
        S0((size_t)B * Hv * DK * DV, 0.0f);
    q35o_gdn_prefill(B, T, Hk, Hv, DK, DV, K, 64, x.data(), z.data(), beta.data(), g.data(), conv_w.data(),
                     norm1.data(), st0.data(), 0, S0.data(), 0, ref.data(), cfg.rms_norm_eps);
    cuda_ok(cudaStreamSynchronize(st));
    expect("GatedDeltaNet without a cache (T=3)", dout.host(), ref);
  }
}

static void attention(const TextConfig &cfg, cudaStream_t st) {
  std::mt19937 rng(2);
  const int B = 2, Hq = cfg.num_attention_heads, Hkv = cfg.num_key_value_heads, D = cfg.head_dim,
            rot = cfg.rotary_dim;
  const int64_t cap = 48;
  const std::vector<float> qn = randn(rng, D, 0.1f), kn = randn(rng, D, 0.1f);
  Dev d_qn(qn), d_kn(kn);
  AttentionCore core(cfg, 7, d_qn.p, d_kn.p);
  Cache cache(cfg, 24, B, cap);
  std::vector<float> oK((size_t)B * Hkv * cap * D, 0.0f), oV(oK.size(), 0.0f);
  std::vector<int32_t> olens(B, 0);
  auto step = [&](int T, const char *label) {
    const std::vector<float> qg = randn(rng, (size_t)B * T * Hq * 2 * D), k = randn(rng, (size_t)B * T * Hkv * D),
                             v = randn(rng, (size_t)B * T * Hkv * D);
    std::vector<int64_t> pos((size_t)B * T);
    for (int b = 0; b < B; ++b)
      for (int t = 0; t < T; ++t) pos[(size_t)b * T + t] = olens[b] + t;
    std::vector<float> cs((size_t)B * T * rot), sn(cs.size());
    q35o_rope_tables(B * T, pos.data(), rot, 1e7f, cs.data(), sn.data());
    Dev dq(qg), dk(k), dv(v), dc(cs), ds(sn), dout((size_t)B * T * Hq * D);
    core.forward(dq.p, dk.p, dv.p, dc.p, ds.p, B, T, cache, dout.p, st);
    std::vector<float> ref((size_t)B * T * Hq * D);
    if (T == 1)
      q35o_gqa_decode(B, Hq, Hkv, D, rot, cap, qg.data(), k.data(), v.data(), qn.data(), kn.data(), cs.data(),
                      sn.data(), oK.data(), oV.data(), olens.data(), ref.data(), cfg.rms_norm_eps);
    else
      q35o_gqa_prefill(B, T, Hq, Hkv, D, rot, cap, qg.data(), k.data(), v.data(), qn.data(), kn.data(), cs.data(),
                       sn.data(), oK.data(), oV.data(), olens.data(), ref.data(), cfg.rms_norm_eps);
    cuda_ok(cudaStreamSynchronize(st));
    expect(label, dout.host(), ref);
  };
  step(37, "Attention prompt T=37 (empty cache)");
  for (int i = 0; i < 3; ++i) step(1, "Attention decode step");
  step(6, "Attention prompt T=6 on the cached keys");
  core.check_status(st);
  const std::vector<int32_t> lens = cache.host_lengths(7, st);
  const bool lens_ok = lens[0] == olens[0] && lens[1] == olens[1] && lens[0] == 46;
  std::printf("%-44s %d %d %s\n", "Attention cached lengths", lens[0], lens[1], lens_ok ? "ok" : "FAIL");
  if (!lens_ok) ++g_fail;
  std::vector<float> Kc(oK.size());
  cuda_ok(cudaMemcpy(Kc.data(), cache.key_states(7), Kc.size() * 4, cudaMemcpyDeviceToHost));
  expect("Attention key cache", Kc, oK);

  // two more steps fill the cache (48); the third has no room: the step is
  // skipped on the device and check_status raises, where the reference panics
  step(1, "Attention decode step (cache 47 of 48)");
  step(1, "Attention decode step (cache 48 of 48)");
  {
    const std::vector<float> qg = randn(rng, (size_t)B * Hq * 2 * D), k = randn(rng, (size_t)B * Hkv * D);
    std::vector<float> cs((size_t)B * rot, 1.0f), sn((size_t)B * rot, 0.0f);
    Dev dq(qg), dk(k), dv(k), dc(cs), ds(sn), dout((size_t)B * Hq * D);
    core.forward(dq.p, dk.p, dv.p, dc.p, ds.p, B, 1, cache, dout.p, st);
    int code = 0;
    try {
      core.check_status(st);
    } catch (const Error &e) {
      code = e.code();
    }
    std::printf("%-44s code %d %s\n", "Attention past capacity raises", code, code == Q35_ERR_CAPACITY ? "ok" : "FAIL");
    if (code != Q35_ERR_CAPACITY) ++g_fail;
  }
}

static void argument_errors(const TextConfig &cfg, cudaStream_t st) {
  int code = 0;
  try {
    Cache bad(cfg, 0, 1, 16);
  } catch (const Error &e) {
    code = e.code();
  }
  std::printf("%-44s code %d %s\n", "Cache with no layers raises", code, code == Q35_ERR_INVALID_ARG ? "ok" : "FAIL");
  if (code != Q35_ERR_INVALID_ARG) ++g_fail;
  code = 0;
  try {
    Dev w(16), n(16);
    GatedDeltaNetCore core(cfg, 0, w.p, n.p);
    Cache c(cfg, 2, 3, 16);
    core.forward(w.p, w.p, w.p, w.p, 2, 1, &c, w.p, st);  // batch 2 against a batch-3 cache
  } catch (const Error &e) {
    code = e.code();
  }
  std::printf("%-44s code %d %s\n", "cache batch mismatch raises", code, code == Q35_ERR_INVALID_ARG ? "ok" : "FAIL");
  if (code != Q35_ERR_INVALID_ARG) ++g_fail;
}

int main() {
  cudaStream_t st;
  cuda_ok(cudaStreamCreate(&st));
  const TextConfig cfg;  // the 2B model's attention shapes
  try {
    gated_delta_net(cfg, st);
    attention(cfg, st);
    argument_errors(cfg, st);
  } catch (const Error &e) {
    std::printf("unexpected q35::host::Error %d: %s\n", e.code(), e.what());
    return 1;
  }
  cuda_ok(cudaStreamDestroy(st));
  std::printf("%s\n", g_fail ? "FAILED" : "all checks passed");
  return g_fail ? 1 : 0;
}
