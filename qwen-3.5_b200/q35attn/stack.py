"""The Qwen3.5 hybrid decoder stack (config 3) over the q35attn kernels.

Mirrors TextForCausalLM / TextModel / DecoderLayer of the reference
(inventwithdean/Qwen-3.5 src/model.rs:27-140, src/text_modules.rs:1040-1085)
with its two forward paths:

* prefill (seq_len > 1): dense projections over the dequantised Q8F weights
  (``Linear::forward``, text_modules.rs:499-506, 578-595, 663, 858-888, 941,
  1007-1009) as q35_q8_gemm tensor-core GEMMs that dequantise each weight tile
  on load, the chunked GDN core (q35_gdn_prefill), the
  causal GQA core (q35_gqa_prefill), then the tied-embedding logits of the last
  position (model.rs:126-138) and argmax;
* decode (seq_len == 1): Q8F GEMVs for every projection (kernels.rs:103-165;
  ``gemv_mode`` 1 walks the same input rows as the reference's kernel, 0 all
  rows), the GDN gate kernel (kernels.rs:174-247), the recurrent GDN core and
  the GQA flash-decode, the Q8F lm_head (kernels.rs:251-291) and argmax
  (kernels.rs:298-371).  One decode step is captured in a CUDA graph; the token
  and the positions stay on the device, so steps run back to back.

Weights are random-initialised as BASELINE config 3 states (int8 uniform in
[-127, 127], per-64 scales |N(0, 0.01)|; no checkpoint is available).  The
tensors that the reference keeps in f32 (conv, norms, in_proj_a/b, A_log,
dt_bias; main.rs:205-218) get the reference's init values where it has them
(RMSNorm weights 0 used as 1 + w, RMSNormGated weight 1) and seeded normals
otherwise.
"""
from __future__ import annotations

import dataclasses

import torch

from . import ops


@dataclasses.dataclass(frozen=True)
class StackConfig:
    hidden: int = 2048
    layer_types: tuple = tuple(("full" if (i + 1) % 4 == 0 else "linear") for i in range(24))  # text_config.rs:69-93
    gdn_hk: int = 16
    gdn_hv: int = 16
    conv_k: int = 4
    gqa_hq: int = 8
    gqa_hkv: int = 2
    rot: int = 64          # partial_rotary_factor 0.25 of head_dim 256
    theta: float = 1e7
    inter: int = 6144
    vocab: int = 248320
    eps: float = 1e-6

    @property
    def conv_dim(self):
        return 2 * self.gdn_hk * 128 + self.gdn_hv * 128


QWEN35_2B = StackConfig()


class Q8F:
    """A Q8F matrix [rows, cols]: int8 values packed 4 per u32 word (stored as
    int32 [rows, cols/4]) and f32 scales [rows, cols/64]."""

    def __init__(self, rows, cols, gen, device):
        q = torch.randint(-127, 128, (rows, cols), dtype=torch.int8, device=device, generator=gen)
        self.words = q.view(torch.int32).contiguous()
        self.scales = (torch.randn(rows, cols // 64, device=device, generator=gen) * 0.01).abs_()
        self.rows, self.cols = rows, cols


class HybridStack:
    def __init__(self, cfg: StackConfig = QWEN35_2B, capacity: int = 2048, seed: int = 0, device="cuda",
                 gemv_mode: int = 1, prefill_chunk: int = 2048, fused: bool = True, gate_overlap: bool = True):
        self.cfg, self.cap, self.dev, self.gemv_mode = cfg, capacity, torch.device(device), gemv_mode
        self.fused, self._plan = fused, None
        self.gate_overlap = gate_overlap
        self._side = torch.cuda.Stream(self.dev) if gate_overlap else None  # created outside any capture
        g = torch.Generator(device=self.dev)
        g.manual_seed(seed)
        c, dev = cfg, self.dev

        def randn(*shape, scale=1.0):
            return torch.randn(*shape, device=dev, generator=g) * scale

        self.embed = Q8F(c.vocab, c.hidden, g, dev)
        self.final_norm = torch.zeros(c.hidden, device=dev)
        self.layers = []
        for kind in c.layer_types:
            L = {"kind": kind, "in_norm": torch.zeros(c.hidden, device=dev),
                 "post_norm": torch.zeros(c.hidden, device=dev),
                 "up": Q8F(c.hidden, c.inter, g, dev), "gate": Q8F(c.hidden, c.inter, g, dev),
                 "down": Q8F(c.inter, c.hidden, g, dev)}
            if kind == "linear":
                L.update(qkv=Q8F(c.hidden, c.conv_dim, g, dev), z=Q8F(c.hidden, c.gdn_hv * 128, g, dev),
                         out=Q8F(c.gdn_hv * 128, c.hidden, g, dev),
                         w_b=randn(c.hidden, c.gdn_hv, scale=0.02), w_a=randn(c.hidden, c.gdn_hv, scale=0.02),
                         a_log=torch.log(torch.rand(c.gdn_hv, device=dev, generator=g) * 15 + 1),
                         dt_bias=torch.ones(c.gdn_hv, device=dev),
                         conv_w=randn(c.conv_dim, c.conv_k, scale=0.25), norm_w=torch.ones(128, device=dev),
                         conv_state=torch.zeros(1, c.conv_dim, c.conv_k - 1, device=dev),
                         rec_state=torch.zeros(1, c.gdn_hv, 128, 128, device=dev))
            else:
                L.update(q=Q8F(c.hidden, c.gqa_hq * 512, g, dev), k=Q8F(c.hidden, c.gqa_hkv * 256, g, dev),
                         v=Q8F(c.hidden, c.gqa_hkv * 256, g, dev), o=Q8F(c.gqa_hq * 256, c.hidden, g, dev),
                         qn_w=torch.zeros(256, device=dev), kn_w=torch.zeros(256, device=dev),
                         K=torch.zeros(1, c.gqa_hkv, capacity, 256, device=dev),
                         V=torch.zeros(1, c.gqa_hkv, capacity, 256, device=dev),
                         lens=torch.zeros(1, dtype=torch.int32, device=dev))
            self.layers.append(L)
        # RoPE tables (text_modules.rs:23-82): cos/sin = cat(f, f), f = pos * theta^(-2i/rot)
        inv = 1.0 / (c.theta ** (torch.arange(0, c.rot, 2, device=dev, dtype=torch.float32) / c.rot))
        ang = torch.arange(capacity, device=dev, dtype=torch.float32)[:, None] * inv[None, :]
        self.rope_cos = torch.cat([ang.cos(), ang.cos()], -1).contiguous()
        self.rope_sin = torch.cat([ang.sin(), ang.sin()], -1).contiguous()
        self.gqa_layers = [L for L in self.layers if L["kind"] == "full"]
        self.prefill_chunk = prefill_chunk
        self._decode_buffers()
        self.graph = None

    # ------------------------------------------------------------ state
    def reset(self):
        for L in self.layers:
            if L["kind"] == "linear":
                L["conv_state"].zero_()
                L["rec_state"].zero_()
            else:
                L["lens"].zero_()

    def _decode_buffers(self):
        c, dev = self.cfg, self.dev
        e = lambda *s: torch.empty(*s, device=dev)
        self.b = {"h": e(c.hidden), "h2": e(c.hidden), "x": e(c.hidden), "xg": e(c.hidden), "attn": e(c.hidden),
                  "mlp": e(c.hidden),
                  "mixed": e(1, c.conv_dim), "z": e(1, c.gdn_hv * 128), "beta": e(1, c.gdn_hv), "g": e(1, c.gdn_hv),
                  "core": e(1, max(c.gdn_hv * 128, c.gqa_hq * 256)), "qg": e(1, c.gqa_hq, 512),
                  "kk": e(1, c.gqa_hkv, 256), "vv": e(1, c.gqa_hkv, 256), "up": e(c.inter), "gt": e(c.inter),
                  "act": e(c.inter), "logits": e(c.vocab), "cos": e(1, c.rot), "sin": e(1, c.rot),
                  "tok": torch.zeros(1, dtype=torch.int32, device=dev)}
        self.gqa_ws = ops.GqaWorkspace(1, c.gqa_hq, c.gqa_hkv, self.cap, device=dev)
        self.argmax_ws = ops.ArgmaxWorkspace(dev)

    def weight_bytes(self):
        """Bytes of all weights (Q8F words + scales and the f32 tensors)."""
        n = self.embed.words.numel() * 4 + self.embed.scales.numel() * 4 + self.final_norm.numel() * 4
        for L in self.layers:
            for k, v in L.items():
                if isinstance(v, Q8F):
                    n += v.words.numel() * 4 + v.scales.numel() * 4
                elif torch.is_tensor(v) and k not in ("conv_state", "rec_state", "K", "V", "lens"):
                    n += v.numel() * v.element_size()
        return n

    def gemv(self, x, W: Q8F, y):
        return ops.q8_gemv(x, W.words, W.scales, y, mode=self.gemv_mode)

    # ------------------------------------------------------------ decode
    def _decode_step(self):
        """One token: embedding of self.b['tok'] -> ... -> argmax into self.b['tok']."""
        if self.fused:
            return self._decode_step_fused()
        c, b = self.cfg, self.b
        ops.q8_embedding(b["tok"], self.embed.words, self.embed.scales, b["h"].view(1, -1))
        if self.gqa_layers:  # every GQA layer decodes at the same position
            ops.rope_gather(self.gqa_layers[0]["lens"], self.rope_cos, self.rope_sin, b["cos"], b["sin"])
        resid = None  # the previous layer's MLP output, added into h by the next norm
        for L in self.layers:
            ops.add_rmsnorm(b["mlp"] if resid else b["h"], L["in_norm"], b["x"],
                            residual=b["h"] if resid else None, sum_out=b["h"] if resid else None, eps=c.eps)
            if L["kind"] == "linear":
                core = b["core"][:, :c.gdn_hv * 128]
                self.gemv(b["x"], L["qkv"], b["mixed"].view(-1))
                self.gemv(b["x"], L["z"], b["z"].view(-1))
                ops.gdn_gate(b["x"].view(1, -1), L["w_b"], L["w_a"], L["a_log"], L["dt_bias"], mode=0,
                             beta=b["beta"], g=b["g"])
                ops.gdn_decode(b["mixed"], b["z"], b["beta"], b["g"], L["conv_w"], L["norm_w"], L["conv_state"],
                               L["rec_state"], core, num_k_heads=c.gdn_hk, num_v_heads=c.gdn_hv, eps=c.eps)
                self.gemv(core.view(-1), L["out"], b["attn"])
            else:
                core = b["core"][:, :c.gqa_hq * 256]
                self.gemv(b["x"], L["q"], b["qg"].view(-1))
                self.gemv(b["x"], L["k"], b["kk"].view(-1))
                self.gemv(b["x"], L["v"], b["vv"].view(-1))
                ops.gqa_decode(b["qg"], b["kk"], b["vv"], L["qn_w"], L["kn_w"], b["cos"], b["sin"], L["K"], L["V"],
                               L["lens"], core, workspace=self.gqa_ws, max_len=self.cap, rotary_dim=c.rot,
                               eps=c.eps)
                self.gemv(core.view(-1), L["o"], b["attn"])
            # h += attn; x = RMSNorm(h) * (1 + post_norm)
            ops.add_rmsnorm(b["attn"], L["post_norm"], b["x"], residual=b["h"], sum_out=b["h"], eps=c.eps)
            self.gemv(b["x"], L["up"], b["up"])
            self.gemv(b["x"], L["gate"], b["gt"])
            ops.silu_mul(b["gt"], b["up"], b["act"])
            self.gemv(b["act"], L["down"], b["mlp"])
            resid = True
        ops.add_rmsnorm(b["mlp"], self.final_norm, b["x"], residual=b["h"], eps=c.eps)
        ops.q8_lm_head(b["x"], self.embed.words, self.embed.scales, b["logits"])
        ops.argmax(b["logits"], b["tok"], self.argmax_ws)

    def _fused_plan(self):
        """Prepared q35_q8_gemv_fused calls of every layer.  The residual stream
        alternates between two buffers (h, h2): each fused norm reads the
        current one and writes h + x into the other, so no kernel reads a
        buffer that the same launch writes."""
        c, b, m = self.cfg, self.b, self.gemv_mode
        W = lambda q: (q.words, q.scales)
        hs = [b["h"], b["h2"]]
        cur, plan = 0, []
        for i, L in enumerate(self.layers):
            first = i == 0
            kw = dict(norm_w=L["in_norm"], eps=c.eps, mode=m,
                      residual=None if first else hs[cur], sum_out=None if first else hs[1 - cur])
            xin = hs[cur] if first else b["mlp"]
            if not first:
                cur = 1 - cur
            if L["kind"] == "linear":  # in_proj_qkvz with the input norm; x_out feeds the gate projection
                front = ops.FusedGemv(xin, [W(L["qkv"]), W(L["z"])], [b["mixed"].view(-1), b["z"].view(-1)],
                                      x_out=b["x"], **kw)
                out = ops.FusedGemv(b["core"][:, :c.gdn_hv * 128].view(-1), [W(L["out"])], [b["attn"]], mode=m)
            else:
                front = ops.FusedGemv(xin, [W(L["q"]), W(L["k"]), W(L["v"])],
                                      [b["qg"].view(-1), b["kk"].view(-1), b["vv"].view(-1)], **kw)
                out = ops.FusedGemv(b["core"][:, :c.gqa_hq * 256].view(-1), [W(L["o"])], [b["attn"]], mode=m)
            mlp = ops.FusedGemv(b["attn"], [W(L["up"]), W(L["gate"])], [b["act"], b["gt"]], residual=hs[cur],
                                norm_w=L["post_norm"], eps=c.eps, sum_out=hs[1 - cur], swiglu=True, mode=m)
            cur = 1 - cur
            down = ops.FusedGemv(b["act"], [W(L["down"])], [b["mlp"]], mode=m)
            plan.append((L, front, out, mlp, down, (xin, kw["residual"])))
        return plan, hs[cur]

    def _decode_step_fused(self):
        c, b = self.cfg, self.b
        if self._plan is None:
            self._plan = self._fused_plan()
        plan, h_last = self._plan
        ops.q8_embedding(b["tok"], self.embed.words, self.embed.scales, b["h"].view(1, -1))
        if self.gqa_layers:
            ops.rope_gather(self.gqa_layers[0]["lens"], self.rope_cos, self.rope_sin, b["cos"], b["sin"])
        main = torch.cuda.current_stream(self.dev)
        for L, front, out, mlp, down, (xin, res) in plan:
            if L["kind"] == "linear" and self._side is not None and self.gate_overlap:
                # The gate projection reads only the layer input: a side branch recomputes the input norm and
                # runs it while the input projections stream their weights; the core waits for both.
                self._side.wait_stream(main)
                with torch.cuda.stream(self._side):
                    ops.add_rmsnorm(xin, L["in_norm"], b["xg"], residual=res, eps=c.eps)
                    ops.gdn_gate(b["xg"].view(1, -1), L["w_b"], L["w_a"], L["a_log"], L["dt_bias"], mode=0,
                                 beta=b["beta"], g=b["g"])
                front()
                main.wait_stream(self._side)
            else:
                front()
                if L["kind"] == "linear":
                    ops.gdn_gate(b["x"].view(1, -1), L["w_b"], L["w_a"], L["a_log"], L["dt_bias"], mode=0,
                                 beta=b["beta"], g=b["g"])
            if L["kind"] == "linear":
                ops.gdn_decode(b["mixed"], b["z"], b["beta"], b["g"], L["conv_w"], L["norm_w"], L["conv_state"],
                               L["rec_state"], b["core"][:, :c.gdn_hv * 128], num_k_heads=c.gdn_hk,
                               num_v_heads=c.gdn_hv, eps=c.eps)
            else:
                ops.gqa_decode(b["qg"], b["kk"], b["vv"], L["qn_w"], L["kn_w"], b["cos"], b["sin"], L["K"], L["V"],
                               L["lens"], b["core"][:, :c.gqa_hq * 256], workspace=self.gqa_ws, max_len=self.cap,
                               rotary_dim=c.rot, eps=c.eps)
            out()
            mlp()  # h += attn; act = up * silu(gate) of RMSNorm(h) * (1 + post_norm)
            down()
        ops.add_rmsnorm(b["mlp"], self.final_norm, b["x"], residual=h_last, eps=c.eps)
        ops.q8_lm_head(b["x"], self.embed.words, self.embed.scales, b["logits"])
        ops.argmax(b["logits"], b["tok"], self.argmax_ws)

    def profile_decode_step(self):
        """One eager decode step with CUDA events around the attention cores
        (q35_gdn_decode, q35_gqa_decode): returns (core ms, step ms)."""
        evs = []
        orig_gdn, orig_gqa = ops.gdn_decode, ops.gqa_decode

        def timed(fn):
            def run(*a, **k):
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                r = fn(*a, **k)
                e.record()
                evs.append((s, e))
                return r
            return run
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ops.gdn_decode, ops.gqa_decode = timed(orig_gdn), timed(orig_gqa)
        try:
            t0.record()
            self._decode_step()
            t1.record()
        finally:
            ops.gdn_decode, ops.gqa_decode = orig_gdn, orig_gqa
        torch.cuda.synchronize(self.dev)
        return sum(s.elapsed_time(e) for s, e in evs), t0.elapsed_time(t1)

    def capture(self):
        """Capture one decode step in a CUDA graph (after a warm-up step)."""
        st = torch.cuda.Stream(self.dev)
        st.wait_stream(torch.cuda.current_stream(self.dev))
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=st):
            self._decode_step()
        return self.graph

    def decode(self, n, tokens_out=None):
        """n greedy steps from the token in self.b['tok']; returns the device tokens."""
        if tokens_out is None:
            tokens_out = torch.empty(n, dtype=torch.int32, device=self.dev)
        for i in range(n):
            if self.graph is not None:
                self.graph.replay()
            else:
                self._decode_step()
            tokens_out[i:i + 1].copy_(self.b["tok"])
        return tokens_out

    # ------------------------------------------------------------ prefill
    def prefill(self, ids):
        """Run the prompt ids [T] (int32, device) through the stack from an empty
        cache; leaves the first generated token in self.b['tok'] and returns it."""
        c, dev = self.cfg, self.dev
        T = ids.numel()
        assert T <= self.cap
        self.reset()
        e = lambda *s: torch.empty(*s, device=dev)
        h = ops.q8_embedding(ids, self.embed.words, self.embed.scales)
        x, attn = e(T, c.hidden), e(T, c.hidden)

        # Linear::forward of the dequantised weights: q35_q8_gemm(_fused) on the
        # tensor cores, each weight tile dequantised on load; projections of the
        # same input share one launch, and the MLP's up / gate pair writes
        # up * silu(gate) from its epilogue
        gws = ops.q8_gemm_workspace(T, max(c.hidden, c.inter, c.gdn_hv * 128, c.gqa_hq * 256), dev)
        W = lambda q: (q.words, q.scales)

        def mm(a, q):
            return ops.q8_gemm(a, q.words, q.scales, workspace=gws)

        gdn_ws = ops.gdn_prefill_workspace(1, T, c.gdn_hk, c.gdn_hv, c.conv_k, dev)
        gqa_ws = ops.GqaPrefillWorkspace(1, c.gqa_hq, c.gqa_hkv, self.cap, T, device=dev)
        cos, sin = self.rope_cos[:T][None].contiguous(), self.rope_sin[:T][None].contiguous()
        act = e(T, c.inter)
        mlp = None
        for L in self.layers:
            if mlp is None:
                ops.add_rmsnorm(h, L["in_norm"], x, eps=c.eps)
            else:
                ops.add_rmsnorm(mlp, L["in_norm"], x, residual=h, sum_out=h, eps=c.eps)
            if L["kind"] == "linear":
                mixed, z = e(T, c.conv_dim), e(T, c.gdn_hv * 128)
                ops.q8_gemm_fused(x, [W(L["qkv"]), W(L["z"])], [mixed, z], workspace=gws)
                beta, g = ops.gdn_gate(x, L["w_b"], L["w_a"], L["a_log"], L["dt_bias"], mode=1)
                core = ops.gdn_prefill(mixed.view(1, T, -1), z.view(1, T, -1), beta.view(1, T, -1),
                                       g.view(1, T, -1), L["conv_w"], L["norm_w"], L["conv_state"], L["rec_state"],
                                       num_k_heads=c.gdn_hk, num_v_heads=c.gdn_hv, workspace=gdn_ws, eps=c.eps)
                attn = mm(core.view(T, -1), L["out"])
            else:
                qg, kk, vv = e(1, T, c.gqa_hq, 512), e(1, T, c.gqa_hkv, 256), e(1, T, c.gqa_hkv, 256)
                ops.q8_gemm_fused(x, [W(L["q"]), W(L["k"]), W(L["v"])],
                                  [qg.view(T, -1), kk.view(T, -1), vv.view(T, -1)], workspace=gws)
                core = ops.gqa_prefill(qg, kk, vv, L["qn_w"], L["kn_w"], cos, sin, L["K"], L["V"], L["lens"],
                                       workspace=gqa_ws, max_len=self.cap, rotary_dim=c.rot, eps=c.eps)
                attn = mm(core.view(T, -1), L["o"])
            ops.add_rmsnorm(attn, L["post_norm"], x, residual=h, sum_out=h, eps=c.eps)
            ops.q8_gemm_fused(x, [W(L["up"]), W(L["gate"])], [act, act], swiglu=True, workspace=gws)
            mlp = mm(act, L["down"])
        last = self.b["x"]
        ops.add_rmsnorm(mlp[T - 1:], self.final_norm, last.view(1, -1), residual=h[T - 1:], eps=c.eps)
        ops.q8_lm_head(last, self.embed.words, self.embed.scales, self.b["logits"])
        ops.argmax(self.b["logits"], self.b["tok"], self.argmax_ws)
        return self.b["tok"]

    def generate(self, ids, n_decode):
        """Prefill the prompt, then n_decode greedy decode steps.  Returns the
        n_decode + 1 generated tokens (the first comes from the prompt)."""
        first = self.prefill(ids).clone()
        rest = self.decode(n_decode)
        return torch.cat([first, rest])
