"""CPU reference of the hybrid decoder stack (test infrastructure: the checker
for q35attn.stack.HybridStack, never part of the product).

Restates the reference's layer loop with the oracle's pinned pieces:
TextModel::forward / TextForCausalLM::forward (model.rs:27-140),
DecoderLayer::forward (text_modules.rs:1053-1085), RMSNorm (:800-809), the MLP
(:999-1011), GatedDeltaNet::forward (:483-667) and Attention::forward
(:842-944).  Decode projections use the oracle's restatement of the Q8F
split-K GEMV (kernels.rs:103-165); prefill projections are dense f32 matmuls
of the dequantised weights (Linear::forward).  Embedding lookup
(kernels.rs:15-45), lm_head (kernels.rs:251-291 at decode, the dense matmul of
model.rs:129-138 at prefill) and argmax are written here with numpy.
"""
from __future__ import annotations

import numpy as np

import oracle


def _q8(W):
    """(int8 values [rows, cols], scales [rows, cols/64]) of a q35attn.stack.Q8F."""
    q = W.words.contiguous().view(-1).cpu().numpy().view(np.int8).reshape(W.rows, W.cols)
    return q, W.scales.cpu().numpy()


def _deq(q, s):
    return q.astype(np.float32) * np.repeat(s, 64, axis=1)


def _rmsnorm(x, w, eps):
    x = x.astype(np.float32)
    inv = (1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + np.float32(eps))).astype(np.float32)
    return (x * inv) * (1.0 + w)


def _silu(x):
    with np.errstate(over="ignore"):  # exp(-x) = inf for very negative x gives silu = -0, as on the GPU
        return x / (1.0 + np.exp(-x))


class StackRef:
    def __init__(self, stack):
        c = stack.cfg
        self.cfg, self.cap, self.exact = c, stack.cap, stack.gemv_mode == 0
        self.emb_q, self.emb_s = _q8(stack.embed)
        self._emb_dense = None
        self.final_norm = stack.final_norm.cpu().numpy()
        self.layers = []
        for L in stack.layers:
            R = {"kind": L["kind"]}
            for k, v in L.items():
                if k == "kind":
                    continue
                if hasattr(v, "words"):
                    R[k] = _q8(v)
                elif k not in ("conv_state", "rec_state", "K", "V", "lens"):
                    R[k] = v.cpu().numpy()
            self.layers.append(R)
        pos = np.arange(self.cap, dtype=np.int64)
        self.cos, self.sin = oracle.rope_tables(pos, rot=c.rot, theta=c.theta)

    def _reset(self):
        c = self.cfg
        for R in self.layers:
            if R["kind"] == "linear":
                R["cst"] = np.zeros((1, c.conv_dim, c.conv_k - 1), np.float32)
                R["S"] = np.zeros((1, c.gdn_hv, 128, 128), np.float32)
            else:
                R["Kc"] = np.zeros((1, c.gqa_hkv, self.cap, 256), np.float32)
                R["Vc"] = np.zeros((1, c.gqa_hkv, self.cap, 256), np.float32)
                R["lens"] = np.zeros(1, np.int32)

    def _embed(self, ids):
        return self.emb_q[ids].astype(np.float32) * np.repeat(self.emb_s[ids], 64, axis=1)

    def _logits(self, x):
        if self._emb_dense is None:  # the tied lm_head weight, dequantised once
            self._emb_dense = self.emb_q.astype(np.float32) * np.repeat(self.emb_s, 64, axis=1)
        return self._emb_dense @ x

    def prefill(self, ids):
        """Returns (first generated token, logits of the last prompt position)."""
        c = self.cfg
        self._reset()
        ids = np.asarray(ids)
        T = ids.size
        h = self._embed(ids)
        mm = lambda x, W: x @ _deq(*W)
        for R in self.layers:
            x = _rmsnorm(h, R["in_norm"], c.eps)
            if R["kind"] == "linear":
                mixed, z = mm(x, R["qkv"]), mm(x, R["z"])
                beta, g = oracle.gate_proj(x, R["w_b"], R["w_a"], R["a_log"], R["dt_bias"], mode=1)
                core, R["cst"], R["S"] = oracle.gdn_prefill(mixed[None], z[None], beta[None], g[None], R["conv_w"],
                                                           R["norm_w"], R["cst"], False, R["S"], False, c.gdn_hk,
                                                           c.gdn_hv, eps=c.eps)
                attn = mm(core.reshape(T, -1), R["out"])
            else:
                qg = mm(x, R["q"]).reshape(1, T, c.gqa_hq, 512)
                kk = mm(x, R["k"]).reshape(1, T, c.gqa_hkv, 256)
                vv = mm(x, R["v"]).reshape(1, T, c.gqa_hkv, 256)
                core, R["Kc"], R["Vc"], R["lens"] = oracle.gqa_prefill(
                    qg, kk, vv, R["qn_w"], R["kn_w"], self.cos[None, :T], self.sin[None, :T], R["Kc"], R["Vc"],
                    R["lens"], rot=c.rot, eps=c.eps)
                attn = mm(core.reshape(T, -1), R["o"])
            h = h + attn
            x = _rmsnorm(h, R["post_norm"], c.eps)
            act = mm(x, R["up"]) * _silu(mm(x, R["gate"]))
            h = h + mm(act, R["down"])
        logits = self._logits(_rmsnorm(h[-1], self.final_norm, c.eps))
        return int(np.argmax(logits)), logits

    def decode(self, tok):
        """One decode step on token tok.  Returns (next token, logits)."""
        c = self.cfg
        gemv = lambda x, W: oracle.q8_gemv(x, W[0], W[1], exact=self.exact)
        h = self._embed(np.array([tok]))[0]
        for R in self.layers:
            x = _rmsnorm(h, R["in_norm"], c.eps)
            if R["kind"] == "linear":
                mixed, z = gemv(x, R["qkv"]), gemv(x, R["z"])
                beta, g = oracle.gate_proj(x[None], R["w_b"], R["w_a"], R["a_log"], R["dt_bias"], mode=0)
                core, R["cst"], R["S"] = oracle.gdn_decode(mixed[None], z[None], beta, g, R["conv_w"], R["norm_w"],
                                                          R["cst"], R["S"], c.gdn_hk, c.gdn_hv, eps=c.eps)
                attn = gemv(core[0], R["out"])
            else:
                pos = int(R["lens"][0])
                qg = gemv(x, R["q"]).reshape(1, c.gqa_hq, 512)
                kk = gemv(x, R["k"]).reshape(1, c.gqa_hkv, 256)
                vv = gemv(x, R["v"]).reshape(1, c.gqa_hkv, 256)
                core, R["Kc"], R["Vc"], R["lens"] = oracle.gqa_decode(
                    qg, kk, vv, R["qn_w"], R["kn_w"], self.cos[pos:pos + 1], self.sin[pos:pos + 1], R["Kc"],
                    R["Vc"], R["lens"], rot=c.rot, eps=c.eps)
                attn = gemv(core[0], R["o"])
            h = h + attn
            x = _rmsnorm(h, R["post_norm"], c.eps)
            act = gemv(x, R["up"]) * _silu(gemv(x, R["gate"]))
            h = h + gemv(act, R["down"])
        logits = self._logits(_rmsnorm(h, self.final_norm, c.eps))
        return int(np.argmax(logits)), logits
