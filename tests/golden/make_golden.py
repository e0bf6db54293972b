"""Generate the golden fixtures that pin the CPU oracle.

The reference (Rust/Burn, inventwithdean/Qwen-3.5) ships no tests or golden
vectors and cannot be built in this container.  Its attention code in
src/text_modules.rs is a line-by-line port of the HF transformers Qwen3.5 torch
functions (`torch_causal_conv1d_update`, `l2norm`,
`torch_chunk_gated_delta_rule`, `torch_recurrent_gated_delta_rule`,
`Qwen3_5RMSNormGated`, `Qwen3_5RMSNorm`, `apply_rotary_pos_emb`,
`eager_attention_forward`, `Qwen3_5TextRotaryEmbedding`).  This script imports
those functions from the installed transformers package (imported, not copied)
and records their outputs on seeded inputs; tests/test_oracle_golden.py then
checks the oracle against them.

Run from the repo root:  python tests/golden/make_golden.py
Output: tests/golden/golden.npz (a few hundred KB).
"""
from __future__ import annotations

import os
import types

import numpy as np
import torch
import torch.nn.functional as F
import transformers
from transformers.models.qwen3_5 import modeling_qwen3_5 as M
from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))


def n(x):
    return x.detach().to(torch.float32).contiguous().numpy()


def main():
    rng = np.random.RandomState(20261201)
    G = {"transformers_version": np.array(transformers.__version__)}

    # --- causal_conv1d_update (text_modules.rs:134-162) -------------------
    B, Cc, K = 2, 24, 4
    x = rng.randn(B, Cc, 1).astype(np.float32)
    st = rng.randn(B, Cc, K - 1).astype(np.float32)
    w = (0.5 * rng.randn(Cc, K)).astype(np.float32)
    st_t = t(st).clone()
    y = M.torch_causal_conv1d_update(t(x), st_t, t(w), None, None)
    G.update(convu_x=x[..., 0], convu_state=st, convu_w=w, convu_y=n(y)[..., 0], convu_state_out=n(st_t))

    # --- causal_conv1d_fn (text_modules.rs:164-182, :531-552) -------------
    T = 10
    xp = rng.randn(B, T, Cc).astype(np.float32)
    prev = rng.randn(B, Cc, K - 1).astype(np.float32)
    for has_prev in (0, 1):
        inp = t(xp).transpose(1, 2)
        if has_prev:
            inp = torch.cat([t(prev), inp], 2)
        yy = F.conv1d(inp, t(w).unsqueeze(1), None, padding=K - 1, groups=Cc)[:, :, : inp.shape[2]]
        yy = F.silu(yy)[:, :, -T:]
        new_state = inp[:, :, -(K - 1):]
        G[f"convp{has_prev}_y"] = n(yy.transpose(1, 2))
        G[f"convp{has_prev}_state_out"] = n(new_state)
    G.update(convp_x=xp, convp_prev=prev, convp_w=w)

    # --- l2norm (text_modules.rs:184-187) ---------------------------------
    xl = rng.randn(5, 128).astype(np.float32)
    G.update(l2_x=xl, l2_y=n(M.l2norm(t(xl), dim=-1, eps=1e-6)))

    # --- RMSNormGated (text_modules.rs:85-117) ----------------------------
    xg = rng.randn(6, 128).astype(np.float32)
    zg = rng.randn(6, 128).astype(np.float32)
    wg = (1.0 + 0.1 * rng.randn(128)).astype(np.float32)
    m = M.Qwen3_5RMSNormGated(128, eps=1e-6)
    with torch.no_grad():
        m.weight.copy_(t(wg))
    G.update(rmsg_x=xg, rmsg_z=zg, rmsg_w=wg, rmsg_y=n(m(t(xg), t(zg))))

    # --- RMSNorm (1+w) (text_modules.rs:800-809) ---------------------------
    xr = rng.randn(4, 256).astype(np.float32)
    wr = (0.1 * rng.randn(256)).astype(np.float32)
    m2 = M.Qwen3_5RMSNorm(256, eps=1e-6)
    with torch.no_grad():
        m2.weight.copy_(t(wr))
    G.update(rms_x=xr, rms_w=wr, rms_y=n(m2(t(xr))))

    # --- rotary tables (text_modules.rs:23-82) ----------------------------
    cfg = Qwen3_5TextConfig(head_dim=256, hidden_size=2048, num_attention_heads=8, num_key_value_heads=2,
                            rope_parameters={"rope_type": "default", "rope_theta": 10000000,
                                             "partial_rotary_factor": 0.25, "mrope_interleaved": True,
                                             "mrope_section": [11, 11, 10]})
    rot = M.Qwen3_5TextRotaryEmbedding(cfg)
    pos = np.array([0, 1, 2, 7, 63, 100, 1000], dtype=np.int64)
    cos, sin = rot(t(np.zeros(1)), torch.from_numpy(pos)[None, :])
    G.update(rope_pos=pos, rope_cos=n(cos[0]), rope_sin=n(sin[0]))

    # --- recurrent gated delta rule (text_modules.rs:365-443) -------------
    for tag, (B, T, H, D) in {"rec_small": (2, 5, 2, 16), "rec_d128": (1, 4, 2, 128)}.items():
        q = rng.randn(B, T, H, D).astype(np.float32)
        k = rng.randn(B, T, H, D).astype(np.float32)
        v = rng.randn(B, T, H, D).astype(np.float32)
        g = (-np.log1p(np.exp(rng.randn(B, T, H)))).astype(np.float32)
        beta = (1 / (1 + np.exp(-rng.randn(B, T, H)))).astype(np.float32)
        S0 = (0.02 * rng.randn(B, H, D, D)).astype(np.float32)
        o, S = M.torch_recurrent_gated_delta_rule(t(q), t(k), t(v), t(g), t(beta), t(S0), True,
                                                  use_qk_l2norm_in_kernel=True)
        G.update({f"{tag}_q": q, f"{tag}_k": k, f"{tag}_v": v, f"{tag}_g": g, f"{tag}_beta": beta,
                  f"{tag}_S0": S0, f"{tag}_out": n(o), f"{tag}_S": n(S)})

    # --- chunked gated delta rule (text_modules.rs:189-363) ---------------
    # ragged T (not a multiple of the chunk) and Hv = 2*Hk (k heads expanded
    # k*rf + r as text_modules.rs:597-615 does)
    for tag, (B, T, Hk, Hv, D, CH) in {"chk_small": (1, 37, 2, 2, 16, 16),
                                      "chk_rf2": (1, 70, 1, 2, 32, 64)}.items():
        q = rng.randn(B, T, Hk, D).astype(np.float32)
        k = rng.randn(B, T, Hk, D).astype(np.float32)
        v = rng.randn(B, T, Hv, D).astype(np.float32)
        g = (-np.log1p(np.exp(rng.randn(B, T, Hv)))).astype(np.float32)
        beta = (1 / (1 + np.exp(-rng.randn(B, T, Hv)))).astype(np.float32)
        S0 = (0.02 * rng.randn(B, Hv, D, D)).astype(np.float32)
        rf = Hv // Hk
        qe = t(q).repeat_interleave(rf, dim=2)
        ke = t(k).repeat_interleave(rf, dim=2)
        o, S = M.torch_chunk_gated_delta_rule(qe, ke, t(v), t(g), t(beta), chunk_size=CH, initial_state=t(S0),
                                              output_final_state=True, use_qk_l2norm_in_kernel=True)
        G.update({f"{tag}_q": q, f"{tag}_k": k, f"{tag}_v": v, f"{tag}_g": g, f"{tag}_beta": beta,
                  f"{tag}_S0": S0, f"{tag}_out": n(o), f"{tag}_S": n(S), f"{tag}_chunk": np.array(CH)})

    # --- gated GQA decode core (text_modules.rs:842-936) ------------------
    B, Hq, Hkv, D, R, L = 2, 4, 2, 32, 16, 9
    qg = rng.randn(B, 1, Hq, 2 * D).astype(np.float32)
    kn = rng.randn(B, 1, Hkv, D).astype(np.float32)
    vn = rng.randn(B, 1, Hkv, D).astype(np.float32)
    qn_w = (0.1 * rng.randn(D)).astype(np.float32)
    kn_w = (0.1 * rng.randn(D)).astype(np.float32)
    Kc = rng.randn(B, Hkv, L, D).astype(np.float32)
    Vc = rng.randn(B, Hkv, L, D).astype(np.float32)
    ang = (L * 0.37 * np.arange(1, R // 2 + 1)).astype(np.float32)[None, :].repeat(B, 0)
    cs = np.concatenate([np.cos(ang), np.cos(ang)], -1).astype(np.float32)
    sn = np.concatenate([np.sin(ang), np.sin(ang)], -1).astype(np.float32)
    qn = M.Qwen3_5RMSNorm(D)
    kn_m = M.Qwen3_5RMSNorm(D)
    with torch.no_grad():
        qn.weight.copy_(t(qn_w))
        kn_m.weight.copy_(t(kn_w))
    qs = qn(t(qg[..., :D])).transpose(1, 2)
    ks = kn_m(t(kn)).transpose(1, 2)
    vs = t(vn).transpose(1, 2)
    qs, ks = M.apply_rotary_pos_emb(qs, ks, t(cs)[:, None, :], t(sn)[:, None, :])
    Kall = torch.cat([t(Kc), ks], 2)
    Vall = torch.cat([t(Vc), vs], 2)
    mod = types.SimpleNamespace(num_key_value_groups=Hq // Hkv, training=False)
    ao, _ = M.eager_attention_forward(mod, qs, Kall, Vall, None, scaling=D ** -0.5)
    ao = ao.reshape(B, 1, Hq * D) * torch.sigmoid(t(qg[..., D:]).reshape(B, 1, Hq * D))
    G.update(gqa_qg=qg[:, 0], gqa_kn=kn[:, 0], gqa_vn=vn[:, 0], gqa_qnw=qn_w, gqa_knw=kn_w, gqa_K=Kc,
             gqa_V=Vc, gqa_cos=cs, gqa_sin=sn, gqa_out=n(ao[:, 0]), gqa_Kall=n(Kall), gqa_Vall=n(Vall))

    # --- prefill beta / g (text_modules.rs:578-595) -----------------------
    N, IN, H = 3, 64, 4
    xh = rng.randn(N, IN).astype(np.float32)
    wb = (0.2 * rng.randn(IN, H)).astype(np.float32)
    wa = (0.2 * rng.randn(IN, H)).astype(np.float32)
    a_log = np.log(rng.uniform(0.01, 16.0, H)).astype(np.float32)
    dt = (1.0 + 0.5 * rng.randn(H)).astype(np.float32)
    xa = t(xh) @ t(wa) + t(dt)
    gp = -torch.exp(t(a_log)) * F.softplus(xa, beta=1.0, threshold=20.0)
    bp = torch.sigmoid(t(xh) @ t(wb))
    G.update(gate_x=xh, gate_wb=wb, gate_wa=wa, gate_alog=a_log, gate_dt=dt, gate_beta=n(bp), gate_g=n(gp))

    np.savez_compressed(OUT, **G)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    torch.manual_seed(0)
    main()
