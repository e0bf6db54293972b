"""Parity of q35_gqa_prefill (q/k norm + RoPE + cache append + causal tcgen05
flash attention + sigmoid gate over a prompt) against the CPU oracle's
restatement of text_modules.rs:866-936 with the causal mask of
model.rs:59-67, through the C ABI.  Tolerance: max rel err <= 1e-3 per tensor
(outputs, caches); lens exact."""
import numpy as np
import pytest
import torch

import oracle
import q35attn
from conftest import max_rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-3
D = 256


def rope(pos, rot):
    return oracle.rope_tables(np.asarray(pos, np.int64), rot=rot, theta=1e7)


def make(seed, B, T, Hq, Hkv, lens0, cap, wscale=0.0):
    rng = np.random.RandomState(seed)
    f = np.float32
    d = {
        "qg": rng.randn(B, T, Hq, 2 * D).astype(f),
        "kn": rng.randn(B, T, Hkv, D).astype(f),
        "vn": rng.randn(B, T, Hkv, D).astype(f),
        "qn_w": (wscale * rng.randn(D)).astype(f),
        "kn_w": (wscale * rng.randn(D)).astype(f),
        "K": np.zeros((B, Hkv, cap, D), f),
        "V": np.zeros((B, Hkv, cap, D), f),
    }
    for b in range(B):
        d["K"][b, :, :lens0[b]] = rng.randn(Hkv, lens0[b], D)
        d["V"][b, :, :lens0[b]] = rng.randn(Hkv, lens0[b], D)
    return d


def run_prefill(B, T, Hq, Hkv, lens0, cap, seed, rot=64, wscale=0.0, max_len=None):
    lens0 = np.asarray(lens0, np.int32)
    d = make(seed, B, T, Hq, Hkv, lens0, cap, wscale)
    pos = lens0[:, None].astype(np.int64) + np.arange(T)[None, :]
    cos, sin = rope(pos, rot) if rot > 0 else (np.zeros((B, T, 0), np.float32),) * 2
    dev = torch.device("cuda:0")
    Td = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    Kc, Vc, lens = Td(d["K"]), Td(d["V"]), Td(lens0)
    ws = q35attn.GqaPrefillWorkspace(B, Hq, Hkv, cap, T, max_len=max_len or cap)
    out = q35attn.gqa_prefill(Td(d["qg"]), Td(d["kn"]), Td(d["vn"]), Td(d["qn_w"]), Td(d["kn_w"]),
                              Td(cos) if rot > 0 else None, Td(sin) if rot > 0 else None, Kc, Vc, lens,
                              workspace=ws, rotary_dim=rot)
    torch.cuda.synchronize()
    ref, oK, oV, olens = oracle.gqa_prefill(d["qg"], d["kn"], d["vn"], d["qn_w"], d["kn_w"], cos, sin,
                                            d["K"], d["V"], lens0, rot=rot)
    return out, Kc, Vc, lens, ws, (ref, oK, oV, olens)


def check(res):
    out, Kc, Vc, lens, ws, (ref, oK, oV, olens) = res
    assert ws.status() == 0
    np.testing.assert_array_equal(lens.cpu().numpy(), olens)
    e = max_rel_err(out.cpu().numpy().reshape(ref.shape), ref)
    assert e <= TOL, e
    assert max_rel_err(Kc.cpu().numpy(), oK) <= TOL
    assert max_rel_err(Vc.cpu().numpy(), oV) == 0.0
    return e


def test_config3_prompt_1024():
    """The config-3 prompt: B = 1, T = 1024 tokens, empty cache, 8/2 heads."""
    e = check(run_prefill(1, 1024, 8, 2, [0], 1024 + 64, seed=1))
    print(f"config3 prompt: out {e:.2e}")


@pytest.mark.parametrize("T,lens0", [(70, [33]), (1, [5]), (129, [0]), (64, [64]), (200, [0, 131])])
def test_ragged_prompts_and_history(T, lens0):
    check(run_prefill(len(lens0), T, 8, 2, lens0, max(lens0) + T + 7, seed=T))


@pytest.mark.parametrize("Hq,Hkv", [(4, 4), (16, 2), (4, 1)])
def test_group_sizes(Hq, Hkv):
    check(run_prefill(1, 150, Hq, Hkv, [20], 200, seed=Hq * 10 + Hkv))


@pytest.mark.parametrize("rot,wscale", [(0, 0.0), (256, 0.1), (64, 0.1)])
def test_rotary_and_norm_weights(rot, wscale):
    check(run_prefill(1, 96, 8, 2, [10], 128, seed=rot + 3, rot=rot, wscale=wscale))


def test_prefill_then_decode():
    """Prompt through q35_gqa_prefill, then decode steps through q35_gqa_decode
    on the same cache: matches the oracle's prefill + decode."""
    B, T, Hq, Hkv, cap = 1, 300, 8, 2, 400
    out, Kc, Vc, lens, ws, (ref, oK, oV, olens) = run_prefill(B, T, Hq, Hkv, [0], cap, seed=9)
    assert max_rel_err(out.cpu().numpy().reshape(ref.shape), ref) <= TOL
    rng = np.random.RandomState(10)
    dws = q35attn.GqaWorkspace(B, Hq, Hkv, cap)
    dev = torch.device("cuda:0")
    Td = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    qn_w = kn_w = np.zeros(D, np.float32)
    for _ in range(5):
        qg = rng.randn(B, Hq, 2 * D).astype(np.float32)
        kn = rng.randn(B, Hkv, D).astype(np.float32)
        vn = rng.randn(B, Hkv, D).astype(np.float32)
        cos, sin = rope(olens, 64)
        o = q35attn.gqa_decode(Td(qg), Td(kn), Td(vn), Td(qn_w), Td(kn_w), Td(cos), Td(sin), Kc, Vc, lens,
                               workspace=dws)
        r, oK, oV, olens = oracle.gqa_decode(qg, kn, vn, qn_w, kn_w, cos, sin, oK, oV, olens)
        assert max_rel_err(o.cpu().numpy(), r) <= TOL
    np.testing.assert_array_equal(lens.cpu().numpy(), olens)


def test_full_cache_is_flagged_and_skipped():
    B, T, Hq, Hkv, cap = 1, 40, 8, 2, 64
    lens0 = np.array([30], np.int32)  # 30 + 40 > 64
    d = make(3, B, T, Hq, Hkv, lens0, cap)
    cos, sin = rope(lens0[:, None] + np.arange(T)[None, :], 64)
    dev = torch.device("cuda:0")
    Td = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    Kc, Vc, lens = Td(d["K"]), Td(d["V"]), Td(lens0)
    ws = q35attn.GqaPrefillWorkspace(B, Hq, Hkv, cap, T)
    q35attn.gqa_prefill(Td(d["qg"]), Td(d["kn"]), Td(d["vn"]), Td(d["qn_w"]), Td(d["kn_w"]), Td(cos), Td(sin),
                        Kc, Vc, lens, workspace=ws)
    torch.cuda.synchronize()
    assert ws.status() & q35attn.STATUS_CACHE_FULL
    assert lens.item() == 30
    assert torch.equal(Kc.cpu(), torch.from_numpy(d["K"]))
