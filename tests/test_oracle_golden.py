"""Pins the CPU oracle against the golden fixtures (tests/golden/make_golden.py).

The fixtures are the outputs of the HF transformers Qwen3.5 torch functions that
the reference's Burn code (src/text_modules.rs) ports line by line.  CPU only.
"""
import numpy as np

import oracle
from conftest import max_rel_err

TOL = 2e-6  # f32 restatement vs f32 torch: reduction-order rounding only


def test_conv1d_update(golden):
    y, st = oracle.conv1d_update(golden["convu_x"], golden["convu_state"], golden["convu_w"])
    assert max_rel_err(y, golden["convu_y"]) < TOL
    np.testing.assert_array_equal(st, golden["convu_state_out"])


def test_conv1d_prefill(golden):
    for has_prev in (0, 1):
        y, st = oracle.conv1d_prefill(golden["convp_x"], golden["convp_prev"], golden["convp_w"], has_prev)
        assert max_rel_err(y, golden[f"convp{has_prev}_y"]) < TOL
        np.testing.assert_array_equal(st, golden[f"convp{has_prev}_state_out"])


def test_l2norm(golden):
    assert max_rel_err(oracle.l2norm(golden["l2_x"]), golden["l2_y"]) < TOL


def test_rmsnorm_gated(golden):
    y = oracle.rmsnorm_gated(golden["rmsg_x"], golden["rmsg_z"], golden["rmsg_w"])
    assert max_rel_err(y, golden["rmsg_y"]) < TOL


def test_rmsnorm(golden):
    assert max_rel_err(oracle.rmsnorm(golden["rms_x"], golden["rms_w"]), golden["rms_y"]) < TOL


def test_rope_tables(golden):
    cos, sin = oracle.rope_tables(golden["rope_pos"], rot=64, theta=1e7)
    # inv_freq is formed as exp(i*(-ln theta/dim)) in the reference and as
    # theta**(-i/dim) upstream; at position 1000 the f32 angles differ by ~1e-4.
    assert np.max(np.abs(cos - golden["rope_cos"])) < 2e-4
    assert np.max(np.abs(sin - golden["rope_sin"])) < 2e-4
    assert np.max(np.abs(cos[:5] - golden["rope_cos"][:5])) < 2e-6


def test_recurrent_gdr(golden):
    for tag in ("rec_small", "rec_d128"):
        out, S = oracle.recurrent_gdr(*(golden[f"{tag}_{n}"] for n in ("q", "k", "v", "g", "beta", "S0")))
        assert max_rel_err(out, golden[f"{tag}_out"]) < 1e-5, tag
        assert max_rel_err(S, golden[f"{tag}_S"]) < 1e-5, tag


def test_chunk_gdr(golden):
    for tag in ("chk_small", "chk_rf2"):
        args = [golden[f"{tag}_{n}"] for n in ("q", "k", "v", "g", "beta", "S0")]
        out, S = oracle.chunk_gdr(*args, chunk=int(golden[f"{tag}_chunk"]))
        assert max_rel_err(out, golden[f"{tag}_out"]) < 1e-5, tag
        assert max_rel_err(S, golden[f"{tag}_S"]) < 1e-5, tag


def test_chunk_equals_recurrent(golden):
    """The reference's implied identity: prefill (chunked) and decode
    (token-by-token) produce the same outputs and final state."""
    tag = "chk_rf2"
    args = [golden[f"{tag}_{n}"] for n in ("q", "k", "v", "g", "beta", "S0")]
    oc, Sc = oracle.chunk_gdr(*args, chunk=64)
    orr, Sr = oracle.recurrent_gdr(*args)
    assert max_rel_err(oc, orr) < 1e-5
    assert max_rel_err(Sc, Sr) < 1e-5


def test_gqa_decode(golden):
    G = golden
    B, Hkv, L, D = G["gqa_K"].shape
    cap = L + 3
    kc = np.zeros((B, Hkv, cap, D), np.float32)
    vc = np.zeros((B, Hkv, cap, D), np.float32)
    kc[:, :, :L] = G["gqa_K"]
    vc[:, :, :L] = G["gqa_V"]
    lens = np.full(B, L, np.int32)
    out, kc2, vc2, lens2 = oracle.gqa_decode(G["gqa_qg"], G["gqa_kn"], G["gqa_vn"], G["gqa_qnw"], G["gqa_knw"],
                                             G["gqa_cos"], G["gqa_sin"], kc, vc, lens, rot=G["gqa_cos"].shape[-1])
    assert max_rel_err(out, G["gqa_out"]) < 1e-5
    assert max_rel_err(kc2[:, :, :L + 1], G["gqa_Kall"]) < 1e-6
    assert max_rel_err(vc2[:, :, :L + 1], G["gqa_Vall"]) < 1e-6
    assert (lens2 == L + 1).all()


def test_gate_proj_prefill(golden):
    G = golden
    beta, g = oracle.gate_proj(G["gate_x"], G["gate_wb"], G["gate_wa"], G["gate_alog"], G["gate_dt"], mode=1)
    assert max_rel_err(beta, G["gate_beta"]) < TOL
    assert max_rel_err(g, G["gate_g"]) < TOL


def test_gate_proj_decode_matches_prefill(golden):
    """kernels.rs:174-247 (8-way split partial sums) vs the prefill matmul path:
    same values up to summation order."""
    G = golden
    b0, g0 = oracle.gate_proj(G["gate_x"], G["gate_wb"], G["gate_wa"], G["gate_alog"], G["gate_dt"], mode=0)
    assert max_rel_err(b0, G["gate_beta"]) < 1e-5
    assert max_rel_err(g0, G["gate_g"]) < 1e-5
