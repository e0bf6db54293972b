"""Parity of q35_gdn_decode (fused conv + l2norm + gated delta rule + gated
RMS norm) against the CPU oracle, through the C ABI.

Tolerance: max|x - ref| / max|ref| <= 1e-3 per tensor, on every step's output
and on the final recurrent and conv state (the contract stated for the port).
"""
import numpy as np
import pytest
import torch

import oracle
import q35attn
from conftest import max_rel_err
from gdn_data import gdn_inputs

pytestmark = pytest.mark.gpu
TOL = 1e-3


def run_gdn(B, Hk, Hv, steps, seed, split=0, K=4):
    d = gdn_inputs(seed, B, Hk, Hv, steps, K)
    dev = torch.device("cuda:0")
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    conv_w, norm_w = T(d["conv_w"]), T(d["norm_w"])
    cst, S = T(d["conv0"]), T(d["S0"])
    ost, oS = d["conv0"].copy(), d["S0"].copy()
    worst = 0.0
    for t in range(steps):
        out = q35attn.gdn_decode(T(d["x"][t]), T(d["z"][t]), T(d["beta"][t]), T(d["g"][t]), conv_w, norm_w, cst, S,
                                 num_k_heads=Hk, num_v_heads=Hv, split=split)
        ref, ost, oS = oracle.gdn_decode(d["x"][t], d["z"][t], d["beta"][t], d["g"][t], d["conv_w"], d["norm_w"],
                                         ost, oS, Hk, Hv)
        worst = max(worst, max_rel_err(out.cpu().numpy(), ref))
    torch.cuda.synchronize()
    return worst, max_rel_err(S.cpu().numpy(), oS), max_rel_err(cst.cpu().numpy(), ost)


def test_config0_256_steps():
    """B=1, 16/16 heads, d=128, 256 sequential steps."""
    e_out, e_S, e_conv = run_gdn(1, 16, 16, 256, seed=0)
    print(f"config0: out {e_out:.2e} state {e_S:.2e} conv {e_conv:.2e}")
    assert e_out <= TOL and e_S <= TOL and e_conv <= 1e-6


@pytest.mark.parametrize("split", [-1, 1, 2, 4, 8])
def test_every_column_split(split):
    e_out, e_S, e_conv = run_gdn(3, 16, 16, 12, seed=10 + split, split=split)
    assert e_out <= TOL and e_S <= TOL and e_conv <= 1e-6


@pytest.mark.parametrize("Hk,Hv,split", [(8, 16, 0), (8, 16, 4), (4, 16, 2), (8, 24, 1), (8, 16, -1), (8, 24, -1)])
def test_value_heads_share_key_heads(Hk, Hv, split):
    """num_v_heads > num_k_heads: k-head h//rf expanded as text_modules.rs:597-615."""
    e_out, e_S, e_conv = run_gdn(2, Hk, Hv, 8, seed=20 + Hv + split, split=split)
    assert e_out <= TOL and e_S <= TOL and e_conv <= 1e-6


@pytest.mark.parametrize("K", [2, 3])
@pytest.mark.parametrize("split", [0, -1])
def test_short_conv_kernels(K, split):
    e_out, e_S, e_conv = run_gdn(2, 16, 16, 6, seed=30 + K, K=K, split=split)
    assert e_out <= TOL and e_S <= TOL and e_conv <= 1e-6


def test_batched_256_sequences_against_sampled_oracle():
    """Config-4 GDN shapes: 256 sequences; every sequence is independent, so
    the oracle checks a sample of them."""
    B, steps = 256, 3
    d = gdn_inputs(7, B, 16, 16, steps)
    dev = torch.device("cuda:0")
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    cst, S = T(d["conv0"]), T(d["S0"])
    outs = []
    for t in range(steps):
        outs.append(q35attn.gdn_decode(T(d["x"][t]), T(d["z"][t]), T(d["beta"][t]), T(d["g"][t]), T(d["conv_w"]),
                                       T(d["norm_w"]), cst, S, num_k_heads=16, num_v_heads=16).cpu().numpy())
    Sg = S.cpu().numpy()
    for b in (0, 1, 77, 255):
        ost, oS = d["conv0"][b:b + 1].copy(), d["S0"][b:b + 1].copy()
        for t in range(steps):
            ref, ost, oS = oracle.gdn_decode(d["x"][t][b:b + 1], d["z"][t][b:b + 1], d["beta"][t][b:b + 1],
                                             d["g"][t][b:b + 1], d["conv_w"], d["norm_w"], ost, oS, 16, 16)
            assert max_rel_err(outs[t][b:b + 1], ref) <= TOL
        assert max_rel_err(Sg[b:b + 1], oS) <= TOL


def test_identity_when_beta_zero_and_no_decay():
    """g = 0 and beta = 0 leave the recurrent state unchanged (a property the
    reference relies on for padded tokens)."""
    B = 2
    d = gdn_inputs(3, B, 16, 16, 1)
    dev = torch.device("cuda:0")
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    S = T(d["S0"])
    q35attn.gdn_decode(T(d["x"][0]), T(d["z"][0]), torch.zeros(B, 16, device=dev), torch.zeros(B, 16, device=dev),
                       T(d["conv_w"]), T(d["norm_w"]), T(d["conv0"]), S, num_k_heads=16, num_v_heads=16)
    np.testing.assert_array_equal(S.cpu().numpy(), d["S0"])
