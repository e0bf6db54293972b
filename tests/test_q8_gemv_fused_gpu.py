"""Parity of q35_q8_gemv_fused (several Q8F projections of one input in one
launch, the decoder's RMSNorm fused in front, the MLP's SwiGLU behind) against
the oracle's restatements: RMSNorm of text_modules.rs:800-809 with the residual
add of :1053-1085, the split-K GEMV of kernels.rs:103-165 (mode 0 every row,
mode 1 the reference's row coverage) and the MLP of :999-1011.  f32 tolerance:
max rel err <= 1e-4 for plain projections, 1e-3 once the norm and SiLU are in
the chain (reduction order differs from the reference's)."""
import numpy as np
import pytest
import torch

import oracle
import q35attn
from conftest import max_rel_err
from test_q8_gemv_oracle import q8_random

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def words(wq):
    return dev(np.ascontiguousarray(wq).view(np.int32))


def rmsnorm(h, w, eps):
    h = h.astype(np.float32)
    inv = np.float32(1.0) / np.sqrt((h * h).mean() + np.float32(eps))
    return (h * inv) * (1.0 + w)


def silu(v):
    with np.errstate(over="ignore"):
        return v / (1.0 + np.exp(-v))


def make(rng, ind, outs):
    mats = [q8_random(rng, ind, o) for o in outs]
    return mats, [(words(q), dev(s)) for q, s in mats]


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("ind,outs", [
    (2048, [6144, 2048]),          # GatedDeltaNet in_proj_qkv + in_proj_z
    (2048, [4096, 512, 512]),      # attention q (with gate) / k / v
    (2048, [256, 512, 768, 1024]),  # four segments of different widths
    (6144, [2048]),                # down_proj
    (1000, [256, 512]),            # ragged last row box
])
def test_segments_match_oracle(ind, outs, mode):
    rng = np.random.RandomState(ind + len(outs) * 31 + mode)
    mats, W = make(rng, ind, outs)
    x = rng.randn(ind).astype(np.float32)
    ys = q35attn.q8_gemv_fused(dev(x), W, mode=mode)
    for (q, s), y in zip(mats, ys):
        assert max_rel_err(y.cpu().numpy(), oracle.q8_gemv(x, q, s, exact=(mode == 0))) <= 1e-4


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("with_res", [False, True])
def test_norm_prologue(mode, with_res):
    rng = np.random.RandomState(7 + mode + 2 * with_res)
    ind, outs, eps = 2048, [6144, 2048], 1e-6
    mats, W = make(rng, ind, outs)
    x = rng.randn(ind).astype(np.float32)
    res = rng.randn(ind).astype(np.float32) if with_res else None
    nw = (0.1 * rng.randn(ind)).astype(np.float32)
    sum_out = torch.full((ind,), np.nan, device="cuda") if with_res else None
    x_out = torch.full((ind,), np.nan, device="cuda")
    ys = q35attn.q8_gemv_fused(dev(x), W, residual=dev(res) if with_res else None, norm_w=dev(nw), eps=eps,
                               sum_out=sum_out, x_out=x_out, mode=mode)
    h = x + res if with_res else x
    xn = rmsnorm(h, nw, eps)
    assert max_rel_err(x_out.cpu().numpy(), xn) <= 1e-5
    if with_res:
        assert torch.equal(sum_out.cpu(), torch.from_numpy(h))
    for (q, s), y in zip(mats, ys):
        assert max_rel_err(y.cpu().numpy(), oracle.q8_gemv(xn, q, s, exact=(mode == 0))) <= 1e-3


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("ind,inter", [(2048, 6144), (1024, 512)])
def test_swiglu_mlp(ind, inter, mode):
    rng = np.random.RandomState(ind + inter + mode)
    mats, W = make(rng, ind, [inter, inter])
    x = rng.randn(ind).astype(np.float32)
    res = rng.randn(ind).astype(np.float32)
    nw = (0.1 * rng.randn(ind)).astype(np.float32)
    h_out = torch.empty(ind, device="cuda")
    act = q35attn.q8_gemv_fused(dev(x), W, residual=dev(res), norm_w=dev(nw), sum_out=h_out, swiglu=True,
                                mode=mode)
    xn = rmsnorm(x + res, nw, 1e-6)
    (qu, su), (qg, sg) = mats
    up = oracle.q8_gemv(xn, qu, su, exact=(mode == 0))
    gate = oracle.q8_gemv(xn, qg, sg, exact=(mode == 0))
    assert max_rel_err(act.cpu().numpy(), up * silu(gate)) <= 1e-3
    assert torch.equal(h_out.cpu(), torch.from_numpy(x + res))
    # without the norm: plain x into both projections
    act2 = q35attn.q8_gemv_fused(dev(x), W, swiglu=True, mode=mode)
    up = oracle.q8_gemv(x, qu, su, exact=(mode == 0))
    gate = oracle.q8_gemv(x, qg, sg, exact=(mode == 0))
    assert max_rel_err(act2.cpu().numpy(), up * silu(gate)) <= 1e-3


def test_deterministic_and_matches_single_gemv():
    rng = np.random.RandomState(3)
    mats, W = make(rng, 2048, [6144, 2048])
    x = dev(rng.randn(2048).astype(np.float32))
    a = q35attn.q8_gemv_fused(x, W, mode=1)
    b = q35attn.q8_gemv_fused(x, W, mode=1)
    for ya, yb, (w, s) in zip(a, b, W):
        assert torch.equal(ya, yb)
        assert max_rel_err(ya.cpu().numpy(), q35attn.q8_gemv(x, w, s, mode=1).cpu().numpy()) <= 1e-5


def test_rejects_bad_calls():
    rng = np.random.RandomState(4)
    _, W = make(rng, 256, [256, 512])
    x = torch.randn(256, device="cuda")
    nw = torch.zeros(256, device="cuda")
    with pytest.raises(q35attn.Q35Error):  # sum_out aliasing x
        q35attn.q8_gemv_fused(x, W, norm_w=nw, sum_out=x)
    with pytest.raises(q35attn.Q35Error):  # swiglu with unequal widths
        q35attn.q8_gemv_fused(x, W, swiglu=True)
    with pytest.raises(q35attn.Q35Error):  # residual without the norm
        q35attn.q8_gemv_fused(x, W, residual=x.clone())
