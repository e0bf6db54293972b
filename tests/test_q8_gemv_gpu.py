"""Parity of q35_q8_gemv against the oracle's restatement of kernels.rs:103-165:
mode 0 (every row) and mode 1 (the reference's row coverage), the 2B decode
projection shapes, the all-ones known answers, ragged column blocks, the
single-split path (lm_head width) and run-to-run determinism.  f32 tolerance:
max rel err <= 1e-4 (the summation order differs from the reference's)."""
import numpy as np
import pytest
import torch

import oracle
import q35attn
from conftest import max_rel_err
from test_q8_gemv_oracle import q8_random, ref_rows

pytestmark = pytest.mark.gpu


def to_dev(wq, sc, x):
    w = torch.from_numpy(np.ascontiguousarray(wq).view(np.int32)).cuda()
    return w, torch.from_numpy(sc).cuda(), torch.from_numpy(x).cuda()


SHAPES = [(2048, 6144), (2048, 2048), (2048, 4096), (2048, 512), (6144, 2048), (2048, 576), (1, 64), (100, 64)]


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("ind,outd", SHAPES)
def test_gemv_matches_oracle(ind, outd, mode):
    rng = np.random.RandomState(ind * 7 + outd + mode)
    wq, sc = q8_random(rng, ind, outd)
    x = rng.randn(ind).astype(np.float32)
    w, s, xd = to_dev(wq, sc, x)
    y = q35attn.q8_gemv(xd, w, s, mode=mode)
    ref = oracle.q8_gemv(x, wq, sc, exact=(mode == 0))
    if not np.any(ref):
        assert not torch.any(y).item()
    else:
        assert max_rel_err(y.cpu().numpy(), ref) <= 1e-4
    y2 = q35attn.q8_gemv(xd, w, s, mode=mode)  # deterministic split-K order
    assert torch.equal(y, y2)


@pytest.mark.parametrize("ind,outd", [(2048, 2048), (2048, 4096), (2048, 512), (2048, 6144), (7, 64)])
def test_row_coverage_known_answers(ind, outd):
    x = torch.ones(ind, device="cuda")
    w = torch.full((ind, outd // 4), 0x01010101, dtype=torch.int32, device="cuda")
    s = torch.ones(ind, outd // 64, device="cuda")
    assert torch.all(q35attn.q8_gemv(x, w, s, mode=1) == float(ref_rows(ind, outd))).item()
    assert torch.all(q35attn.q8_gemv(x, w, s, mode=0) == float(ind)).item()


def test_lm_head_width_single_split():
    rng = np.random.RandomState(5)
    ind, outd = 2048, 248320
    wq, sc = q8_random(rng, ind, outd)
    x = rng.randn(ind).astype(np.float32)
    w, s, xd = to_dev(wq, sc, x)
    y = q35attn.q8_gemv(xd, w, s, mode=0)
    cols = rng.choice(outd, 512, replace=False)
    dense = wq[:, cols].astype(np.float64) * sc[:, cols // 64].astype(np.float64)
    ref = x.astype(np.float64) @ dense
    assert max_rel_err(y.cpu().numpy()[cols], ref) <= 1e-4


def test_rejects_bad_shapes():
    x = torch.ones(64, device="cuda")
    w = torch.zeros(64, 8, dtype=torch.int32, device="cuda")  # out = 32: not a multiple of 64
    with pytest.raises(q35attn.Q35Error):
        q35attn.q8_gemv(x, w, torch.ones(64, 1, device="cuda"))
