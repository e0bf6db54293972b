"""Pins the oracle's Q8F GEMV (oracle/q35_oracle.c q35o_q8_gemv, restating
kernels.rs:103-165 and the split count of :504).  The reference ships no test
vectors for it, so the pins are (1) a float64 dequantise-and-matmul for the
exact mode, (2) known answers for the reference's row coverage: with W, x and
the scales all ones every output equals the number of input rows the split-K
kernel walks, which for the 2B projections is 2016 / 2000 / 2048 rows (the
counts derived from :119-131 and :504), and (3) a planted case in which only
the rows the reference skips carry weight."""
import numpy as np
import pytest

import oracle


def ref_rows(in_dim, out_dim):
    splits = min(max(25000 // out_dim, 1), max(in_dim // 80, 1))
    chunk = in_dim // splits
    return splits * (chunk // 8) * 8


def q8_random(rng, ind, outd):
    wq = rng.randint(-127, 128, size=(ind, outd)).astype(np.int8)
    sc = np.abs(0.01 * rng.randn(ind, outd // 64)).astype(np.float32)
    return wq, sc


@pytest.mark.parametrize("ind,outd", [(2048, 6144), (2048, 512), (6144, 2048), (100, 64)])
def test_exact_mode_matches_float64(ind, outd):
    rng = np.random.RandomState(ind + outd)
    wq, sc = q8_random(rng, ind, outd)
    x = rng.randn(ind).astype(np.float32)
    dense = wq.astype(np.float64) * np.repeat(sc.astype(np.float64), 64, axis=1)
    ref = x.astype(np.float64) @ dense
    y = oracle.q8_gemv(x, wq, sc, exact=True)
    assert np.max(np.abs(y - ref)) / np.max(np.abs(ref)) <= 1e-5


@pytest.mark.parametrize("ind,outd,rows", [
    (2048, 2048, 2016),   # in_proj_z, out_proj, o_proj: 12 splits of 170 -> 168 rows each
    (2048, 4096, 2016),   # q_proj (8 heads x [query | gate] x 256): 6 splits of 341 -> 336
    (2048, 512, 2000),    # k_proj, v_proj: 25 splits of 81 -> 80
    (2048, 6144, 2048),   # in_proj_qkv, up, gate: 4 splits of 512
    (6144, 2048, 6144),   # down: 12 splits of 512
    (100, 64, 96),        # 1 split of 100 -> 96
])
def test_reference_row_coverage_known_answers(ind, outd, rows):
    assert ref_rows(ind, outd) == rows
    ones = np.ones(ind, np.float32)
    y = oracle.q8_gemv(ones, np.ones((ind, outd), np.int8), np.ones((ind, outd // 64), np.float32), exact=False)
    assert np.all(y == rows)
    y = oracle.q8_gemv(ones, np.ones((ind, outd), np.int8), np.ones((ind, outd // 64), np.float32), exact=True)
    assert np.all(y == ind)


def test_only_skipped_rows_planted():
    # in 2048 -> out 2048: 12 splits of 170 rows, the last 2 of each split and
    # rows 2040..2047 are never read by the reference kernel
    ind = outd = 2048
    skipped = [s * 170 + j for s in range(12) for j in (168, 169)] + list(range(2040, 2048))
    assert len(skipped) == ind - ref_rows(ind, outd)
    wq = np.zeros((ind, outd), np.int8)
    wq[skipped, :] = 5
    sc = np.ones((ind, outd // 64), np.float32)
    x = np.ones(ind, np.float32)
    assert np.all(oracle.q8_gemv(x, wq, sc, exact=False) == 0.0)
    assert np.all(oracle.q8_gemv(x, wq, sc, exact=True) == 5.0 * len(skipped))
