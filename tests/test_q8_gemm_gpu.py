"""q35_q8_gemm -- the Q8F prefill projection (Linear::forward over the
dequantised weight, text_modules.rs:499-506, 663, 858-888, 941, 1007-1009) on
the tensor cores -- against the dense product x @ (q * s) in float64 and
against the oracle's Q8F row product (oracle.q8_gemv, every input row).

The kernel computes with bf16 hi/lo splits of x and of the f32 weight
(relative error near 2^-16 per product), so the tolerance here is
max rel err <= 1e-4, ten times tighter than the attention path's 1e-3."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle
import q35attn
from q35attn import _lib
from conftest import max_rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-4


def q8f(rng, rows, cols):
    q = rng.randint(-127, 128, size=(rows, cols)).astype(np.int8)
    s = np.abs(0.01 * rng.randn(rows, cols // 64)).astype(np.float32)
    return q, s


def dense(q, s):
    """The f32 weight the reference multiplies with: fl(q * s)."""
    return (q.astype(np.float32) * np.repeat(s, 64, axis=1)).astype(np.float32)


def run(x, q, s):
    dev = torch.device("cuda:0")
    w = torch.from_numpy(np.ascontiguousarray(q).view(np.int32)).to(dev)
    y = q35attn.q8_gemm(torch.from_numpy(x).to(dev), w, torch.from_numpy(s).to(dev))
    torch.cuda.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("T,K,N", [(1024, 2048, 6144), (1024, 6144, 2048), (45, 2048, 512), (129, 2048, 4096),
                                   (1, 2048, 256), (300, 64, 768)])
def test_matches_dense_product(T, K, N):
    rng = np.random.RandomState(T + K + N)
    q, s = q8f(rng, K, N)
    x = rng.randn(T, K).astype(np.float32)
    y = run(x, q, s)
    ref = x.astype(np.float64) @ dense(q, s).astype(np.float64)
    err = max_rel_err(y, ref)
    print(f"T={T} K={K} N={N}: max rel err {err:.2e}")
    assert err <= TOL
    assert q35attn.device_status() == 0


def test_rows_match_oracle_row_product():
    """Rows of the product against the oracle's Q8F row product (the CPU
    restatement of the reference's GEMV, every input row)."""
    rng = np.random.RandomState(3)
    T, K, N = 70, 2048, 2048
    q, s = q8f(rng, K, N)
    x = rng.randn(T, K).astype(np.float32)
    y = run(x, q, s)
    for t in (0, 1, 37, 69):
        ref = oracle.q8_gemv(x[t], q, s, exact=True)
        assert max_rel_err(y[t], ref) <= TOL


def test_known_answer_all_ones():
    """q = 1, s = 1, x = 1: every output is exactly K."""
    K, N, T = 2048, 512, 130
    q = np.ones((K, N), np.int8)
    s = np.ones((K, N // 64), np.float32)
    y = run(np.ones((T, K), np.float32), q, s)
    np.testing.assert_array_equal(y, np.full((T, N), float(K), np.float32))


def test_fused_segments_and_swiglu():
    """Several projections of the same rows in one launch (q/k/v, qkv/z) and
    the MLP's up/gate pair with up * silu(gate) written by the epilogue."""
    dev = torch.device("cuda:0")
    rng = np.random.RandomState(21)
    T, K = 200, 2048
    x = rng.randn(T, K).astype(np.float32)
    xd = torch.from_numpy(x).to(dev)
    ws = q35attn.q8_gemm_workspace(T, K)
    mats = [q8f(rng, K, N) for N in (4096, 512, 512)]
    dev_w = [(torch.from_numpy(np.ascontiguousarray(q).view(np.int32)).to(dev), torch.from_numpy(s).to(dev))
             for q, s in mats]
    ys = [torch.empty(T, q.shape[1], device=dev) for q, _ in mats]
    q35attn.q8_gemm_fused(xd, dev_w, ys, workspace=ws)
    torch.cuda.synchronize()
    for (q, s), y in zip(mats, ys):
        assert max_rel_err(y.cpu().numpy(), x.astype(np.float64) @ dense(q, s).astype(np.float64)) <= TOL
    # SwiGLU
    up, gate = q8f(rng, K, 1024), q8f(rng, K, 1024)
    dev_w = [(torch.from_numpy(np.ascontiguousarray(q).view(np.int32)).to(dev), torch.from_numpy(s).to(dev))
             for q, s in (up, gate)]
    act = torch.empty(T, 1024, device=dev)
    q35attn.q8_gemm_fused(xd, dev_w, [act, act], swiglu=True, workspace=ws)
    torch.cuda.synchronize()
    u = x.astype(np.float64) @ dense(*up).astype(np.float64)
    g = x.astype(np.float64) @ dense(*gate).astype(np.float64)
    assert max_rel_err(act.cpu().numpy(), u * (g / (1.0 + np.exp(-g)))) <= TOL
    assert q35attn.device_status() == 0


def test_rejects_unsupported_shapes():
    lib = q35attn.load()
    buf = torch.zeros(1 << 16, device="cuda:0")
    p = buf.data_ptr()
    n = buf.numel() * 4
    assert lib.q35_q8_gemm(4, 48, 256, p, p, p, p, p, n, None) == _lib.ERR_UNSUPPORTED   # in_dim % 32
    assert lib.q35_q8_gemm(4, 64, 320, p, p, p, p, p, n, None) == _lib.ERR_UNSUPPORTED   # out_dim % 256
    assert lib.q35_q8_gemm(4, 64, 256, p + 4, p, p, p, p, n, None) == _lib.ERR_INVALID_ARG  # unaligned x
    assert lib.q35_q8_gemm(4, 64, 256, p, p, p, p, p, 16, None) == _lib.ERR_WORKSPACE  # workspace too small
    assert lib.q35_q8_gemm(0, 64, 256, None, None, None, None, None, 0, None) == _lib.OK
