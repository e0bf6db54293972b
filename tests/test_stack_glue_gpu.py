"""Decoder-stack glue kernels against numpy: q35_add_rmsnorm
(text_modules.rs:800-809 with the residual add of :1053-1085) on one and
several rows, in place (sum_out == residual, out == x) and above the
register-cached width, and q35_silu_mul (:999-1011).  f32 tolerance 1e-5."""
import numpy as np
import pytest
import torch

from q35attn import ops
from conftest import max_rel_err

pytestmark = pytest.mark.gpu


def ref_norm(h, w, eps):
    inv = 1.0 / np.sqrt((h.astype(np.float64) ** 2).mean(-1, keepdims=True) + eps)
    return h * inv * (1.0 + w)


@pytest.mark.parametrize("rows,dim", [(1, 2048), (3, 2048), (1, 4096), (2, 1000), (1, 5000), (4, 64)])
@pytest.mark.parametrize("inplace", [False, True])
def test_add_rmsnorm(rows, dim, inplace):
    rng = np.random.RandomState(rows * 31 + dim + inplace)
    x = rng.randn(rows, dim).astype(np.float32)
    r = rng.randn(rows, dim).astype(np.float32)
    w = (0.1 * rng.randn(dim)).astype(np.float32)
    xd, rd, wd = (torch.from_numpy(a).cuda() for a in (x, r, w))
    if inplace:  # h += x in the residual buffer, the normalised row over x
        ops.add_rmsnorm(xd, wd, xd, residual=rd, sum_out=rd)
        out, h = xd, rd
    else:
        out, h = torch.empty_like(xd), torch.empty_like(xd)
        ops.add_rmsnorm(xd, wd, out, residual=rd, sum_out=h)
    assert torch.equal(h.cpu(), torch.from_numpy(x + r))
    assert max_rel_err(out.cpu().numpy(), ref_norm(x + r, w, 1e-6)) <= 1e-5


def test_add_rmsnorm_without_residual():
    rng = np.random.RandomState(1)
    x = rng.randn(2048).astype(np.float32)
    w = (0.1 * rng.randn(2048)).astype(np.float32)
    out = ops.add_rmsnorm(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), torch.empty(2048, device="cuda"))
    assert max_rel_err(out.cpu().numpy(), ref_norm(x, w, 1e-6)) <= 1e-5


def test_silu_mul():
    rng = np.random.RandomState(2)
    g, u = rng.randn(2, 6144).astype(np.float32) * 4
    out = ops.silu_mul(torch.from_numpy(g).cuda(), torch.from_numpy(u).cuda(), torch.empty(6144, device="cuda"))
    assert max_rel_err(out.cpu().numpy(), u * g / (1 + np.exp(-g))) <= 1e-5
