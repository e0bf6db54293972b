"""q35_gqa_decode_noalloc: the GQA decode step for callers that cannot
allocate device memory (engines that reserve every byte up front and forbid
cudaMalloc while serving, or FFI hosts with no device allocator).  It must give
the same results as q35_gqa_decode with a caller-provided workspace.

This file is named to be collected last: it reuses the library's fixed scratch
array, and must pass both alone in a fresh process and after the other tests.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle
import q35attn
from q35attn import _lib
from conftest import max_rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-3  # the parity tolerance used by every GPU test


def _call_noalloc(dims, max_len, qg, kn, vn, qw, kw, cos, sin, K, V, lens, out):
    lib = q35attn.load()
    rc = lib.q35_gqa_decode_noalloc(C.byref(dims), int(max_len), qg.data_ptr(), kn.data_ptr(), vn.data_ptr(),
                                    qw.data_ptr(), kw.data_ptr(), cos.data_ptr(), sin.data_ptr(), K.data_ptr(),
                                    V.data_ptr(), lens.data_ptr(), out.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream)
    _lib.check(rc)


def test_noalloc_matches_workspace_entry_point_two_calls():
    B, Hq, Hkv, D, L0, cap = 3, 8, 2, 256, 1500, 1600
    dev = torch.device("cuda:0")
    rng = np.random.RandomState(77)
    K0 = torch.from_numpy(rng.randn(B, Hkv, cap, D).astype(np.float32)).to(dev)
    V0 = torch.from_numpy(rng.randn(B, Hkv, cap, D).astype(np.float32)).to(dev)
    lens0 = torch.tensor([L0, 7, 900], dtype=torch.int32, device=dev)
    qw = torch.from_numpy((0.1 * rng.randn(D)).astype(np.float32)).to(dev)
    kw = torch.from_numpy((0.1 * rng.randn(D)).astype(np.float32)).to(dev)
    Ka, Va, la = K0.clone(), V0.clone(), lens0.clone()   # workspace entry point
    Kb, Vb, lb = K0.clone(), V0.clone(), lens0.clone()   # no-alloc entry point
    ws = q35attn.GqaWorkspace(B, Hq, Hkv, cap, device=dev)
    dims = q35attn.ops.gqa_dims(B, Hq, Hkv, cap)
    for step in range(2):  # two calls in a row: the fixed scratch is reused
        qg = torch.from_numpy(rng.randn(B, Hq, 2 * D).astype(np.float32)).to(dev)
        kn = torch.from_numpy(rng.randn(B, Hkv, D).astype(np.float32)).to(dev)
        vn = torch.from_numpy(rng.randn(B, Hkv, D).astype(np.float32)).to(dev)
        cos_np, sin_np = oracle.rope_tables(la.cpu().numpy().astype(np.int64), rot=64, theta=1e7)
        cos, sin = torch.from_numpy(cos_np).to(dev), torch.from_numpy(sin_np).to(dev)
        out_a = q35attn.gqa_decode(qg, kn, vn, qw, kw, cos, sin, Ka, Va, la, workspace=ws)
        out_b = torch.full_like(out_a, float("nan"))
        _call_noalloc(dims, cap, qg, kn, vn, qw, kw, cos, sin, Kb, Vb, lb, out_b)
        torch.cuda.synchronize()
        assert torch.isfinite(out_b).all()
        assert max_rel_err(out_b.cpu().numpy(), out_a.cpu().numpy()) <= TOL, step
        assert torch.equal(la, lb)
        assert max_rel_err(Kb.cpu().numpy(), Ka.cpu().numpy()) <= TOL
        assert max_rel_err(Vb.cpu().numpy(), Va.cpu().numpy()) <= TOL
    assert la.cpu().tolist() == [L0 + 2, 9, 902]


def test_noalloc_rejects_calls_beyond_its_scratch():
    """256 sequences at 32K context need more than the fixed array holds."""
    dims = q35attn.ops.gqa_dims(256, 8, 2, 40000)
    need = q35attn.load().q35_gqa_decode_workspace_size(C.byref(dims), 32769)
    assert need > (16 << 20)
    lib = q35attn.load()
    rc = lib.q35_gqa_decode_noalloc(C.byref(dims), 32769, *([None] * 11), None)
    assert rc == _lib.ERR_WORKSPACE
    assert "scratch" in lib.q35_last_error().decode()
