"""q35_gqa_decode_noalloc: the GQA decode step for callers that cannot
allocate device memory (engines that reserve every byte up front and forbid
cudaMalloc while serving, or FFI hosts with no device allocator).  It must give
the same results as q35_gqa_decode with a caller-provided workspace, and the
same results as the CPU oracle.

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


class _Case:
    """One batch of caches, stepped through both entry points side by side.
    Only the first `fill` rows of each cache hold data (every lens[b] stays
    below it), so the oracle works on that prefix alone."""

    def __init__(self, rng, dev, B, Hq, Hkv, cap, lens, fill):
        D = 256
        self.B, self.Hq, self.Hkv, self.cap, self.D, self.fill = B, Hq, Hkv, cap, D, fill
        self.dev = dev
        self.Ka = torch.empty(B, Hkv, cap, D, device=dev)
        self.Va = torch.empty(B, Hkv, cap, D, device=dev)
        self.Ka[:, :, :fill] = torch.from_numpy(rng.randn(B, Hkv, fill, D).astype(np.float32)).to(dev)
        self.Va[:, :, :fill] = torch.from_numpy(rng.randn(B, Hkv, fill, D).astype(np.float32)).to(dev)
        self.Kb, self.Vb = self.Ka.clone(), self.Va.clone()
        self.la = torch.tensor(lens, dtype=torch.int32, device=dev)
        self.lb = self.la.clone()
        self.qw = torch.from_numpy((0.1 * rng.randn(D)).astype(np.float32)).to(dev)
        self.kw = torch.from_numpy((0.1 * rng.randn(D)).astype(np.float32)).to(dev)
        self.ws = q35attn.GqaWorkspace(B, Hq, Hkv, cap, max_len=cap, device=dev)
        self.dims = q35attn.ops.gqa_dims(B, Hq, Hkv, cap)

    def step(self, rng):
        B, Hq, Hkv, D, dev = self.B, self.Hq, self.Hkv, self.D, self.dev
        qg_np = rng.randn(B, Hq, 2 * D).astype(np.float32)
        kn_np = rng.randn(B, Hkv, D).astype(np.float32)
        vn_np = rng.randn(B, Hkv, D).astype(np.float32)
        l_np = self.la.cpu().numpy()
        cos_np, sin_np = oracle.rope_tables(l_np.astype(np.int64), rot=64, theta=1e7)
        qg, kn, vn = (torch.from_numpy(a).to(dev) for a in (qg_np, kn_np, vn_np))
        cos, sin = torch.from_numpy(cos_np).to(dev), torch.from_numpy(sin_np).to(dev)
        # the oracle on the filled prefix of the caches, before either call
        Kp = self.Ka[:, :, :self.fill].cpu().numpy()
        Vp = self.Va[:, :, :self.fill].cpu().numpy()
        ref, Kr, Vr, lr = oracle.gqa_decode(qg_np, kn_np, vn_np, self.qw.cpu().numpy(), self.kw.cpu().numpy(),
                                            cos_np, sin_np, Kp, Vp, l_np)
        out_a = q35attn.gqa_decode(qg, kn, vn, self.qw, self.kw, cos, sin, self.Ka, self.Va, self.la,
                                   workspace=self.ws, max_len=self.cap)
        out_b = torch.full_like(out_a, float("nan"))
        _call_noalloc(self.dims, self.cap, qg, kn, vn, self.qw, self.kw, cos, sin, self.Kb, self.Vb, self.lb,
                      out_b)
        torch.cuda.synchronize()
        assert self.ws.status() == 0
        ob = out_b.cpu().numpy()
        assert np.isfinite(ob).all()
        assert max_rel_err(ob, out_a.cpu().numpy()) <= TOL
        assert max_rel_err(ob, ref) <= TOL
        assert torch.equal(self.la, self.lb)
        assert self.lb.cpu().numpy().tolist() == lr.tolist()
        for b in range(B):  # the appended row, against both references
            p = int(l_np[b])
            kb = self.Kb[b, :, p].cpu().numpy()
            vb = self.Vb[b, :, p].cpu().numpy()
            assert max_rel_err(kb, self.Ka[b, :, p].cpu().numpy()) <= TOL
            assert max_rel_err(kb, Kr[b, :, p]) <= TOL
            assert max_rel_err(vb, Vr[b, :, p]) <= TOL


def test_noalloc_matches_workspace_entry_point_and_oracle():
    """Two calls in a row on a few-sequence batch (split partials merged by
    the combine kernel); then a batch whose grid takes the many-sequence
    ticket-tree merge, whose counter region has a different layout; then the
    small batch again.  Every call is compared with q35_gqa_decode and with
    the CPU oracle."""
    dev = torch.device("cuda:0")
    rng = np.random.RandomState(77)
    small = _Case(rng, dev, B=3, Hq=8, Hkv=2, cap=1600, lens=[1500, 7, 900], fill=1504)
    for _ in range(2):
        small.step(rng)
    assert small.lb.cpu().tolist() == [1502, 9, 902]

    # many-sequence schedule: (B * Hkv) * ceil(cap / 2048) >= 16 * SMs splits.
    # The grid is sized by the capacity hint, so the caches stay mostly empty.
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    Hkv, cap = 8, 40000
    B = max(16, -(-16 * sms // (Hkv * (-(-cap // 2048)))))
    dims = q35attn.ops.gqa_dims(B, 8, Hkv, cap)
    assert q35attn.load().q35_gqa_decode_workspace_size(C.byref(dims), cap) <= (16 << 20)
    lens = rng.randint(0, 600, size=B).tolist()
    lens[0] = 0  # an empty cache
    big = _Case(rng, dev, B=B, Hq=8, Hkv=Hkv, cap=cap, lens=lens, fill=640)
    big.step(rng)
    del big
    torch.cuda.empty_cache()

    small.step(rng)
    assert small.lb.cpu().tolist() == [1503, 10, 903]


def test_noalloc_rejects_calls_beyond_its_scratch():
    """256 sequences at 32K context need more than the fixed array holds; the
    call is refused before anything is queued on the stream."""
    dims = q35attn.ops.gqa_dims(256, 8, 2, 40000)
    lib = q35attn.load()
    need = lib.q35_gqa_decode_workspace_size(C.byref(dims), 32769)
    assert need > (16 << 20)
    dummy = torch.zeros(64, device="cuda:0")  # never read: the call is refused on the host
    p = dummy.data_ptr()
    rc = lib.q35_gqa_decode_noalloc(C.byref(dims), 32769, *([p] * 11), None)
    assert rc == _lib.ERR_WORKSPACE
    assert "scratch" in lib.q35_last_error().decode()
    rc = lib.q35_gqa_decode_noalloc(C.byref(dims), 32769, *([None] * 11), None)
    assert rc == _lib.ERR_INVALID_ARG
