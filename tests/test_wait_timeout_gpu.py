"""Bounded in-kernel waits that run out.

Every wait of the library's kernels on an mbarrier gives up after a time
limit, sets Q35_STATUS_WAIT_TIMEOUT in a status word the caller can read, and
the kernel returns with every copy and tensor-core operation it started
waited for.  The test hook q35_test_arm_wait_fault makes the next call
withhold one of its copies and wait only 2 ms, so the give-up path runs
without faulting or hanging the GPU; afterwards the context is still usable
and a normal call matches the oracle again.  (The reference panics on such
errors instead, kernels.rs:442,472.)"""
import numpy as np
import pytest
import torch

import oracle
import q35attn
from q35attn import _lib
from conftest import max_rel_err
from gdn_data import gdn_inputs

pytestmark = pytest.mark.gpu
TOL = 1e-3
SITE_PREFILL_STATE, SITE_GQA_DECODE = 1, 2
WAIT_TIMEOUT = 0x4


def _arm(site):
    _lib.check(q35attn.load().q35_test_arm_wait_fault(site))


def _prefill_inputs(T, B=1, H=16, seed=5):
    d = gdn_inputs(seed, B, H, H, T)
    tr = lambda a: np.ascontiguousarray(a.transpose(1, 0, 2))
    return d, tr(d["x"]), tr(d["z"]), tr(d["beta"]), tr(d["g"])


def test_prefill_state_pass_wait_runs_out():
    T, H = 200, 16  # 4 chunks: chunk 1's W copy is withheld
    d, x, z, beta, g = _prefill_inputs(T)
    Tt = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    ws = q35attn.gdn_prefill_workspace(1, T, H, H)
    assert q35attn.ops.workspace_status(ws) == 0
    S = Tt(d["S0"])
    cst = Tt(d["conv0"])
    _arm(SITE_PREFILL_STATE)
    q35attn.gdn_prefill(Tt(x), Tt(z), Tt(beta), Tt(g), Tt(d["conv_w"]), Tt(d["norm_w"]), cst, S, num_k_heads=H,
                        num_v_heads=H, has_prev_conv=True, has_init_state=True, workspace=ws)
    torch.cuda.synchronize()  # the call returned: nothing is left waiting
    assert q35attn.ops.workspace_status(ws, clear=True) & WAIT_TIMEOUT
    assert torch.isnan(S).any(), "the final state of a failed pass is poisoned"
    assert q35attn.ops.workspace_status(ws) == 0  # cleared

    # the hook is consumed; the same call now runs normally and matches the oracle
    S, cst = Tt(d["S0"]), Tt(d["conv0"])
    out = q35attn.gdn_prefill(Tt(x), Tt(z), Tt(beta), Tt(g), Tt(d["conv_w"]), Tt(d["norm_w"]), cst, S,
                              num_k_heads=H, num_v_heads=H, has_prev_conv=True, has_init_state=True, workspace=ws)
    ref, _, rS = oracle.gdn_prefill(x, z, beta, g, d["conv_w"], d["norm_w"], d["conv0"], 1, d["S0"], 1, H, H)
    torch.cuda.synchronize()
    assert q35attn.ops.workspace_status(ws) == 0
    assert max_rel_err(out.cpu().numpy(), ref) <= TOL
    assert max_rel_err(S.cpu().numpy(), rS) <= TOL


def test_gqa_decode_wait_runs_out():
    """Split 0 of (sequence 0, kv head 0) withholds its K/V copies: its
    consumers give up after 2 ms, the split contributes nothing, the status
    word says so, and every counter is left consistent -- the next step is
    exact again."""
    B, Hq, Hkv, D, cap = 2, 8, 2, 256, 700
    rng = np.random.RandomState(9)
    dev = torch.device("cuda:0")
    Tt = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    K = Tt(rng.randn(B, Hkv, cap, D).astype(np.float32))
    V = Tt(rng.randn(B, Hkv, cap, D).astype(np.float32))
    lens = torch.tensor([500, 37], dtype=torch.int32, device=dev)
    w0 = torch.zeros(D, device=dev)
    ws = q35attn.GqaWorkspace(B, Hq, Hkv, cap, device=dev)

    def inputs():
        qg = rng.randn(B, Hq, 2 * D).astype(np.float32)
        kn = rng.randn(B, Hkv, D).astype(np.float32)
        vn = rng.randn(B, Hkv, D).astype(np.float32)
        cos, sin = oracle.rope_tables(lens.cpu().numpy().astype(np.int64), rot=64, theta=1e7)
        return qg, kn, vn, cos, sin

    qg, kn, vn, cos, sin = inputs()
    _arm(SITE_GQA_DECODE)
    q35attn.gqa_decode(Tt(qg), Tt(kn), Tt(vn), w0, w0, Tt(cos), Tt(sin), K, V, lens, workspace=ws)
    torch.cuda.synchronize()  # the call returned: nothing is left waiting
    assert ws.status(clear=True) & WAIT_TIMEOUT
    assert lens.cpu().tolist() == [501, 38]

    # the next step runs normally and matches the oracle on the state the GPU holds
    qg, kn, vn, cos, sin = inputs()
    Kh, Vh, lh = K.cpu().numpy(), V.cpu().numpy(), lens.cpu().numpy()
    out = q35attn.gqa_decode(Tt(qg), Tt(kn), Tt(vn), w0, w0, Tt(cos), Tt(sin), K, V, lens, workspace=ws)
    ref, _, _, lr = oracle.gqa_decode(qg, kn, vn, np.zeros(D, np.float32), np.zeros(D, np.float32), cos, sin, Kh,
                                      Vh, lh)
    torch.cuda.synchronize()
    assert ws.status() == 0
    assert max_rel_err(out.cpu().numpy(), ref) <= TOL
    assert lens.cpu().tolist() == lr.tolist()


def test_arm_rejects_unknown_site():
    assert q35attn.load().q35_test_arm_wait_fault(7) == _lib.ERR_INVALID_ARG
    _arm(0)
