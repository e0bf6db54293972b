"""Parity of q35_gqa_decode (fused q/k norm + RoPE + cache append + split-K
flash-decode + sigmoid gate) against the CPU oracle, through the C ABI.
Tolerance: max rel err <= 1e-3 per tensor (outputs every step, cache, lens)."""
import numpy as np
import pytest
import torch

import oracle
import q35attn
from conftest import max_rel_err
from gdn_data import gqa_inputs

pytestmark = pytest.mark.gpu
TOL = 1e-3


def rope(pos, rot=64):
    return oracle.rope_tables(np.asarray(pos, np.int64), rot=rot, theta=1e7)


def run_gqa(B, Hq, Hkv, steps, lens0, cap, seed, wscale=0.0, rot=64, max_len=None, check_every=1):
    lens0 = np.asarray(lens0, np.int32)
    d = gqa_inputs(seed, B, Hq, Hkv, steps, int(lens0.max()), cap, wscale=wscale)
    for b in range(B):  # ragged: zero the tail beyond each sequence's length
        d["K"][b, :, lens0[b]:] = 0
        d["V"][b, :, lens0[b]:] = 0
    dev = torch.device("cuda:0")
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    Kc, Vc, lens = T(d["K"]), T(d["V"]), T(lens0)
    ws = q35attn.GqaWorkspace(B, Hq, Hkv, cap, max_len=max_len or cap)
    oK, oV, olens = d["K"].copy(), d["V"].copy(), lens0.copy()
    worst = 0.0
    for t in range(steps):
        cos, sin = rope(olens, rot)
        out = q35attn.gqa_decode(T(d["qg"][t]), T(d["kn"][t]), T(d["vn"][t]), T(d["qn_w"]), T(d["kn_w"]), T(cos),
                                 T(sin), Kc, Vc, lens, workspace=ws, rotary_dim=rot)
        ref, oK, oV, olens = oracle.gqa_decode(d["qg"][t], d["kn"][t], d["vn"][t], d["qn_w"], d["kn_w"], cos, sin,
                                               oK, oV, olens, rot=rot)
        if t % check_every == 0 or t == steps - 1:
            worst = max(worst, max_rel_err(out.cpu().numpy(), ref))
    torch.cuda.synchronize()
    assert ws.status() == 0
    np.testing.assert_array_equal(lens.cpu().numpy(), olens)
    return worst, max_rel_err(Kc.cpu().numpy(), oK), max_rel_err(Vc.cpu().numpy(), oV)


def test_config1_4096_context_128_steps():
    """8 q heads, 2 kv heads, d=256, RoPE on 64 dims
    (theta 1e7), 4096 cached tokens, 128 decode steps."""
    e_out, e_k, e_v = run_gqa(1, 8, 2, 128, [4096], 4096 + 128, seed=1, check_every=1)
    print(f"config1: out {e_out:.2e} K {e_k:.2e} V {e_v:.2e}")
    assert e_out <= TOL and e_k <= TOL and e_v == 0.0


def test_config1_with_norm_weights():
    e_out, e_k, e_v = run_gqa(1, 8, 2, 16, [4096], 4200, seed=2, wscale=0.1)
    assert e_out <= TOL and e_k <= TOL and e_v == 0.0


@pytest.mark.parametrize("Hq,Hkv", [(8, 2), (4, 4), (16, 2), (4, 2)])
def test_ragged_batch_and_group_sizes(Hq, Hkv):
    """Ragged lengths, including an empty cache (L=0 -> output is the gated
    new value) and lengths that straddle split boundaries."""
    lens0 = [0, 1, 17, 300, 2049]
    e_out, e_k, e_v = run_gqa(5, Hq, Hkv, 3, lens0, 2100, seed=3 + Hq)
    assert e_out <= TOL and e_k <= TOL and e_v == 0.0


def test_partial_rotary_dims():
    for rot in (0, 32, 256):
        e_out, e_k, e_v = run_gqa(2, 8, 2, 2, [40, 7], 64, seed=40 + rot, rot=rot)
        assert e_out <= TOL and e_k <= TOL and e_v == 0.0


def test_tight_max_len_hint():
    e_out, e_k, e_v = run_gqa(2, 8, 2, 4, [100, 90], 4096, seed=5, max_len=104)
    assert e_out <= TOL and e_k <= TOL and e_v == 0.0


def test_empty_cache_returns_gated_value():
    """L = 0: softmax over the single new key is 1, so out = v * sigmoid(gate)."""
    B, Hq, Hkv, D, cap = 1, 8, 2, 256, 8
    rng = np.random.RandomState(9)
    dev = torch.device("cuda:0")
    qg = torch.from_numpy(rng.randn(B, Hq, 2 * D).astype(np.float32)).to(dev)
    kn = torch.from_numpy(rng.randn(B, Hkv, D).astype(np.float32)).to(dev)
    vn = torch.from_numpy(rng.randn(B, Hkv, D).astype(np.float32)).to(dev)
    w = torch.zeros(D, device=dev)
    cos, sin = rope([0])
    Kc = torch.zeros(B, Hkv, cap, D, device=dev)
    Vc = torch.zeros(B, Hkv, cap, D, device=dev)
    lens = torch.zeros(B, dtype=torch.int32, device=dev)
    ws = q35attn.GqaWorkspace(B, Hq, Hkv, cap)
    out = q35attn.gqa_decode(qg, kn, vn, w, w, torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev), Kc, Vc,
                             lens, workspace=ws)
    exp = (vn.repeat_interleave(Hq // Hkv, dim=1) * torch.sigmoid(qg[:, :, D:])).reshape(B, Hq * D)
    assert max_rel_err(out.cpu().numpy(), exp.cpu().numpy()) <= 1e-6
    assert int(lens.item()) == 1


@pytest.mark.parametrize("cap", [16, 200])  # one split per pair (in-kernel output) / four splits (split combine)
def test_full_cache_sets_status_and_skips(cap):
    """A sequence whose cache is full is skipped on the device (status bit,
    lens, cache and output untouched) while the others proceed."""
    B, Hq, Hkv, D = 2, 8, 2, 256
    dev = torch.device("cuda:0")
    rng = np.random.RandomState(11)
    qg = torch.from_numpy(rng.randn(B, Hq, 2 * D).astype(np.float32)).to(dev)
    kn = torch.from_numpy(rng.randn(B, Hkv, D).astype(np.float32)).to(dev)
    vn = torch.from_numpy(rng.randn(B, Hkv, D).astype(np.float32)).to(dev)
    w = torch.zeros(D, device=dev)
    cos, sin = rope([16, 5])
    Kc = torch.randn(B, Hkv, cap, D, device=dev)
    Vc = torch.randn(B, Hkv, cap, D, device=dev)
    K0 = Kc.clone()
    lens = torch.tensor([cap, 5], dtype=torch.int32, device=dev)
    out = torch.full((B, Hq * D), 7.0, device=dev)
    ws = q35attn.GqaWorkspace(B, Hq, Hkv, cap)
    q35attn.gqa_decode(qg, kn, vn, w, w, torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev), Kc, Vc, lens,
                       out, workspace=ws)
    assert ws.status(clear=True) & q35attn.STATUS_CACHE_FULL
    assert ws.status() == 0
    assert lens.cpu().tolist() == [cap, 6]
    assert torch.all(out[0] == 7.0) and not torch.all(out[1] == 7.0)
    assert torch.equal(Kc[0], K0[0])


def test_length_hint_refuses_the_step():
    """lens + 1 beyond the max_len the workspace was planned for: the step is
    refused on the device (status bit), lens and the output stay as they were,
    for both merge schedules."""
    B, Hq, Hkv, D = 1, 8, 2, 256
    dev = torch.device("cuda:0")
    for l0, max_len in ((70, 64), (200, 130)):
        cap = 256
        rng = np.random.RandomState(l0)
        qg = torch.from_numpy(rng.randn(B, Hq, 2 * D).astype(np.float32)).to(dev)
        kn = torch.from_numpy(rng.randn(B, Hkv, D).astype(np.float32)).to(dev)
        vn = torch.from_numpy(rng.randn(B, Hkv, D).astype(np.float32)).to(dev)
        w = torch.zeros(D, device=dev)
        cos, sin = rope([l0])
        Kc, Vc = torch.randn(B, Hkv, cap, D, device=dev), torch.randn(B, Hkv, cap, D, device=dev)
        lens = torch.tensor([l0], dtype=torch.int32, device=dev)
        out = torch.full((B, Hq * D), 7.0, device=dev)
        ws = q35attn.GqaWorkspace(B, Hq, Hkv, cap, max_len=max_len)
        q35attn.gqa_decode(qg, kn, vn, w, w, torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev), Kc, Vc,
                           lens, out, workspace=ws, max_len=max_len)
        assert ws.status() & q35attn.STATUS_LEN_HINT
        assert int(lens.item()) == l0 and torch.all(out == 7.0)


def test_split_combine_schedule_matches_oracle_at_32k():
    """One sequence at 32K context: the few-sequence schedule (short splits,
    separate combine kernel) against the oracle, three steps."""
    e_out, e_k, e_v = run_gqa(1, 8, 2, 3, [32768], 32768 + 4, seed=12, check_every=1)
    assert e_out <= TOL and e_k <= TOL and e_v == 0.0


def test_config4_shapes_long_splits():
    """Config-4 GQA shapes at full context (32K cached tokens) with a batch
    large enough to take the long-split (2048 keys per CTA) schedule; a sample
    of sequences is checked against the oracle on every step."""
    B, L0, steps, Hq, Hkv, D = 96, 32768, 2, 8, 2, 256
    cap = L0 + steps + 1
    dev = torch.device("cuda:0")
    gen = torch.Generator(device=dev)
    gen.manual_seed(4)
    Kc = torch.empty(B, Hkv, cap, D, device=dev)
    Vc = torch.empty(B, Hkv, cap, D, device=dev)
    Kc.normal_(generator=gen)
    Vc.normal_(generator=gen)
    sample = [0, 47, 95]
    oK = Kc[sample].cpu().numpy()
    oV = Vc[sample].cpu().numpy()
    lens = torch.full((B,), L0, dtype=torch.int32, device=dev)
    olens = np.full(len(sample), L0, np.int32)
    w = torch.zeros(D, device=dev)
    ws = q35attn.GqaWorkspace(B, Hq, Hkv, cap)
    rng = np.random.RandomState(8)
    for t in range(steps):
        qg = rng.randn(B, Hq, 2 * D).astype(np.float32)
        kn = rng.randn(B, Hkv, D).astype(np.float32)
        vn = rng.randn(B, Hkv, D).astype(np.float32)
        cos, sin = rope(np.full(B, L0 + t))
        T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        out = q35attn.gqa_decode(T(qg), T(kn), T(vn), w, w, T(cos), T(sin), Kc, Vc, lens, workspace=ws).cpu().numpy()
        ref, oK, oV, olens = oracle.gqa_decode(qg[sample], kn[sample], vn[sample], np.zeros(D, np.float32),
                                               np.zeros(D, np.float32), cos[sample], sin[sample], oK, oV, olens)
        assert max_rel_err(out[sample], ref) <= TOL
    assert ws.status() == 0
    assert (lens.cpu().numpy() == L0 + steps).all()
    assert max_rel_err(Kc[sample][:, :, L0:L0 + steps].cpu().numpy(), oK[:, :, L0:L0 + steps]) <= TOL


def test_known_answer_equal_scores():
    """Hand-computed answer at the kernel's head size (d=256): q = ones (its
    RMSNorm leaves it), cached key 16 e0 and new key 16 e1 (RMSNorm: mean square
    1), identity RoPE tables; both scores are 16/sqrt(256) = 1, so the output is
    the mean of the two values -- v0[i] = i and v_new[i] = 256 - i, mean 128 --
    times sigmoid(0) = 1/2: 64 everywhere."""
    D, dev = 256, torch.device("cuda:0")
    qg = torch.zeros(1, 1, 2 * D, device=dev)
    qg[0, 0, :D] = 1.0
    kn = torch.zeros(1, 1, D, device=dev)
    kn[0, 0, 1] = 16.0
    vn = (256.0 - torch.arange(D, device=dev, dtype=torch.float32)).view(1, 1, D)
    Kc, Vc = torch.zeros(1, 1, 4, D, device=dev), torch.zeros(1, 1, 4, D, device=dev)
    Kc[0, 0, 0, 0] = 16.0
    Vc[0, 0, 0] = torch.arange(D, device=dev, dtype=torch.float32)
    lens = torch.ones(1, dtype=torch.int32, device=dev)
    w = torch.zeros(D, device=dev)
    cos, sin = torch.ones(1, 64, device=dev), torch.zeros(1, 64, device=dev)
    ws = q35attn.GqaWorkspace(1, 1, 1, 4)
    out = q35attn.gqa_decode(qg, kn, vn, w, w, cos, sin, Kc, Vc, lens, workspace=ws)
    assert torch.allclose(out, torch.full_like(out, 64.0), atol=1e-3)
    assert int(lens.item()) == 2 and float(Kc[0, 0, 1, 1]) == pytest.approx(16.0, rel=1e-5)


def _ragged_many(B, Hq, Hkv, cap, lens0, sample, steps, seed, arm_first=False):
    """Many sequences of ragged length on the many-sequence schedule (long
    splits, in-kernel merge tree); the sampled sequences are followed by the
    oracle, every sequence's lens is checked."""
    D = 256
    dev = torch.device("cuda:0")
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    Kc = torch.empty(B, Hkv, cap, D, device=dev)
    Vc = torch.empty(B, Hkv, cap, D, device=dev)
    Kc.normal_(generator=gen)
    Vc.normal_(generator=gen)
    lens = torch.from_numpy(lens0.astype(np.int32)).to(dev)
    oK, oV = Kc[sample].cpu().numpy(), Vc[sample].cpu().numpy()
    olens = lens0[sample].astype(np.int32)
    for i, b in enumerate(sample):  # the oracle sees only each sequence's own keys
        oK[i, :, olens[i]:] = 0
        oV[i, :, olens[i]:] = 0
    w = (0.1 * np.random.RandomState(seed).randn(D)).astype(np.float32)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    ws = q35attn.GqaWorkspace(B, Hq, Hkv, cap)
    rng = np.random.RandomState(seed + 1)
    errs = []
    for t in range(steps):
        qg = rng.randn(B, Hq, 2 * D).astype(np.float32)
        kn = rng.randn(B, Hkv, D).astype(np.float32)
        vn = rng.randn(B, Hkv, D).astype(np.float32)
        cos, sin = rope(lens0 + t)
        if arm_first and t == 0:
            from q35attn import _lib
            _lib.check(q35attn.load().q35_test_arm_wait_fault(2))
        out = q35attn.gqa_decode(T(qg), T(kn), T(vn), T(w), T(w), T(cos), T(sin), Kc, Vc, lens,
                                 workspace=ws).cpu().numpy()
        ref, oK, oV, olens = oracle.gqa_decode(qg[sample], kn[sample], vn[sample], w, w, cos[sample], sin[sample],
                                               oK, oV, olens)
        if arm_first and t == 0:
            assert ws.status(clear=True) & q35attn.STATUS_WAIT_TIMEOUT
        else:
            errs.append(max_rel_err(out[sample], ref))
    assert ws.status() == 0
    np.testing.assert_array_equal(lens.cpu().numpy(), lens0 + steps)
    return max(errs)


def test_many_ragged_sequences_long_splits():
    """256 sequences of ragged length (1 to 9,200 cached keys, some only a
    few keys long, some at split boundaries) at a length hint that selects the
    many-sequence schedule: splits without keys, splits ending inside a tile,
    pairs merged from one to five splits."""
    B, Hq, Hkv, cap = 256, 8, 2, 9300
    rng = np.random.RandomState(31)
    lens0 = rng.randint(1, 9200, size=B)
    lens0[:8] = [1, 2, 15, 16, 17, 9199, 2048, 2049]
    sample = np.array([0, 1, 2, 3, 4, 5, 6, 7, 100, 255])
    err = _ragged_many(B, Hq, Hkv, cap, lens0, sample, 3, seed=32)
    assert err <= TOL


def test_long_splits_wait_runs_out_then_recovers():
    """On the many-sequence schedule the first split withholds its copies
    (test hook): the step reports Q35_STATUS_WAIT_TIMEOUT, every sequence
    still advances (its new key is in the cache), the merge tree's counters
    stay consistent, and the next step matches the oracle."""
    B, Hq, Hkv, cap = 256, 8, 2, 9300
    rng = np.random.RandomState(41)
    lens0 = rng.randint(1, 9200, size=B)
    sample = np.array([0, 1, 128, 255])
    err = _ragged_many(B, Hq, Hkv, cap, lens0, sample, 2, seed=42, arm_first=True)
    assert err <= TOL
