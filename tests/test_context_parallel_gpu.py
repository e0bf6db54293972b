"""Context-parallel single-sequence decode, emulated on one GPU: the KV cache
split along its length into N shards (q35_gqa_decode_partial per shard,
q35_gqa_combine_partials over the gathered partials) and the GDN heads split
N ways must reproduce the unsharded oracle.  Tolerance max rel err <= 1e-3."""
import numpy as np
import pytest
import torch

import oracle
import q35attn
from conftest import max_rel_err
from gdn_data import gdn_inputs
from q35attn.parallel import ShardPlan, split_range

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.mark.parametrize("N", [2, 3, 8])
def test_gqa_length_split_matches_oracle(N):
    Hq, Hkv, D, L0, steps = 8, 2, 256, 4096 + 37, 3
    rng = np.random.RandomState(200 + N)
    K = rng.randn(1, Hkv, L0 + steps, D).astype(np.float32)
    V = rng.randn(1, Hkv, L0 + steps, D).astype(np.float32)
    qw = (0.1 * rng.randn(D)).astype(np.float32)
    kw = (0.1 * rng.randn(D)).astype(np.float32)
    dev = torch.device("cuda:0")
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    shards = []
    for r in range(N):
        lo, hi = split_range(L0, N, r)
        cap = (hi - lo) + (steps if r == N - 1 else 0) + 1
        Kr = np.zeros((1, Hkv, cap, D), np.float32)
        Vr = np.zeros((1, Hkv, cap, D), np.float32)
        Kr[:, :, :hi - lo] = K[:, :, lo:hi]
        Vr[:, :, :hi - lo] = V[:, :, lo:hi]
        shards.append(dict(K=T(Kr), V=T(Vr), lens=torch.tensor([hi - lo], dtype=torch.int32, device=dev),
                           ws=q35attn.GqaWorkspace(1, Hq, Hkv, cap, device=dev), cap=cap))
    oK, oV, olens = K.copy(), V.copy(), np.array([L0], np.int32)
    oK[:, :, L0:] = 0
    oV[:, :, L0:] = 0
    for t in range(steps):
        qg = rng.randn(1, Hq, 2 * D).astype(np.float32)
        kn = rng.randn(1, Hkv, D).astype(np.float32)
        vn = rng.randn(1, Hkv, D).astype(np.float32)
        cos, sin = oracle.rope_tables(np.array([L0 + t]), rot=64, theta=1e7)
        parts = torch.empty(N, 1, Hq, D + 2, device=dev)
        for r, sh in enumerate(shards):
            tail = r == N - 1
            q35attn.gqa_decode_partial(T(qg), T(kn) if tail else None, T(vn) if tail else None, T(qw), T(kw),
                                       T(cos), T(sin), sh["K"], sh["V"], sh["lens"], parts[r], workspace=sh["ws"],
                                       max_len=sh["cap"])
        out = q35attn.gqa_combine_partials(parts, T(qg))
        ref, oK, oV, olens = oracle.gqa_decode(qg, kn, vn, qw, kw, cos, sin, oK, oV, olens)
        assert max_rel_err(out.cpu().numpy(), ref) <= TOL, (N, t)
    assert int(shards[-1]["lens"].item()) == split_range(L0, N, N - 1)[1] - split_range(L0, N, N - 1)[0] + steps
    for sh in shards[:-1]:
        assert sh["ws"].status() == 0


@pytest.mark.parametrize("N", [2, 4, 8])
def test_gdn_heads_split_matches_unsharded(N):
    Hk = Hv = 16
    d = gdn_inputs(300 + N, 1, Hk, Hv, 4)
    dev = torch.device("cuda:0")
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    plans = [ShardPlan(N, r, Hk, Hv, 0) for r in range(N)]
    st = []
    for pl in plans:
        qs, ks, vs = pl.channel_slices()
        chans = np.r_[qs, ks, vs]
        v0, v1 = pl.gdn_v_heads
        st.append(dict(ch=chans, conv=T(d["conv0"][:, chans]), S=T(d["S0"][:, v0:v1]), w=T(d["conv_w"][chans]),
                       heads=(v0, v1)))
    ost, oS = d["conv0"].copy(), d["S0"].copy()
    for t in range(4):
        outs = []
        for pl, s in zip(plans, st):
            v0, v1 = s["heads"]
            outs.append(q35attn.gdn_decode(T(d["x"][t][:, s["ch"]]), T(d["z"][t][:, v0 * 128:v1 * 128]),
                                           T(d["beta"][t][:, v0:v1]), T(d["g"][t][:, v0:v1]), s["w"],
                                           T(d["norm_w"]), s["conv"], s["S"], num_k_heads=Hk // N,
                                           num_v_heads=Hv // N))
        full = torch.cat(outs, dim=1).cpu().numpy()
        ref, ost, oS = oracle.gdn_decode(d["x"][t], d["z"][t], d["beta"][t], d["g"][t], d["conv_w"], d["norm_w"],
                                         ost, oS, Hk, Hv)
        assert max_rel_err(full, ref) <= TOL
    S_all = np.concatenate([s["S"].cpu().numpy() for s in st], axis=1)
    assert max_rel_err(S_all, oS) <= TOL
