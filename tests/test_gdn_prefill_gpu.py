"""Parity of q35_gdn_prefill (conv + chunked WY delta rule + gated norm)
against the oracle's chunked restatement AND its token-by-token recurrence
(the reference's implied identity).  Tolerance max rel err <= 1e-3."""
import numpy as np
import pytest
import torch

import oracle
import q35attn
from conftest import max_rel_err
from gdn_data import gdn_inputs

pytestmark = pytest.mark.gpu
TOL = 1e-3


def prefill_case(B, T, Hk, Hv, seed, has_prev, has_init, K=4):
    d = gdn_inputs(seed, B, Hk, Hv, T, K)
    x = np.ascontiguousarray(d["x"].transpose(1, 0, 2))
    z = np.ascontiguousarray(d["z"].transpose(1, 0, 2))
    beta = np.ascontiguousarray(d["beta"].transpose(1, 0, 2))
    g = np.ascontiguousarray(d["g"].transpose(1, 0, 2))
    Tt = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    cst, S = Tt(d["conv0"]), Tt(d["S0"])
    out = q35attn.gdn_prefill(Tt(x), Tt(z), Tt(beta), Tt(g), Tt(d["conv_w"]), Tt(d["norm_w"]), cst, S,
                              num_k_heads=Hk, num_v_heads=Hv, has_prev_conv=has_prev, has_init_state=has_init)
    ref, rst, rS = oracle.gdn_prefill(x, z, beta, g, d["conv_w"], d["norm_w"], d["conv0"], has_prev, d["S0"],
                                      has_init, Hk, Hv)
    torch.cuda.synchronize()
    return d, (x, z, beta, g), out.cpu().numpy(), cst.cpu().numpy(), S.cpu().numpy(), ref, rst, rS


@pytest.mark.parametrize("T", [1, 3, 63, 64, 65, 130])
@pytest.mark.parametrize("has_prev,has_init", [(0, 0), (1, 1)])
def test_ragged_lengths(T, has_prev, has_init):
    _, _, out, cst, S, ref, rst, rS = prefill_case(2, T, 16, 16, 100 + T, has_prev, has_init)
    assert max_rel_err(out, ref) <= TOL
    assert max_rel_err(S, rS) <= TOL
    np.testing.assert_allclose(cst, rst, rtol=0, atol=0)


def test_value_heads_share_key_heads():
    _, _, out, cst, S, ref, rst, rS = prefill_case(1, 150, 8, 16, 7, 1, 1)
    assert max_rel_err(out, ref) <= TOL and max_rel_err(S, rS) <= TOL
    np.testing.assert_array_equal(cst, rst)


def test_config2_8192_tokens_vs_recurrence():
    """prompt 8192, chunk 64, 16/16 heads; outputs and final
    state against the token-by-token recurrence (and the chunked oracle)."""
    oracle.set_threads(max(1, min(32, __import__("os").cpu_count() or 1)))
    d, (x, z, beta, g), out, cst, S, ref, rst, rS = prefill_case(1, 8192, 16, 16, 2, 0, 1)
    e_chunk_out, e_chunk_S = max_rel_err(out, ref), max_rel_err(S, rS)
    # token-by-token: conv (prefill form) + recurrent rule + gated norm
    y, _ = oracle.conv1d_prefill(x, np.zeros_like(d["conv0"]), d["conv_w"], 0)
    q, k, v = y[..., :2048].reshape(1, 8192, 16, 128), y[..., 2048:4096].reshape(1, 8192, 16, 128), \
        y[..., 4096:].reshape(1, 8192, 16, 128)
    core, Sr = oracle.recurrent_gdr(q, k, v, g, beta, d["S0"])
    rec = oracle.rmsnorm_gated(core.reshape(-1, 128), z.reshape(-1, 128), d["norm_w"]).reshape(out.shape)
    e_rec_out, e_rec_S = max_rel_err(out, rec), max_rel_err(S, Sr)
    print(f"config2: vs chunk out {e_chunk_out:.2e} S {e_chunk_S:.2e}; vs recurrence out {e_rec_out:.2e} "
          f"S {e_rec_S:.2e}")
    assert max(e_chunk_out, e_chunk_S, e_rec_out, e_rec_S) <= TOL


def test_prefill_then_decode_matches_oracle():
    """Module flow of GatedDeltaNet::forward: first call (no cache) takes the
    chunked path and fills the conv / recurrent state; later seq_len == 1
    calls take the decode path (text_modules.rs:511-515, 627-647)."""
    B, Hk, Hv, T, steps = 2, 16, 16, 77, 5
    d = gdn_inputs(55, B, Hk, Hv, T + steps)
    Tt = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    xs = np.ascontiguousarray(d["x"].transpose(1, 0, 2))
    zs = np.ascontiguousarray(d["z"].transpose(1, 0, 2))
    bs = np.ascontiguousarray(d["beta"].transpose(1, 0, 2))
    gs = np.ascontiguousarray(d["g"].transpose(1, 0, 2))
    cst = torch.zeros(B, 6144, 3, device="cuda")
    S = torch.zeros(B, Hv, 128, 128, device="cuda")
    q35attn.gdn_prefill(Tt(xs[:, :T]), Tt(zs[:, :T]), Tt(bs[:, :T]), Tt(gs[:, :T]), Tt(d["conv_w"]),
                        Tt(d["norm_w"]), cst, S, num_k_heads=Hk, num_v_heads=Hv)
    _, ost, oS = oracle.gdn_prefill(xs[:, :T], zs[:, :T], bs[:, :T], gs[:, :T], d["conv_w"], d["norm_w"],
                                    np.zeros((B, 6144, 3), np.float32), 0, np.zeros((B, Hv, 128, 128), np.float32),
                                    0, Hk, Hv)
    for t in range(T, T + steps):
        out = q35attn.gdn_decode(Tt(xs[:, t]), Tt(zs[:, t]), Tt(bs[:, t]), Tt(gs[:, t]), Tt(d["conv_w"]),
                                 Tt(d["norm_w"]), cst, S, num_k_heads=Hk, num_v_heads=Hv)
        ref, ost, oS = oracle.gdn_decode(xs[:, t], zs[:, t], bs[:, t], gs[:, t], d["conv_w"], d["norm_w"], ost, oS,
                                         Hk, Hv)
        assert max_rel_err(out.cpu().numpy(), ref) <= TOL
    assert max_rel_err(S.cpu().numpy(), oS) <= TOL
