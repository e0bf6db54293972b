"""End-to-end hybrid decoder stack (config-3 structure: GDN and GQA layers,
RMSNorm + residual, SwiGLU MLP, Q8F projections, tied Q8F lm_head, greedy
argmax) on the q35attn kernels, against the CPU reference of oracle/stack_ref.py
built from the pinned oracle pieces.  A reduced configuration (4 layers, 2-head
GDN, 2/1-head GQA, vocab 4096) keeps the CPU side fast; hidden stays 2048.
Logits: max rel err <= 1e-3 per step; the reference is teacher-forced with the
GPU's tokens, and every GPU token must equal the reference argmax unless the
reference's top-2 gap is below 1e-4 of its max logit.  Decode runs both with
the fused projections (q35_q8_gemv_fused: norm + GEMVs + SwiGLU per launch)
and with one launch per projection."""
import numpy as np
import pytest
import torch

import q35attn.stack as qs
from conftest import max_rel_err
from stack_ref import StackRef

pytestmark = pytest.mark.gpu
SMALL = qs.StackConfig(layer_types=("linear", "linear", "linear", "full"), gdn_hk=2, gdn_hv=2, gqa_hq=2,
                       gqa_hkv=1, inter=512, vocab=4096)


def _check_token(tok, logits):
    top = np.sort(logits)[-2:]
    if top[1] - top[0] > 1e-4 * abs(top[1]):
        assert tok == int(np.argmax(logits))


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("gemv_mode", [1, 0])
def test_small_stack_prefill_and_decode(gemv_mode, fused):
    st = qs.HybridStack(SMALL, capacity=128, seed=3, gemv_mode=gemv_mode, fused=fused)
    ids = torch.from_numpy(np.random.RandomState(4).randint(0, SMALL.vocab, 45).astype(np.int32)).cuda()
    ref = StackRef(st)
    tok = int(st.prefill(ids).item())
    rtok, rlog = ref.prefill(ids.cpu().numpy())
    assert max_rel_err(st.b["logits"].cpu().numpy(), rlog) <= 1e-3
    _check_token(tok, rlog)
    st.capture()
    for step in range(6):
        st.graph.replay()
        torch.cuda.synchronize()
        rtok, rlog = ref.decode(tok)  # teacher-forced with the GPU's token
        e = max_rel_err(st.b["logits"].cpu().numpy(), rlog)
        assert e <= 1e-3, (step, e)
        tok = int(st.b["tok"].item())
        _check_token(tok, rlog)
    assert int(st.gqa_layers[0]["lens"].item()) == 45 + 6


def test_full_2b_stack_against_reference():
    """BASELINE config 3 at its stated shape: 24 layers (18 GDN, 6 GQA), hidden
    2048, 16-head GDN, 8/2-head GQA, intermediate 6144, vocab 248,320, random
    Q8F weights, a 1024-token prompt.  Prefill logits (projections on
    q35_q8_gemm) and 8 graph-replayed decode steps (fused Q8F GEMVs, the
    reference's row coverage), teacher-forced, against the CPU reference stack
    within 1e-3, with the greedy-token rule of the reduced test."""
    T, steps = 1024, 8
    st = qs.HybridStack(qs.QWEN35_2B, capacity=T + steps + 8, seed=11)
    ids = torch.from_numpy(np.random.RandomState(12).randint(0, qs.QWEN35_2B.vocab, T).astype(np.int32)).cuda()
    tok = int(st.prefill(ids).item())
    ref = StackRef(st)
    _, rlog = ref.prefill(ids.cpu().numpy())
    e = max_rel_err(st.b["logits"].cpu().numpy(), rlog)
    print(f"2B prefill logits max rel err {e:.2e}")
    assert e <= 1e-3
    _check_token(tok, rlog)
    st.capture()
    for step in range(steps):
        st.graph.replay()
        torch.cuda.synchronize()
        _, rlog = ref.decode(tok)
        e = max_rel_err(st.b["logits"].cpu().numpy(), rlog)
        print(f"2B decode step {step} logits max rel err {e:.2e}")
        assert e <= 1e-3, (step, e)
        tok = int(st.b["tok"].item())
        _check_token(tok, rlog)
    assert int(st.gqa_layers[0]["lens"].item()) == T + steps


def test_generate_is_deterministic():
    st = qs.HybridStack(SMALL, capacity=96, seed=5)
    ids = torch.arange(30, dtype=torch.int32, device="cuda") * 7
    a = st.generate(ids, 8).cpu()
    st.capture()
    b = st.generate(ids, 8).cpu()
    assert torch.equal(a, b)


def test_stack_from_safetensors_checkpoint(tmp_path):
    """A stack loaded through q35attn.checkpoint (HF names, Linear [out, in],
    Q8F quantisation) runs prefill and graph decode in agreement with the CPU
    reference stack built from the same loaded tensors."""
    from safetensors.torch import save_file

    from q35attn import checkpoint as ck
    cfg = qs.StackConfig(layer_types=("linear", "full"), gdn_hk=2, gdn_hv=2, gqa_hq=2, gqa_hkv=1, inter=512,
                         vocab=1024)
    g = torch.Generator().manual_seed(6)
    r = lambda *s: torch.randn(*s, generator=g) * 0.02
    H, conv = cfg.hidden, cfg.conv_dim
    t = {"model.language_model.embed_tokens.weight": r(cfg.vocab, H), "model.language_model.norm.weight": r(H)}
    for i, kind in enumerate(cfg.layer_types):
        p = f"model.language_model.layers.{i}."
        t.update({p + "input_layernorm.weight": r(H), p + "post_attention_layernorm.weight": r(H),
                  p + "mlp.up_proj.weight": r(cfg.inter, H), p + "mlp.gate_proj.weight": r(cfg.inter, H),
                  p + "mlp.down_proj.weight": r(H, cfg.inter)})
        if kind == "linear":
            a = p + "linear_attn."
            t.update({a + "in_proj_qkv.weight": r(conv, H), a + "in_proj_z.weight": r(cfg.gdn_hv * 128, H),
                      a + "in_proj_b.weight": r(cfg.gdn_hv, H), a + "in_proj_a.weight": r(cfg.gdn_hv, H),
                      a + "A_log": torch.log(torch.rand(cfg.gdn_hv, generator=g) * 15 + 1),
                      a + "dt_bias": torch.ones(cfg.gdn_hv), a + "conv1d.weight": r(conv, 1, 4) * 10,
                      a + "norm.weight": torch.ones(128), a + "out_proj.weight": r(H, cfg.gdn_hv * 128)})
        else:
            a = p + "self_attn."
            t.update({a + "q_proj.weight": r(cfg.gqa_hq * 512, H), a + "k_proj.weight": r(cfg.gqa_hkv * 256, H),
                      a + "v_proj.weight": r(cfg.gqa_hkv * 256, H), a + "o_proj.weight": r(H, cfg.gqa_hq * 256),
                      a + "q_norm.weight": r(256), a + "k_norm.weight": r(256)})
    path = str(tmp_path / "model.safetensors")
    save_file(t, path)
    st = qs.HybridStack(cfg, capacity=64, seed=1)
    ck.load_into(st, ck.read_safetensors(path))
    assert torch.equal(st.layers[0]["w_b"].cpu(), t["model.language_model.layers.0.linear_attn.in_proj_b.weight"].t())
    ref = StackRef(st)
    ids = torch.arange(20, dtype=torch.int32, device="cuda") * 37 % cfg.vocab
    tok = int(st.prefill(ids).item())
    _, rlog = ref.prefill(ids.cpu().numpy())
    assert max_rel_err(st.b["logits"].cpu().numpy(), rlog) <= 1e-3
    st.capture()
    for _ in range(3):
        st.graph.replay()
        torch.cuda.synchronize()
        _, rlog = ref.decode(tok)
        assert max_rel_err(st.b["logits"].cpu().numpy(), rlog) <= 1e-3
        tok = int(st.b["tok"].item())
