"""Checkpoint import (q35attn.checkpoint, after main.rs:160-222): key mapping of
a Hugging Face safetensors file, the Linear transposition to [in, out], the
conv1d squeeze, the A_log rename, and the Q8F quantiser's bound |w - q*scale| <=
scale/2 with one scale per 64-value block.  CPU only."""
import numpy as np
import pytest
import torch

from q35attn import checkpoint as ck


def hf_tensors(hidden=128, inter=256, vocab=256, hk=1, hv=1, hq=2, hkv=1, seed=0):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g) * 0.05
    conv = 2 * hk * 128 + hv * 128
    t = {"model.language_model.embed_tokens.weight": r(vocab, hidden),
         "model.language_model.norm.weight": r(hidden),
         "model.visual.blocks.0.attn.qkv.weight": r(8, 8)}  # not the text model: ignored
    for i, kind in enumerate(("linear", "full")):
        p = f"model.language_model.layers.{i}."
        t[p + "input_layernorm.weight"] = r(hidden)
        t[p + "post_attention_layernorm.weight"] = r(hidden)
        t[p + "mlp.up_proj.weight"] = r(inter, hidden)
        t[p + "mlp.gate_proj.weight"] = r(inter, hidden)
        t[p + "mlp.down_proj.weight"] = r(hidden, inter)
        if kind == "linear":
            a = p + "linear_attn."
            t[a + "in_proj_qkv.weight"] = r(conv, hidden)
            t[a + "in_proj_z.weight"] = r(hv * 128, hidden)
            t[a + "in_proj_b.weight"] = r(hv, hidden)
            t[a + "in_proj_a.weight"] = r(hv, hidden)
            t[a + "A_log"] = r(hv)
            t[a + "dt_bias"] = r(hv)
            t[a + "conv1d.weight"] = r(conv, 1, 4)
            t[a + "norm.weight"] = r(128)
            t[a + "out_proj.weight"] = r(hidden, hv * 128)
        else:
            a = p + "self_attn."
            t[a + "q_proj.weight"] = r(hq * 512, hidden)
            t[a + "k_proj.weight"] = r(hkv * 256, hidden)
            t[a + "v_proj.weight"] = r(hkv * 256, hidden)
            t[a + "o_proj.weight"] = r(hidden, hq * 256)
            t[a + "q_norm.weight"] = r(256)
            t[a + "k_norm.weight"] = r(256)
    return t


def check_q8(pair, w_in_out):
    words, scales = pair
    assert words.dtype == torch.int32 and words.shape == (w_in_out.shape[0], w_in_out.shape[1] // 4)
    assert scales.shape == (w_in_out.shape[0], w_in_out.shape[1] // 64)
    err = (ck.dequantize_q8f(words, scales) - w_in_out).abs()
    assert bool((err <= scales.repeat_interleave(64, dim=1) * 0.5 + 1e-9).all())


def test_quantizer_bound_and_zero_block():
    w = torch.randn(8, 192) * 3
    w[2, 64:128] = 0.0
    words, scales = ck.quantize_q8f(w)
    check_q8((words, scales), w)
    assert float(scales[2, 1]) == 1.0 and torch.all(ck.dequantize_q8f(words, scales)[2, 64:128] == 0)
    q = words.view(torch.int8)
    assert int(q.abs().max()) == 127  # every block's largest value maps to +-127
    with pytest.raises(ValueError):
        ck.quantize_q8f(torch.randn(4, 100))


def test_safetensors_mapping(tmp_path):
    from safetensors.torch import save_file
    t = hf_tensors()
    path = str(tmp_path / "model.safetensors")
    save_file(t, path)
    W = ck.read_safetensors(path)
    check_q8(W["embed"], t["model.language_model.embed_tokens.weight"])
    assert torch.equal(W["final_norm"], t["model.language_model.norm.weight"])
    assert sorted(W["layers"]) == [0, 1]
    L0, L1 = W["layers"][0], W["layers"][1]
    p0, p1 = "model.language_model.layers.0.", "model.language_model.layers.1."
    check_q8(L0["up"], t[p0 + "mlp.up_proj.weight"].t())
    check_q8(L0["down"], t[p0 + "mlp.down_proj.weight"].t())
    check_q8(L0["qkv"], t[p0 + "linear_attn.in_proj_qkv.weight"].t())
    check_q8(L0["out"], t[p0 + "linear_attn.out_proj.weight"].t())
    assert torch.equal(L0["w_b"], t[p0 + "linear_attn.in_proj_b.weight"].t())
    assert torch.equal(L0["a_log"], t[p0 + "linear_attn.A_log"])
    assert L0["conv_w"].shape == (384, 4) and torch.equal(L0["conv_w"], t[p0 + "linear_attn.conv1d.weight"][:, 0])
    check_q8(L1["q"], t[p1 + "self_attn.q_proj.weight"].t())
    check_q8(L1["o"], t[p1 + "self_attn.o_proj.weight"].t())
    assert torch.equal(L1["kn_w"], t[p1 + "self_attn.k_norm.weight"])
    assert set(L0) == {"in_norm", "post_norm", "up", "gate", "down", "qkv", "z", "out", "w_b", "w_a", "a_log",
                       "dt_bias", "conv_w", "norm_w"}
    assert set(L1) == {"in_norm", "post_norm", "up", "gate", "down", "q", "k", "v", "o", "qn_w", "kn_w"}


def test_prefix_without_model():
    t = {k[len("model."):]: v for k, v in hf_tensors().items()}
    W = ck.convert(t)
    assert sorted(W["layers"]) == [0, 1] and "embed" in W
