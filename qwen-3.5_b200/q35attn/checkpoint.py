"""Checkpoint import for the hybrid stack: a Hugging Face safetensors file of
the Qwen3.5 text model into the Q8F / f32 tensors that HybridStack uses.

Follows the reference's conversion (inventwithdean/Qwen-3.5 src/main.rs:160-222,
``_quantize_and_save``):

* keys: the ``model.`` prefix is optional, the text model lives under
  ``language_model.`` and ``A_log`` is the module's ``a_log``;
* PyTorch ``Linear`` weights are ``[out, in]`` and are transposed to the
  ``[in, out]`` layout the projections use (the PyTorchToBurnAdapter);
  ``conv1d.weight`` ``[C, 1, K]`` is squeezed to ``[C, K]``; everything is cast
  to f32 (FloatCastAdapter);
* the embedding (tied lm_head), the MLP projections, the attention q/k/v/o and
  the GatedDeltaNet in_proj_qkv / in_proj_z / out_proj are quantised to Q8F
  with one f32 scale per block of 64 consecutive values of a row (QuantScheme
  per_block([64]), MinMax calibration); in_proj_a / in_proj_b, the norms,
  conv1d, A_log and dt_bias stay f32.

The quantiser here is symmetric: scale = max|block| / 127 and
q = round(w / scale) in [-127, 127].  The reference's calibration is Burn's
(not in this repository), so a block can differ from it by one rounding step;
the error bound that both satisfy, |w - q * scale| <= scale / 2, is what the
tests check.
"""
from __future__ import annotations

import re

import torch

_LAYER = re.compile(r"^(?:model\.)?language_model\.layers\.(\d+)\.(.+)$")
_TOP = re.compile(r"^(?:model\.)?language_model\.(embed_tokens\.weight|norm\.weight)$")

# checkpoint suffix -> (HybridStack layer key, kind); kind "q8" = transposed and quantised Linear,
# "lin" = transposed f32 Linear, "f32" = as stored, "conv" = [C, 1, K] -> [C, K]
_LAYER_KEYS = {
    "input_layernorm.weight": ("in_norm", "f32"),
    "post_attention_layernorm.weight": ("post_norm", "f32"),
    "mlp.up_proj.weight": ("up", "q8"),
    "mlp.gate_proj.weight": ("gate", "q8"),
    "mlp.down_proj.weight": ("down", "q8"),
    "linear_attn.in_proj_qkv.weight": ("qkv", "q8"),
    "linear_attn.in_proj_z.weight": ("z", "q8"),
    "linear_attn.out_proj.weight": ("out", "q8"),
    "linear_attn.in_proj_b.weight": ("w_b", "lin"),
    "linear_attn.in_proj_a.weight": ("w_a", "lin"),
    "linear_attn.A_log": ("a_log", "f32"),
    "linear_attn.a_log": ("a_log", "f32"),
    "linear_attn.dt_bias": ("dt_bias", "f32"),
    "linear_attn.conv1d.weight": ("conv_w", "conv"),
    "linear_attn.norm.weight": ("norm_w", "f32"),
    "self_attn.q_proj.weight": ("q", "q8"),
    "self_attn.k_proj.weight": ("k", "q8"),
    "self_attn.v_proj.weight": ("v", "q8"),
    "self_attn.o_proj.weight": ("o", "q8"),
    "self_attn.q_norm.weight": ("qn_w", "f32"),
    "self_attn.k_norm.weight": ("kn_w", "f32"),
}


def quantize_q8f(w: torch.Tensor):
    """Q8F of a [rows, cols] f32 matrix (cols % 64 == 0): (words int32 [rows,
    cols/4] holding 4 little-endian int8 per word, scales f32 [rows, cols/64])."""
    rows, cols = w.shape
    if cols % 64:
        raise ValueError(f"Q8F needs a multiple of 64 columns, got {cols}")
    blk = w.float().reshape(rows, cols // 64, 64)
    amax = blk.abs().amax(-1)
    scales = torch.where(amax > 0, amax / 127.0, torch.ones_like(amax))
    q = torch.round(blk / scales[..., None]).clamp_(-127, 127).to(torch.int8).reshape(rows, cols)
    return q.contiguous().view(torch.int32), scales.contiguous()


def dequantize_q8f(words: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    q = words.contiguous().view(torch.int8).float()
    return q * scales.repeat_interleave(64, dim=1)


def convert(tensors: dict) -> dict:
    """Maps a {checkpoint key: tensor} dict onto {"embed": (words, scales),
    "final_norm": t, "layers": {i: {key: tensor or (words, scales)}}}.  Keys
    outside the text model (vision tower, MTP heads) are ignored."""
    out = {"layers": {}}
    for name, t in tensors.items():
        m = _TOP.match(name)
        if m:
            if m.group(1) == "embed_tokens.weight":
                out["embed"] = quantize_q8f(t.float())
            else:
                out["final_norm"] = t.float().contiguous()
            continue
        m = _LAYER.match(name)
        if not m or m.group(2) not in _LAYER_KEYS:
            continue
        key, kind = _LAYER_KEYS[m.group(2)]
        if kind == "q8":
            v = quantize_q8f(t.float().t())
        elif kind == "lin":
            v = t.float().t().contiguous()
        elif kind == "conv":
            v = t.float().reshape(t.shape[0], t.shape[-1]).contiguous()
        else:
            v = t.float().contiguous()
        out["layers"].setdefault(int(m.group(1)), {})[key] = v
    return out


def read_safetensors(path: str) -> dict:
    from safetensors.torch import load_file
    return convert(load_file(path))


def load_into(stack, weights: dict) -> None:
    """Copies converted weights into a HybridStack built with the matching
    StackConfig (shapes are checked; every tensor of the stack must be given)."""
    def put(dst, src, what):
        if hasattr(dst, "words"):
            words, scales = src
            if tuple(words.shape) != tuple(dst.words.shape) or tuple(scales.shape) != tuple(dst.scales.shape):
                raise ValueError(f"{what}: shape {tuple(words.shape)} does not match {tuple(dst.words.shape)}")
            dst.words.copy_(words)
            dst.scales.copy_(scales)
        else:
            if tuple(src.shape) != tuple(dst.shape):
                raise ValueError(f"{what}: shape {tuple(src.shape)} does not match {tuple(dst.shape)}")
            dst.copy_(src)

    if "embed" not in weights or "final_norm" not in weights:
        raise ValueError("checkpoint lacks embed_tokens or the final norm")
    put(stack.embed, weights["embed"], "embed_tokens")
    put(stack.final_norm, weights["final_norm"], "norm")
    for i, L in enumerate(stack.layers):
        W = weights["layers"].get(i, {})
        for key, dst in L.items():
            if key in ("kind", "conv_state", "rec_state", "K", "V", "lens"):
                continue
            if key not in W:
                raise ValueError(f"layer {i}: checkpoint lacks {key}")
            put(dst, W[key], f"layer {i} {key}")
    stack.reset()
    stack.graph = None
    stack._plan = None
