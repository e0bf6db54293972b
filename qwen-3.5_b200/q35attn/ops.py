"""Torch-facing wrappers of the C ABI (device tensors in, device tensors out).

PyTorch is used only for device memory and streams; every computation runs in
libq35attn's sm_100a kernels.  Inputs must be contiguous float32 CUDA tensors
(int32 for ``lens``); anything else raises instead of being converted.
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import GdnDims, GqaDims, Q35Error, Q8Segment, check, load

__all__ = ["gdn_decode", "gdn_prefill", "gdn_prefill_workspace", "gdn_gate", "GqaWorkspace", "gqa_decode", "GqaPrefillWorkspace", "gqa_prefill",
           "q8_gemv", "q8_gemv_fused", "q8_gemm", "q8_gemm_fused", "q8_gemm_workspace", "device_status", "launch_count", "Q35Error"]


def _req(t: torch.Tensor, name: str, dtype=torch.float32) -> int:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must live on a CUDA device (got {t.device})")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype} (got {t.dtype})")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t.data_ptr()


def _stream(stream) -> int:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


def launch_count(reset: bool = False) -> int:
    return int(load().q35_launch_count(1 if reset else 0))


def gdn_dims(batch, num_k_heads, num_v_heads, conv_kernel=4, eps=1e-6, head_dim=128) -> GdnDims:
    return GdnDims(batch, num_k_heads, num_v_heads, head_dim, head_dim, conv_kernel, eps)


def gdn_decode(mixed_qkv, z, beta, g, conv_w, norm_w, conv_state, rec_state, out=None, *, num_k_heads,
               num_v_heads, eps=1e-6, split=0, stream=None):
    """One decode step of the Gated DeltaNet core; conv_state / rec_state are
    updated in place.  Returns ``out`` [B, Hv*128]."""
    B = mixed_qkv.shape[0]
    if out is None:
        out = torch.empty(B, num_v_heads * 128, device=mixed_qkv.device, dtype=torch.float32)
    d = gdn_dims(B, num_k_heads, num_v_heads, conv_w.shape[1], eps)
    ptrs = [_req(t, n) for t, n in ((mixed_qkv, "mixed_qkv"), (z, "z"), (beta, "beta"), (g, "g"),
                                     (conv_w, "conv_w"), (norm_w, "norm_w"), (conv_state, "conv_state"),
                                     (rec_state, "rec_state"), (out, "out"))]
    lib = load()
    if split:
        check(lib.q35_gdn_decode_split(C.byref(d), int(split), *ptrs, _stream(stream)))
    else:
        check(lib.q35_gdn_decode(C.byref(d), *ptrs, _stream(stream)))
    return out


def gdn_prefill_workspace(B, T, num_k_heads, num_v_heads, conv_kernel=4, device="cuda", stream=None):
    """Workspace of q35_gdn_prefill; its leading status word is zeroed."""
    d = gdn_dims(B, num_k_heads, num_v_heads, conv_kernel)
    n = int(load().q35_gdn_prefill_workspace_size(C.byref(d), int(T)))
    buf = torch.empty(max(n, 256), dtype=torch.uint8, device=device)
    check(load().q35_workspace_init(buf.data_ptr(), 256, _stream(stream)))
    return buf


def workspace_status(workspace: torch.Tensor, clear=False, stream=None) -> int:
    """Q35_STATUS_* bits of a workspace's leading status word (synchronizes)."""
    v = C.c_uint32(0)
    check(load().q35_workspace_status(workspace.data_ptr(), C.byref(v), int(clear), _stream(stream)))
    return int(v.value)


def gdn_prefill(mixed_qkv, z, beta, g, conv_w, norm_w, conv_state, rec_state, out=None, *, num_k_heads,
                num_v_heads, has_prev_conv=False, has_init_state=False, workspace=None, eps=1e-6, stream=None):
    """Chunked prefill over T tokens; conv_state / rec_state updated in place.
    Returns ``out`` [B, T, Hv*128]."""
    B, T = mixed_qkv.shape[:2]
    if out is None:
        out = torch.empty(B, T, num_v_heads * 128, device=mixed_qkv.device, dtype=torch.float32)
    if workspace is None:
        workspace = gdn_prefill_workspace(B, T, num_k_heads, num_v_heads, conv_w.shape[1], mixed_qkv.device)
    d = gdn_dims(B, num_k_heads, num_v_heads, conv_w.shape[1], eps)
    lib = load()
    check(lib.q35_gdn_prefill(C.byref(d), int(T), _req(mixed_qkv, "mixed_qkv"), _req(z, "z"), _req(beta, "beta"),
                              _req(g, "g"), _req(conv_w, "conv_w"), _req(norm_w, "norm_w"),
                              _req(conv_state, "conv_state"), int(bool(has_prev_conv)), _req(rec_state, "rec_state"),
                              int(bool(has_init_state)), _req(out, "out"), _req(workspace, "workspace", torch.uint8),
                              workspace.numel(), _stream(stream)))
    return out


def gdn_gate(x, w_b, w_a, a_log, dt_bias, mode=0, beta=None, g=None, stream=None):
    N, in_dim = x.shape
    H = w_b.shape[1]
    if beta is None:
        beta = torch.empty(N, H, device=x.device, dtype=torch.float32)
    if g is None:
        g = torch.empty(N, H, device=x.device, dtype=torch.float32)
    check(load().q35_gdn_gate(N, in_dim, H, _req(x, "x"), _req(w_b, "w_b"), _req(w_a, "w_a"), _req(a_log, "a_log"),
                              _req(dt_bias, "dt_bias"), _req(beta, "beta"), _req(g, "g"), int(mode),
                              _stream(stream)))
    return beta, g


def q8_gemv(x, w, scales, y=None, *, mode=0, stream=None):
    """y [out] = x [in] @ W for a Q8F matrix: w [in, out/4] int32/uint32 words
    (4 little-endian int8 columns each), scales [in, out/64].  mode 1 covers
    only the rows the reference's split-K kernel covers."""
    in_dim = x.numel()
    out_dim = w.shape[1] * 4
    if w.dtype not in (torch.int32, torch.uint32) or not w.is_contiguous() or w.device.type != "cuda":
        raise TypeError("w must be a contiguous int32/uint32 CUDA tensor")
    if y is None:
        y = torch.empty(out_dim, device=x.device, dtype=torch.float32)
    check(load().q35_q8_gemv(in_dim, out_dim, _req(x, "x"), w.data_ptr(), _req(scales, "scales"), _req(y, "y"),
                             int(mode), _stream(stream)))
    return y


def q8_gemm_workspace(n_rows, in_dim, device="cuda"):
    """Workspace of q35_q8_gemm / q35_q8_gemm_fused (x split into bf16 terms)."""
    n = int(load().q35_q8_gemm_workspace_size(int(n_rows), int(in_dim)))
    if n == 0:
        raise Q35Error(1, "invalid q8_gemm sizes for a workspace")
    return torch.empty(n, dtype=torch.uint8, device=device)


def q8_gemm(x, w, scales, y=None, *, workspace=None, stream=None):
    """y [T, out] = x [T, in] @ W for a Q8F matrix (layout as for q8_gemv),
    the prefill projection, on the tensor cores with W dequantised on load."""
    T, in_dim = x.shape
    out_dim = w.shape[1] * 4
    if y is None:
        y = torch.empty(T, out_dim, device=x.device, dtype=torch.float32)
    if workspace is None:
        workspace = q8_gemm_workspace(T, in_dim, x.device)
    check(load().q35_q8_gemm(int(T), int(in_dim), int(out_dim), _req(x, "x"), _words(w), _req(scales, "scales"),
                             _req(y, "y"), _req(workspace, "workspace", torch.uint8), workspace.numel(),
                             _stream(stream)))
    return y


def q8_gemm_fused(x, weights, ys, *, swiglu=False, workspace=None, stream=None):
    """Up to four Q8F projections of the same rows x [T, in] in one launch:
    weights = [(words, scales), ...], ys = [y [T, out_i], ...].  With
    swiglu=True, exactly (up, gate): ys[0] receives up * silu(gate)."""
    T, in_dim = x.shape
    n = len(weights)
    segs = (Q8Segment * n)()
    for i, ((w, sc), y) in enumerate(zip(weights, ys)):
        segs[i].w = _words(w)
        segs[i].scales = _req(sc, "scales")
        segs[i].y = _req(y, "y")
        segs[i].out_dim = int(w.shape[1] * 4)
    if workspace is None:
        workspace = q8_gemm_workspace(T, in_dim, x.device)
    check(load().q35_q8_gemm_fused(int(T), int(in_dim), n, segs, _req(x, "x"), int(bool(swiglu)),
                                   _req(workspace, "workspace", torch.uint8), workspace.numel(), _stream(stream)))
    return ys[0]


def device_status(clear=False, stream=None) -> int:
    """Q35_STATUS_* bits of this device's status word (kernels without a workspace)."""
    v = C.c_uint32(0)
    check(load().q35_device_status(C.byref(v), int(clear), _stream(stream)))
    return int(v.value)


def _words(w, name="w") -> int:
    if w.dtype not in (torch.int32, torch.uint32) or not w.is_contiguous() or w.device.type != "cuda":
        raise TypeError(f"{name} must be a contiguous int32/uint32 CUDA tensor")
    return w.data_ptr()


class FusedGemv:
    """A prepared q35_q8_gemv_fused call: the segment table is built once, so a
    decode step (or a CUDA graph capture) pays no per-call Python packing."""

    def __init__(self, x, weights, ys, *, residual=None, norm_w=None, eps=1e-6, sum_out=None, x_out=None,
                 swiglu=False, mode=0):
        if not 1 <= len(weights) <= 4 or len(ys) != len(weights):
            raise ValueError("1 to 4 (w, scales) pairs, one y each")
        self.in_dim = x.numel()
        segs = (Q8Segment * len(weights))()
        for k, ((w, sc), y) in enumerate(zip(weights, ys)):
            segs[k].w = _words(w)
            segs[k].scales = _req(sc, "scales")
            segs[k].y = _req(y, "y")
            segs[k].out_dim = w.shape[1] * 4
        self.segs = segs
        opt = lambda t, n: 0 if t is None else _req(t, n)
        self.args = (self.in_dim, len(weights), segs, _req(x, "x"), opt(residual, "residual"), opt(norm_w, "norm_w"),
                     float(eps), opt(sum_out, "sum_out"), opt(x_out, "x_out"), int(bool(swiglu)), int(mode))
        self._keep = (x, weights, ys, residual, norm_w, sum_out, x_out)

    def __call__(self, stream=None):
        check(load().q35_q8_gemv_fused(*self.args, _stream(stream)))


def q8_gemv_fused(x, weights, *, ys=None, residual=None, norm_w=None, eps=1e-6, sum_out=None, x_out=None,
                  swiglu=False, mode=0, stream=None):
    """Up to four Q8F GEMVs of one input in one launch (q35_q8_gemv_fused):
    weights = [(w, scales), ...]; with norm_w the input is RMSNorm(x +
    residual) * (1 + norm_w) and sum_out / x_out receive x + residual and the
    normalised input; swiglu=True takes (up, gate) and returns up * silu(gate).
    Returns the list of outputs (one tensor when swiglu)."""
    if ys is None:
        ys = [torch.empty(w.shape[1] * 4, device=x.device, dtype=torch.float32) for w, _ in weights]
    FusedGemv(x, weights, ys, residual=residual, norm_w=norm_w, eps=eps, sum_out=sum_out, x_out=x_out,
              swiglu=swiglu, mode=mode)(stream)
    return ys[0] if swiglu else ys


def gqa_dims(batch, num_q_heads, num_kv_heads, capacity, rotary_dim=64, eps=1e-6, head_dim=256) -> GqaDims:
    return GqaDims(batch, num_q_heads, num_kv_heads, head_dim, rotary_dim, 0, capacity, eps)


class GqaWorkspace:
    """Scratch for the split-K partials and arrival counters of q35_gqa_decode,
    zeroed once at creation (the kernel leaves it reusable)."""

    def __init__(self, batch, num_q_heads, num_kv_heads, capacity, max_len=None, device="cuda", stream=None):
        self.dims = gqa_dims(batch, num_q_heads, num_kv_heads, capacity)
        self.max_len = int(max_len or capacity)
        n = int(load().q35_gqa_decode_workspace_size(C.byref(self.dims), self.max_len))
        if n == 0:
            raise Q35Error(1, "invalid GQA dims for workspace")
        self.buf = torch.empty(n, dtype=torch.uint8, device=device)
        check(load().q35_workspace_init(self.buf.data_ptr(), n, _stream(stream)))

    def status(self, clear=False, stream=None) -> int:
        v = C.c_uint32(0)
        check(load().q35_workspace_status(self.buf.data_ptr(), C.byref(v), int(clear), _stream(stream)))
        return int(v.value)


def gqa_decode(q_gate, k_new, v_new, qn_w, kn_w, cos, sin, k_cache, v_cache, lens, out=None, *, workspace,
               max_len=None, rotary_dim=None, eps=1e-6, stream=None):
    """One gated-GQA decode step; appends to k_cache/v_cache at lens[b] and
    increments lens.  Returns ``out`` [B, Hq*256]."""
    B, Hq, _ = q_gate.shape
    Hkv, cap = k_cache.shape[1], k_cache.shape[2]
    rot = int(rotary_dim if rotary_dim is not None else cos.shape[-1])
    if out is None:
        out = torch.empty(B, Hq * 256, device=q_gate.device, dtype=torch.float32)
    d = gqa_dims(B, Hq, Hkv, cap, rot, eps)
    ml = int(max_len if max_len is not None else workspace.max_len)
    check(load().q35_gqa_decode(C.byref(d), ml, _req(q_gate, "q_gate"), _req(k_new, "k_new"), _req(v_new, "v_new"),
                                _req(qn_w, "qn_w"), _req(kn_w, "kn_w"), _req(cos, "cos"), _req(sin, "sin"),
                                _req(k_cache, "k_cache"), _req(v_cache, "v_cache"), _req(lens, "lens", torch.int32),
                                _req(out, "out"), workspace.buf.data_ptr(), workspace.buf.numel(), _stream(stream)))
    return out


class GqaPrefillWorkspace:
    """Scratch of q35_gqa_prefill (blocked q / k / v tiles + status word) for
    prompts of seq_len tokens with lens[b] + seq_len <= max_len."""

    def __init__(self, batch, num_q_heads, num_kv_heads, capacity, seq_len, max_len=None, device="cuda"):
        self.dims = gqa_dims(batch, num_q_heads, num_kv_heads, capacity)
        self.seq_len = int(seq_len)
        self.max_len = int(max_len or capacity)
        n = int(load().q35_gqa_prefill_workspace_size(C.byref(self.dims), self.seq_len, self.max_len))
        if n == 0:
            raise Q35Error(1, "invalid GQA prefill shape for workspace")
        self.buf = torch.zeros(n, dtype=torch.uint8, device=device)

    def status(self, clear=False, stream=None) -> int:
        v = C.c_uint32(0)
        check(load().q35_workspace_status(self.buf.data_ptr(), C.byref(v), int(clear), _stream(stream)))
        return int(v.value)


def gqa_prefill(q_gate, k_new, v_new, qn_w, kn_w, cos, sin, k_cache, v_cache, lens, out=None, *, workspace=None,
                max_len=None, rotary_dim=None, eps=1e-6, stream=None):
    """Gated-GQA attention over a prompt: q_gate [B, T, Hq, 512], k_new / v_new
    [B, T, Hkv, 256], cos / sin [B, T, rot]; appends to the caches at lens[b]
    and adds T to lens.  Returns ``out`` [B, T, Hq*256]."""
    B, T, Hq, _ = q_gate.shape
    Hkv, cap = k_cache.shape[1], k_cache.shape[2]
    rot = int(rotary_dim if rotary_dim is not None else cos.shape[-1])
    if out is None:
        out = torch.empty(B, T, Hq * 256, device=q_gate.device, dtype=torch.float32)
    if workspace is None:
        workspace = GqaPrefillWorkspace(B, Hq, Hkv, cap, T, max_len, q_gate.device)
    d = gqa_dims(B, Hq, Hkv, cap, rot, eps)
    ml = int(max_len if max_len is not None else workspace.max_len)
    cp = _req(cos, "cos") if rot > 0 else None
    sp = _req(sin, "sin") if rot > 0 else None
    check(load().q35_gqa_prefill(C.byref(d), int(T), ml, _req(q_gate, "q_gate"), _req(k_new, "k_new"),
                                 _req(v_new, "v_new"), _req(qn_w, "qn_w"), _req(kn_w, "kn_w"), cp, sp,
                                 _req(k_cache, "k_cache"), _req(v_cache, "v_cache"), _req(lens, "lens", torch.int32),
                                 _req(out, "out"), workspace.buf.data_ptr(), workspace.buf.numel(), _stream(stream)))
    return out


def gqa_decode_partial(q_gate, k_new, v_new, qn_w, kn_w, cos, sin, k_cache, v_cache, lens, partial_out=None, *,
                       workspace, max_len=None, rotary_dim=None, eps=1e-6, stream=None):
    """Context-parallel shard of a GQA decode step: writes the unnormalised
    softmax partial [B, Hq, 256+2] = [o | m (log2 units) | l] over this shard's
    keys.  k_new / v_new None: attend cached keys only (no append)."""
    B, Hq, _ = q_gate.shape
    Hkv, cap = k_cache.shape[1], k_cache.shape[2]
    rot = int(rotary_dim if rotary_dim is not None else cos.shape[-1])
    if partial_out is None:
        partial_out = torch.empty(B, Hq, 256 + 2, device=q_gate.device, dtype=torch.float32)
    d = gqa_dims(B, Hq, Hkv, cap, rot, eps)
    ml = int(max_len if max_len is not None else workspace.max_len)
    kp = _req(k_new, "k_new") if k_new is not None else None
    vp = _req(v_new, "v_new") if v_new is not None else None
    check(load().q35_gqa_decode_partial(C.byref(d), ml, _req(q_gate, "q_gate"), kp, vp, _req(qn_w, "qn_w"),
                                        _req(kn_w, "kn_w"), _req(cos, "cos"), _req(sin, "sin"),
                                        _req(k_cache, "k_cache"), _req(v_cache, "v_cache"),
                                        _req(lens, "lens", torch.int32), _req(partial_out, "partial_out"),
                                        workspace.buf.data_ptr(), workspace.buf.numel(), _stream(stream)))
    return partial_out


def gqa_combine_partials(parts, q_gate, out=None, stream=None):
    """parts [n, B, Hq, 258] -> out [B, Hq*256] = merged softmax * sigmoid(gate)."""
    n, B, Hq, _ = parts.shape
    if out is None:
        out = torch.empty(B, Hq * 256, device=parts.device, dtype=torch.float32)
    check(load().q35_gqa_combine_partials(B, Hq, 256, n, _req(parts, "parts"), _req(q_gate, "q_gate"),
                                          _req(out, "out"), _stream(stream)))
    return out


# ---------------------------------------------------------------- stack glue

def q8_embedding(ids, table, scales, out=None, stream=None):
    """out [n, dim] = dequantised rows ids of a Q8F table ([vocab, dim/4] words, [vocab, dim/64] scales)."""
    n = ids.numel()
    vocab, dim = table.shape[0], table.shape[1] * 4
    if out is None:
        out = torch.empty(n, dim, device=table.device, dtype=torch.float32)
    check(load().q35_q8_embedding(n, vocab, dim, _req(ids, "ids", torch.int32), table.data_ptr(),
                                  _req(scales, "scales"), _req(out, "out"), _stream(stream)))
    return out


def add_rmsnorm(x, weight, out, residual=None, sum_out=None, eps=1e-6, stream=None):
    """out = RMSNorm(x + residual) * (1 + weight) row-wise; sum_out = x + residual."""
    dim = weight.numel()
    rows = x.numel() // dim
    check(load().q35_add_rmsnorm(rows, dim, _req(x, "x"), _req(residual, "residual") if residual is not None else None,
                                 _req(weight, "weight"), C.c_float(eps), _req(out, "out"),
                                 _req(sum_out, "sum_out") if sum_out is not None else None, _stream(stream)))
    return out


def silu_mul(gate, up, out, stream=None):
    check(load().q35_silu_mul(gate.numel(), _req(gate, "gate"), _req(up, "up"), _req(out, "out"), _stream(stream)))
    return out


def q8_lm_head(x, table, scales, logits, stream=None):
    check(load().q35_q8_lm_head(table.shape[0], x.numel(), _req(x, "x"), table.data_ptr(), _req(scales, "scales"),
                                _req(logits, "logits"), _stream(stream)))
    return logits


class ArgmaxWorkspace:
    def __init__(self, device="cuda"):
        self.buf = torch.empty(int(load().q35_argmax_workspace_size()), dtype=torch.uint8, device=device)


def argmax(x, out, workspace, stream=None):
    check(load().q35_argmax(x.numel(), _req(x, "x"), _req(out, "out", torch.int32), workspace.buf.data_ptr(),
                            workspace.buf.numel(), _stream(stream)))
    return out


def q8_dequant(words, scales, out, stream=None):
    rows, cols = words.shape[0], words.shape[1] * 4
    check(load().q35_q8_dequant(rows, cols, words.data_ptr(), _req(scales, "scales"), _req(out, "out"),
                                _stream(stream)))
    return out


def rope_gather(lens, table_cos, table_sin, cos_out, sin_out, stream=None):
    B = lens.numel()
    max_pos, rot = table_cos.shape
    check(load().q35_rope_gather(B, rot, max_pos, _req(lens, "lens", torch.int32), _req(table_cos, "table_cos"),
                                 _req(table_sin, "table_sin"), _req(cos_out, "cos_out"), _req(sin_out, "sin_out"),
                                 _stream(stream)))
