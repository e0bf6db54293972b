"""ctypes wrapper for the CPU oracle (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline legs of bench.py
may import this module; the product path (qwen-3.5_b200/q35attn) never does.
Every function takes and returns numpy float32 / int32 arrays with the layouts
documented in q35_oracle.h and restates the reference function cited there.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libq35oracle.so")
_lib = None


def build(force: bool = False) -> str:
    src = os.path.join(_HERE, "q35_oracle.c")
    stale = (not os.path.exists(_LIB_PATH)) or os.path.getmtime(_LIB_PATH) < max(
        os.path.getmtime(src), os.path.getmtime(os.path.join(_HERE, "q35_oracle.h")))
    if force or stale:
        subprocess.run(["make", "-s", "-C", _HERE, "CC=gcc"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(_LIB_PATH)
    return _lib


def _f(a):
    assert a.dtype == np.float32 and a.flags.c_contiguous, (a.dtype, a.flags)
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _i32(a):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(C.POINTER(C.c_int32))


def _c(a, dt=np.float32):
    return np.ascontiguousarray(a, dtype=dt)


def set_threads(n: int) -> None:
    lib().q35o_set_threads(int(n))


def conv1d_update(x, conv_state, w):
    """text_modules.rs:134-162.  Returns (y, new_state)."""
    x, st, w = _c(x), _c(conv_state).copy(), _c(w)
    B, Cc = x.shape
    K = w.shape[1]
    y = np.empty_like(x)
    lib().q35o_conv1d_update(B, Cc, K, _f(x), _f(st), _f(w), _f(y))
    return y, st


def conv1d_prefill(x, conv_state, w, has_prev):
    x, st, w = _c(x), _c(conv_state).copy(), _c(w)
    B, T, Cc = x.shape
    K = w.shape[1]
    y = np.empty_like(x)
    lib().q35o_conv1d_prefill(B, T, Cc, K, _f(x), _f(st), int(has_prev), _f(w), _f(y))
    return y, st


def l2norm(x, eps=1e-6):
    x = _c(x).copy()
    d = x.shape[-1]
    lib().q35o_l2norm(C.c_int64(x.size // d), d, _f(x), C.c_float(eps))
    return x


def rmsnorm_gated(x, z, w, eps=1e-6):
    x, z, w = _c(x), _c(z), _c(w)
    d = x.shape[-1]
    y = np.empty_like(x)
    lib().q35o_rmsnorm_gated(C.c_int64(x.size // d), d, _f(x), _f(z), _f(w), C.c_float(eps), _f(y))
    return y


def rmsnorm(x, w, eps=1e-6):
    x, w = _c(x).copy(), _c(w)
    d = x.shape[-1]
    lib().q35o_rmsnorm(C.c_int64(x.size // d), d, _f(x), _f(w), C.c_float(eps))
    return x


def rope_tables(pos, rot=64, theta=1e7):
    pos = np.ascontiguousarray(pos, dtype=np.int64)
    n = pos.size
    cos = np.empty((n, rot), np.float32)
    sin = np.empty((n, rot), np.float32)
    lib().q35o_rope_tables(n, pos.ctypes.data_as(C.POINTER(C.c_int64)), rot, C.c_float(theta), _f(cos), _f(sin))
    return cos.reshape(pos.shape + (rot,)), sin.reshape(pos.shape + (rot,))


def gate_proj(x, wb, wa, a_log, dt_bias, mode=0):
    x, wb, wa, a_log, dt_bias = map(_c, (x, wb, wa, a_log, dt_bias))
    N, ind = x.shape
    H = wb.shape[1]
    beta = np.empty((N, H), np.float32)
    g = np.empty((N, H), np.float32)
    lib().q35o_gate_proj(N, ind, H, _f(x), _f(wb), _f(wa), _f(a_log), _f(dt_bias), _f(beta), _f(g), int(mode))
    return beta, g


def recurrent_gdr(q, k, v, g, beta, S):
    """q,k [B,T,Hk,DK]; v [B,T,Hv,DV]; g,beta [B,T,Hv]; S [B,Hv,DK,DV]."""
    q, k, v, g, beta, S = _c(q), _c(k), _c(v), _c(g), _c(beta), _c(S).copy()
    B, T, Hk, DK = q.shape
    Hv, DV = v.shape[2], v.shape[3]
    out = np.empty((B, T, Hv, DV), np.float32)
    lib().q35o_recurrent_gdr(B, T, Hk, Hv, DK, DV, _f(q), _f(k), _f(v), _f(g), _f(beta), _f(S), _f(out))
    return out, S


def chunk_gdr(q, k, v, g, beta, S, chunk=64):
    q, k, v, g, beta, S = _c(q), _c(k), _c(v), _c(g), _c(beta), _c(S).copy()
    B, T, Hk, DK = q.shape
    Hv, DV = v.shape[2], v.shape[3]
    out = np.empty((B, T, Hv, DV), np.float32)
    lib().q35o_chunk_gdr(B, T, Hk, Hv, DK, DV, chunk, _f(q), _f(k), _f(v), _f(g), _f(beta), _f(S), _f(out))
    return out, S


def gdn_decode(mixed_qkv, z, beta, g, conv_w, norm_w, conv_state, S, Hk, Hv, DK=128, DV=128, eps=1e-6,
               inplace=False):
    """Decode core of GatedDeltaNet::forward.  Returns (out, conv_state', S');
    with inplace=True the (contiguous float32) states are updated in place."""
    a = [_c(x) for x in (mixed_qkv, z, beta, g, conv_w, norm_w)]
    if inplace:
        st, S = _c(conv_state), _c(S)
    else:
        st, S = _c(conv_state).copy(), _c(S).copy()
    B = a[0].shape[0]
    K = a[4].shape[1]
    out = np.empty((B, Hv * DV), np.float32)
    lib().q35o_gdn_decode(B, Hk, Hv, DK, DV, K, *[_f(x) for x in a], _f(st), _f(S), _f(out), C.c_float(eps))
    return out, st, S


def gdn_prefill(mixed_qkv, z, beta, g, conv_w, norm_w, conv_state, has_prev, S, has_init,
                Hk, Hv, DK=128, DV=128, chunk=64, eps=1e-6):
    """Chunked branch of GatedDeltaNet::forward.  Returns (out, conv_state', S')."""
    a = [_c(x) for x in (mixed_qkv, z, beta, g, conv_w, norm_w)]
    st, S = _c(conv_state).copy(), _c(S).copy()
    B, T = a[0].shape[:2]
    K = a[4].shape[1]
    out = np.empty((B, T, Hv * DV), np.float32)
    lib().q35o_gdn_prefill(B, T, Hk, Hv, DK, DV, K, chunk, *[_f(x) for x in a], _f(st), int(has_prev),
                           _f(S), int(has_init), _f(out), C.c_float(eps))
    return out, st, S


def gqa_decode(q_gate, k_new, v_new, qn_w, kn_w, cos, sin, k_cache, v_cache, lens, rot=64, eps=1e-6,
               inplace=False):
    """Attention::forward decode core.  k_cache/v_cache [B,Hkv,cap,D] are copied (or, with
    inplace=True, updated in place when already contiguous float32) and returned updated
    together with lens.  Returns (out, k_cache', v_cache', lens')."""
    q_gate, k_new, v_new, qn_w, kn_w, cos, sin = map(_c, (q_gate, k_new, v_new, qn_w, kn_w, cos, sin))
    if inplace:
        kc, vc, lens = _c(k_cache), _c(v_cache), _c(lens, np.int32)
    else:
        kc, vc = _c(k_cache).copy(), _c(v_cache).copy()
        lens = _c(lens, np.int32).copy()
    B, Hq, D2 = q_gate.shape
    D = D2 // 2
    Hkv, cap = kc.shape[1], kc.shape[2]
    out = np.empty((B, Hq * D), np.float32)
    lib().q35o_gqa_decode(B, Hq, Hkv, D, rot, C.c_int64(cap), _f(q_gate), _f(k_new), _f(v_new), _f(qn_w),
                          _f(kn_w), _f(cos), _f(sin), _f(kc), _f(vc), _i32(lens), _f(out), C.c_float(eps))
    return out, kc, vc, lens


def gqa_prefill(q_gate, k_new, v_new, qn_w, kn_w, cos, sin, k_cache, v_cache, lens, rot=64, eps=1e-6):
    q_gate, k_new, v_new, qn_w, kn_w, cos, sin = map(_c, (q_gate, k_new, v_new, qn_w, kn_w, cos, sin))
    kc, vc = _c(k_cache).copy(), _c(v_cache).copy()
    lens = _c(lens, np.int32).copy()
    B, T, Hq, D2 = q_gate.shape
    D = D2 // 2
    Hkv, cap = kc.shape[1], kc.shape[2]
    out = np.empty((B, T, Hq * D), np.float32)
    lib().q35o_gqa_prefill(B, T, Hq, Hkv, D, rot, C.c_int64(cap), _f(q_gate), _f(k_new), _f(v_new), _f(qn_w),
                           _f(kn_w), _f(cos), _f(sin), _f(kc), _f(vc), _i32(lens), _f(out), C.c_float(eps))
    return out, kc, vc, lens


def q8_gemv(x, wq, scales, exact=False):
    x, scales = _c(x), _c(scales)
    wq = np.ascontiguousarray(wq, dtype=np.int8)
    ind, outd = wq.shape
    y = np.empty(outd, np.float32)
    lib().q35o_q8_gemv(ind, outd, _f(x), wq.ctypes.data_as(C.POINTER(C.c_int8)), _f(scales), _f(y), int(exact))
    return y


