"""ctypes binding of libq35attn.so (the C ABI declared in include/q35attn.h).

Pointers are passed as integers (``tensor.data_ptr()``), streams as the raw
``cudaStream_t`` integer (``torch.cuda.current_stream().cuda_stream``).  Every
non-zero status is raised as :class:`Q35Error` carrying the library's message.
There is no fallback: if the shared library is missing or fails to load, the
import fails loudly.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libq35attn.so")

OK, ERR_INVALID_ARG, ERR_UNSUPPORTED, ERR_CAPACITY, ERR_WORKSPACE, ERR_CUDA, ERR_DEVICE = range(7)
STATUS_CACHE_FULL, STATUS_LEN_HINT, STATUS_WAIT_TIMEOUT = 0x1, 0x2, 0x4

_ERR_NAMES = {1: "INVALID_ARG", 2: "UNSUPPORTED", 3: "CAPACITY", 4: "WORKSPACE", 5: "CUDA", 6: "DEVICE"}


class Q35Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"q35attn error {code} ({_ERR_NAMES.get(code, '?')}): {msg}")
        self.code = code


class GdnDims(C.Structure):
    _fields_ = [("batch", C.c_int32), ("num_k_heads", C.c_int32), ("num_v_heads", C.c_int32),
                ("head_k_dim", C.c_int32), ("head_v_dim", C.c_int32), ("conv_kernel", C.c_int32),
                ("eps", C.c_float)]


class GqaDims(C.Structure):
    _fields_ = [("batch", C.c_int32), ("num_q_heads", C.c_int32), ("num_kv_heads", C.c_int32),
                ("head_dim", C.c_int32), ("rotary_dim", C.c_int32), ("reserved", C.c_int32),
                ("capacity", C.c_int64), ("eps", C.c_float)]


class Q8Segment(C.Structure):
    _fields_ = [("w", C.c_void_p), ("scales", C.c_void_p), ("y", C.c_void_p), ("out_dim", C.c_int32)]


_P = C.c_void_p
_I32, _I64, _SZ = C.c_int32, C.c_int64, C.c_size_t

# name -> (restype, argtypes); the symbol test checks this table against the header
SIGNATURES = {
    "q35_gdn_decode": (C.c_int, [C.POINTER(GdnDims), _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "q35_gdn_decode_split": (C.c_int, [C.POINTER(GdnDims), _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "q35_gdn_prefill_workspace_size": (_SZ, [C.POINTER(GdnDims), _I32]),
    "q35_gdn_prefill": (C.c_int, [C.POINTER(GdnDims), _I32, _P, _P, _P, _P, _P, _P, _P, _I32, _P, _I32, _P, _P, _SZ,
                                  _P]),
    "q35_gdn_gate": (C.c_int, [_I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _I32, _P]),
    "q35_q8_gemv": (C.c_int, [_I32, _I32, _P, _P, _P, _P, _I32, _P]),
    "q35_q8_gemv_fused": (C.c_int, [_I32, _I32, C.POINTER(Q8Segment), _P, _P, _P, C.c_float, _P, _P, _I32, _I32,
                                    _P]),
    "q35_q8_embedding": (C.c_int, [_I32, _I32, _I32, _P, _P, _P, _P, _P]),
    "q35_add_rmsnorm": (C.c_int, [_I32, _I32, _P, _P, _P, C.c_float, _P, _P, _P]),
    "q35_silu_mul": (C.c_int, [_I64, _P, _P, _P, _P]),
    "q35_q8_lm_head": (C.c_int, [_I32, _I32, _P, _P, _P, _P, _P]),
    "q35_argmax_workspace_size": (_SZ, []),
    "q35_argmax": (C.c_int, [_I32, _P, _P, _P, _SZ, _P]),
    "q35_q8_dequant": (C.c_int, [_I32, _I32, _P, _P, _P, _P]),
    "q35_rope_gather": (C.c_int, [_I32, _I32, _I32, _P, _P, _P, _P, _P, _P]),
    "q35_gqa_decode_workspace_size": (_SZ, [C.POINTER(GqaDims), _I64]),
    "q35_workspace_init": (C.c_int, [_P, _SZ, _P]),
    "q35_gqa_decode": (C.c_int, [C.POINTER(GqaDims), _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "q35_gqa_prefill_workspace_size": (_SZ, [C.POINTER(GqaDims), _I32, _I64]),
    "q35_gqa_prefill": (C.c_int, [C.POINTER(GqaDims), _I32, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                  _SZ, _P]),
    "q35_workspace_status": (C.c_int, [_P, C.POINTER(C.c_uint32), _I32, _P]),
    "q35_gqa_decode_partial": (C.c_int, [C.POINTER(GqaDims), _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                         _SZ, _P]),
    "q35_gqa_combine_partials": (C.c_int, [_I32, _I32, _I32, _I32, _P, _P, _P, _P]),
    "q35_gqa_decode_noalloc": (C.c_int, [C.POINTER(GqaDims), _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "q35_last_error": (C.c_char_p, []),
    "q35_version": (C.c_char_p, []),
    "q35_launch_count": (C.c_uint64, [_I32]),
    "q35_test_arm_wait_fault": (C.c_int, [_I32]),
    "q35_cp_create": (C.c_int, [_I32, _I32, _I32, _I32, _I32, _I32, C.POINTER(C.c_void_p), _P]),
    "q35_cp_connect": (C.c_int, [_P, _P]),
    "q35_cp_exchange": (C.c_int, [_P, _P, _P, _P, _P, _P, _P]),
    "q35_cp_status": (C.c_int, [_P, C.POINTER(C.c_uint32), _I32, _P]),
    "q35_cp_disconnect": (C.c_int, [_P]),
    "q35_cp_destroy": (C.c_int, [_P]),
    "q35_device_status": (C.c_int, [C.POINTER(C.c_uint32), _I32, _P]),
    "q35_q8_gemm_workspace_size": (_SZ, [_I32, _I32]),
    "q35_q8_gemm": (C.c_int, [_I32, _I32, _I32, _P, _P, _P, _P, _P, _SZ, _P]),
    "q35_q8_gemm_fused": (C.c_int, [_I32, _I32, _I32, C.POINTER(Q8Segment), _P, _I32, _P, _SZ, _P]),
}

_lib = None


def load(path: str = LIB_PATH):
    """Load the library (building it first if the in-tree .so is stale)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path) or os.environ.get("Q35_AUTOBUILD", "1") == "1":
        from . import build as _build
        if _build.is_stale():
            _build.build()
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc != OK:
        raise Q35Error(rc, load().q35_last_error().decode())
