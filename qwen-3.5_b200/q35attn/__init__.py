"""q35attn -- B200 (sm_100a) attention hot path of the Qwen3.5 hybrid decoder.

Gated DeltaNet (decode, chunked prefill, gate projection), gated GQA
flash-decode and prefill, the Q8F decode GEMV and prefill GEMM, behind the C ABI of include/q35attn.h.  The Python layer is a
thin ctypes binding over device pointers; all math runs in libq35attn.so.
"""
from ._lib import (GdnDims, GqaDims, LIB_PATH, Q35Error, STATUS_CACHE_FULL, STATUS_LEN_HINT,  # noqa: F401
                   STATUS_WAIT_TIMEOUT, load)
from .ops import (GqaPrefillWorkspace, GqaWorkspace, gdn_decode, gdn_gate, gdn_prefill,  # noqa: F401
                  gdn_prefill_workspace, gqa_combine_partials, gqa_decode, gqa_decode_partial, gqa_prefill, launch_count,
                  q8_gemm, q8_gemm_fused, q8_gemm_workspace, q8_gemv, q8_gemv_fused, device_status,
                  workspace_status)
from .parallel import PeerExchange  # noqa: F401

__version__ = "0.1.0"
