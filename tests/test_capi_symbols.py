"""CPU checks of the C ABI library: it loads, exports every symbol the header
declares, the ctypes table matches the header, and host-side argument
validation rejects bad calls before any device work."""
import ctypes as C
import os
import re
import subprocess

import pytest

import q35attn
from q35attn import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include")) if f.endswith(".h")]


def declared_functions():
    names = set()
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b(q35_\w+)\s*\(", src):
            names.add(m.group(1))
    return names


def exported_symbols():
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True, check=True)
    return {line.split()[-1] for line in out.stdout.splitlines() if line.strip()}


def test_library_loads():
    lib = q35attn.load()
    assert lib.q35_version().decode().startswith("q35attn")


def test_every_declared_symbol_is_exported():
    decl = declared_functions()
    assert len(decl) >= 10
    missing = decl - exported_symbols()
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_ctypes_table_covers_header():
    assert declared_functions() == set(_lib.SIGNATURES)


def test_validation_errors_without_device():
    lib = q35attn.load()
    # NULL dims
    assert lib.q35_gdn_decode(None, *([None] * 10)) == _lib.ERR_INVALID_ARG
    assert "NULL" in lib.q35_last_error().decode()
    # unsupported head dim
    d = _lib.GdnDims(1, 16, 16, 64, 64, 4, 1e-6)
    assert lib.q35_gdn_decode(C.byref(d), *([None] * 10)) == _lib.ERR_UNSUPPORTED
    # Hv not a multiple of Hk
    d = _lib.GdnDims(1, 3, 16, 128, 128, 4, 1e-6)
    assert lib.q35_gdn_decode(C.byref(d), *([None] * 10)) == _lib.ERR_INVALID_ARG
    # batch 0 is a no-op
    d = _lib.GdnDims(0, 16, 16, 128, 128, 4, 1e-6)
    assert lib.q35_gdn_decode(C.byref(d), *([None] * 10)) == _lib.OK
    # GQA: group size 3 unsupported, max_len beyond capacity rejected on the host
    g = _lib.GqaDims(1, 6, 2, 256, 64, 0, 100, 1e-6)
    assert lib.q35_gqa_decode(C.byref(g), 10, *([None] * 12), 0, None) == _lib.ERR_UNSUPPORTED
    g = _lib.GqaDims(1, 8, 2, 256, 64, 0, 100, 1e-6)
    assert lib.q35_gqa_decode(C.byref(g), 101, *([None] * 12), 0, None) == _lib.ERR_CAPACITY
    assert lib.q35_gqa_decode(C.byref(g), 10, *([None] * 12), 0, None) == _lib.ERR_INVALID_ARG
    # odd rotary dim
    g = _lib.GqaDims(1, 8, 2, 256, 63, 0, 100, 1e-6)
    assert lib.q35_gqa_decode(C.byref(g), 10, *([None] * 12), 0, None) == _lib.ERR_INVALID_ARG
    # gate: bad mode
    assert lib.q35_gdn_gate(1, 64, 16, *([None] * 7), 2, None) == _lib.ERR_INVALID_ARG
    # prefill flags
    d = _lib.GdnDims(1, 16, 16, 128, 128, 4, 1e-6)
    assert lib.q35_gdn_prefill(C.byref(d), 8, *([None] * 7), 2, None, 0, None, None, 0, None) == _lib.ERR_INVALID_ARG


def test_peer_exchange_validation_without_device():
    """q35_cp_* refuse bad shapes and NULL handles before touching a device;
    a valid request then fails on the missing GPU, never in an allocation."""
    lib = q35attn.load()
    ctx, h = C.c_void_p(), (C.c_ubyte * 64)()
    assert lib.q35_cp_create(0, 0, 1, 256, 8, 256, C.byref(ctx), h) == _lib.ERR_INVALID_ARG   # world 0
    assert lib.q35_cp_create(9, 0, 1, 256, 8, 256, C.byref(ctx), h) == _lib.ERR_INVALID_ARG   # world > 8
    assert lib.q35_cp_create(2, 2, 1, 256, 8, 256, C.byref(ctx), h) == _lib.ERR_INVALID_ARG   # rank >= world
    assert lib.q35_cp_create(2, 0, 0, 256, 8, 256, C.byref(ctx), h) == _lib.ERR_INVALID_ARG   # no sequence
    assert lib.q35_cp_create(2, 0, 1, 256, 8, 128, C.byref(ctx), h) == _lib.ERR_UNSUPPORTED   # head_dim
    assert lib.q35_cp_create(2, 0, 1, 255, 8, 256, C.byref(ctx), h) == _lib.ERR_UNSUPPORTED   # odd n_gdn
    assert lib.q35_cp_create(2, 0, 1, 256, 8, 256, None, h) == _lib.ERR_INVALID_ARG
    import torch
    rc = lib.q35_cp_create(2, 0, 1, 256, 8, 256, C.byref(ctx), h)
    if torch.cuda.is_available():
        assert rc == _lib.OK and lib.q35_cp_destroy(ctx) == _lib.OK
    else:
        assert rc == _lib.ERR_DEVICE  # the shape is valid; the device check comes last
    assert lib.q35_cp_exchange(None, *([None] * 5), None) == _lib.ERR_INVALID_ARG
    assert lib.q35_cp_connect(None, h) == _lib.ERR_INVALID_ARG
    assert lib.q35_cp_disconnect(None) == _lib.ERR_INVALID_ARG
    assert lib.q35_cp_destroy(None) == _lib.OK


def test_workspace_sizes_are_positive_and_monotone():
    lib = q35attn.load()
    g = _lib.GqaDims(256, 8, 2, 256, 64, 0, 40000, 1e-6)
    a = lib.q35_gqa_decode_workspace_size(C.byref(g), 4097)
    b = lib.q35_gqa_decode_workspace_size(C.byref(g), 32769)
    assert 0 < a <= b
    d = _lib.GdnDims(1, 16, 16, 128, 128, 4, 1e-6)
    # per (head, chunk): U, W^T, k', q' [64x128] + Aqk [64x64] + decay slot (64) + S_c^T [128x128] + v'^T [128x64]
    rec = 4 * 64 * 128 + 64 * 64 + 64 + 128 * 128 + 128 * 64
    assert lib.q35_gdn_prefill_workspace_size(C.byref(d), 8192) == 256 + 16 * 128 * rec * 4  # status header
    assert lib.q35_gdn_prefill_workspace_size(C.byref(d), 0) == 0


def test_python_wrappers_refuse_cpu_tensors():
    import torch
    x = torch.zeros(1, 6144)
    with pytest.raises(ValueError):
        q35attn.gdn_decode(x, torch.zeros(1, 2048), torch.zeros(1, 16), torch.zeros(1, 16), torch.zeros(6144, 4),
                           torch.ones(128), torch.zeros(1, 6144, 3), torch.zeros(1, 16, 128, 128),
                           out=torch.zeros(1, 2048), num_k_heads=16, num_v_heads=16)


def test_fused_gemv_validation_without_device():
    lib = q35attn.load()
    seg = (_lib.Q8Segment * 2)()
    for k in range(2):
        seg[k].w, seg[k].scales, seg[k].y, seg[k].out_dim = 4096, 8192, 12288, 256
    call = lambda n, x=1 << 20, res=None, nw=None, so=None, xo=None, sw=0, mode=0, ind=256: lib.q35_q8_gemv_fused(
        ind, n, seg, x, res, nw, 1e-6, so, xo, sw, mode, None)
    assert call(0) == _lib.ERR_INVALID_ARG           # no segment
    assert call(5) == _lib.ERR_INVALID_ARG           # more than four
    assert call(2, x=(1 << 20) + 4) == _lib.ERR_INVALID_ARG  # x not 16-byte aligned
    assert call(1, sw=1) == _lib.ERR_INVALID_ARG     # swiglu needs (up, gate)
    assert call(2, res=1 << 21) == _lib.ERR_INVALID_ARG  # residual without norm_w
    assert call(2, nw=1 << 21, so=1 << 20) == _lib.ERR_INVALID_ARG  # sum_out aliases x
    assert call(2, ind=254) == _lib.ERR_UNSUPPORTED  # in_dim % 4
    assert call(2, nw=1 << 21, ind=8196) == _lib.ERR_UNSUPPORTED  # too long for the norm's shared memory
    seg[1].out_dim = 320
    assert call(2) == _lib.ERR_UNSUPPORTED           # out_dim % 256
    seg[1].out_dim = 256
    assert call(2, mode=2) == _lib.ERR_INVALID_ARG
