"""Runs the C++ host layer's parity driver (tests/host/q35_host_parity.cpp) on
the GPU: GatedDeltaNetCore and AttentionCore driven through a Cache as the
reference's modules are (prompt, decode steps, a further prompt on the cached
state, cache: None), each output and the cached states against the CPU oracle
within max rel err 1e-3, plus the error behaviour (capacity, bad arguments)."""
import subprocess

import pytest

from q35attn import _lib
from test_host_cpp import build_driver

pytestmark = pytest.mark.gpu


def test_host_layer_parity(tmp_path):
    _lib.load()
    exe = build_driver(tmp_path / "q35_host_parity")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all checks passed" in r.stdout
