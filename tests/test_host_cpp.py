"""The C++ host layer (qwen-3.5_b200/host/q35_modules.hpp): the library exports
it, and its parity driver (tests/host/q35_host_parity.cpp) compiles against the
headers.  The driver itself runs in tests/test_host_cpp_gpu.py."""
import os
import subprocess

from q35attn import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def build_driver(out_path):
    import oracle
    oracle.build()
    lib_dir = os.path.dirname(_lib.LIB_PATH)
    orc_dir = os.path.join(ROOT, "oracle", "_build")
    cmd = ["g++", "-std=c++17", "-O2", "-Wall", os.path.join(ROOT, "tests", "host", "q35_host_parity.cpp"),
           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "qwen-3.5_b200", "host"),
           "-I", os.path.join(ROOT, "oracle"), "-I", "/usr/local/cuda/include",
           "-L", lib_dir, "-lq35attn", "-L", orc_dir, "-lq35oracle", "-L", "/usr/local/cuda/lib64", "-lcudart",
           f"-Wl,-rpath,{lib_dir}:{orc_dir}", "-o", str(out_path)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    return out_path


def test_library_exports_the_host_layer():
    _lib.load()
    out = subprocess.run(["nm", "-DC", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True, check=True)
    for sym in ("q35::host::Cache::Cache(", "q35::host::GatedDeltaNetCore::forward(",
                "q35::host::AttentionCore::forward(", "q35::host::AttentionCore::check_status("):
        assert sym in out.stdout, sym


def test_parity_driver_compiles(tmp_path):
    _lib.load()
    assert os.path.exists(build_driver(tmp_path / "q35_host_parity"))
