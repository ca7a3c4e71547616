"""The C ABI library builds, loads and exports every symbol include/*.h declares
(CPU only: no compute call is made)."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from nesle_b200 import _lib, build

ROOT = Path(__file__).resolve().parents[1]


def declared_functions() -> set[str]:
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(nesle_[a-z0-9_]+)\s*\(", text))
    return names


@pytest.fixture(scope="module")
def lib_path() -> Path:
    return build.build()


def test_header_declares_the_boundary():
    names = declared_functions()
    assert {"nesle_create", "nesle_destroy", "nesle_step", "nesle_reset", "nesle_reset_envs", "nesle_render",
            "nesle_device_ptr", "nesle_last_error"} <= names


def test_library_exports_every_declared_symbol(lib_path):
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib_path)], capture_output=True, text=True, check=True)
    exported = set(re.findall(r"\bT (nesle_[a-z0-9_]+)", out.stdout))
    missing = declared_functions() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_ctypes_binding_covers_the_header(lib_path):
    assert declared_functions() == set(_lib.SIGNATURES)
    lib = _lib.load()
    for name in _lib.SIGNATURES:
        assert isinstance(getattr(lib, name), ctypes._CFuncPtr)
    assert lib.nesle_abi_version() == 2


def test_cpu_only_entry_points(lib_path):
    """parse_fcs and argument validation need no GPU."""
    from nesle_b200 import workloads as w
    from nesle_b200._cuda_core import parse_fcs_state

    s = w.random_snapshot(3, 0x8123)
    d = parse_fcs_state(w.write_fcs(s))
    assert (d["pc"], d["a"], d["x"]) == (0x8123, s.a, s.x) and d["cpu_ram"] == s.cpu_ram
    with pytest.raises(ValueError, match="bad magic"):
        parse_fcs_state(b"XXXX" + w.write_fcs(s)[4:])
    with pytest.raises(ValueError):
        parse_fcs_state(w.write_fcs(s)[:32])
    lib = _lib.load()
    h = ctypes.c_void_p()
    args, keep = _lib.make_create_args(0, 4, w.config1().rom.image)
    assert lib.nesle_create(ctypes.byref(args), ctypes.byref(h)) == _lib.NESLE_ERR_INVALID
    assert b"num_envs must be positive" in lib.nesle_last_error()
    args, keep = _lib.make_create_args(4, 4, b"NES\x1a" + bytes(12))
    assert lib.nesle_create(ctypes.byref(args), ctypes.byref(h)) == _lib.NESLE_ERR_INVALID
    assert b"NROM" in lib.nesle_last_error()


def test_state_blob_layout_matches_the_library(lib_path):
    lib = _lib.load()
    assert lib.nesle_state_bytes() == _lib.STATE_BYTES
    end = 0
    for name, (off, size) in _lib.STATE_PARTS.items():
        assert off == end and off % 16 == 0, name  # consecutive, 16-byte aligned
        end = off + size
    assert end == _lib.STATE_BYTES and _lib.ENV_RECORD_DTYPE.itemsize == 128



def test_integration_cpp_stub_compiles():
    """The C++ host loop quoted in the integration guide
    (tests/native/integration_stub.cpp) type-checks against include/nesle_b200.h."""
    import shutil
    from pathlib import Path

    gxx = shutil.which("g++")
    cuda_inc = Path("/usr/local/cuda/include")
    if not gxx or not (cuda_inc / "cuda_runtime.h").exists():
        pytest.skip("g++ or the CUDA headers are not available")
    root = Path(__file__).resolve().parents[1]
    r = subprocess.run([gxx, "-std=c++17", "-fsyntax-only", "-I", str(root / "include"), "-I", str(cuda_inc),
                        str(root / "tests" / "native" / "integration_stub.cpp")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
