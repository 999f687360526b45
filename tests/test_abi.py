"""The C ABI library loads and exports what include/*.h declares, the
reference's Python binds it, and its creates validate their arguments (CPU only)."""
import ctypes as ct
import os
import re
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from util import example

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names.update(re.findall(r"\b(needle2_\w+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def lib_path():
    from openneedle_b200 import build
    return build.build()


def test_library_exports_every_declared_symbol(lib_path):
    names = declared_functions()
    assert len(names) >= 18
    exported = subprocess.run(["nm", "-D", "--defined-only", str(lib_path)], capture_output=True, text=True,
                              check=True).stdout
    missing = [n for n in names if not re.search(rf"\bT {n}\b", exported)]
    assert not missing, missing
    lib = ct.CDLL(str(lib_path))
    for n in names:
        assert getattr(lib, n)


def test_library_is_self_contained(lib_path):
    deps = subprocess.run(["ldd", str(lib_path)], capture_output=True, text=True).stdout
    assert "libtorch" not in deps and "libc10" not in deps and "libcudart.so" not in deps


def test_features_and_sdot_flag_without_gpu(lib_path):
    lib = ct.CDLL(str(lib_path))
    lib.needle2_native_features.restype = ct.c_char_p
    assert b"cuda-sm100a" in lib.needle2_native_features()
    assert lib.needle2_sdot_supported() == 1


def test_reference_binding_accepts_library(lib_path, tmp_path):
    """OpenNeedle's own ctypes layer binds this library via NEEDLE2_NATIVE_LIBRARY."""
    from oracle import oracle as O
    if O.reference_package() is None:
        pytest.skip(f"reference package unavailable under {O.REF_ROOT}")
    code = ("import needle2.native as n; lib = n._library(); "
            "print(n.features()); print(n.sdot_available())")
    env = dict(os.environ, NEEDLE2_NATIVE_LIBRARY=str(lib_path), PYTHONPATH=str(O.REF_ROOT))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, cwd=tmp_path)
    assert out.returncode == 0, out.stderr
    assert "cuda-sm100a" in out.stdout and "True" in out.stdout


def test_create_validates_arguments_before_touching_the_gpu(lib_path):
    """The C ABI's create calls reject bad geometry with NULL and a message of
    their own (the reference's creates have no error channel; its Python
    checks first, needle2/native.py:172-208)."""
    lib = ct.CDLL(str(lib_path))
    lib.needle2_b200_error.restype = ct.c_char_p
    for name in ("needle2_cq_create", "needle2_sdot_create"):
        getattr(lib, name).argtypes = [ct.c_void_p, ct.c_void_p, ct.c_int, ct.c_int, ct.c_int, ct.c_int, ct.c_void_p]
        getattr(lib, name).restype = ct.c_void_p
    packed, norms, shape, cb, _ = example(2)
    p, n, c = packed.ctypes.data, norms.ctypes.data, cb.ctypes.data
    cases = [("needle2_cq_create", (p, n, 0, 257, 2, 128, c), "positive two-dimensional"),
             ("needle2_cq_create", (p, n, 9, 257, 6, 128, c), "storage bits"),
             ("needle2_cq_create", (p, n, 9, 257, 2, 96, c), "power of two"),
             ("needle2_cq_create", (None, n, 9, 257, 2, 128, c), "null"),
             ("needle2_sdot_create", (p, n, 9, 257, 3, 128, c), "SDOT requires CQ2/CQ4"),
             ("needle2_sdot_create", (p, n, 9, 257, 2, 32, c), "SDOT requires CQ2/CQ4")]
    for name, args, message in cases:
        assert getattr(lib, name)(*args) is None
        assert message in lib.needle2_b200_error().decode()


def test_create_fails_loudly_without_gpu():
    """No silent CPU fallback: on a machine without a GPU, construction raises."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from openneedle_b200.native import DeviceMatrix
    packed, norms, shape, cb, _ = example(4)
    m = DeviceMatrix(packed, norms, shape, 4, 128, cb)
    with pytest.raises(RuntimeError, match="needle2_cq_create"):
        m.fp32(np.zeros(shape[1], np.float32))
    with pytest.raises(RuntimeError, match="needle2_sdot_create"):
        m.sdot(np.zeros(shape[1], np.float32))
