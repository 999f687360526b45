"""The C ABI library loads and exports what include/*.h declares (CPU only),
and the host-side validation mirrors the reference's (needle2/native.py:172-276)."""
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
    ref = Path("/root/reference")
    if not (ref / "needle2" / "native.py").is_file():
        pytest.skip("reference sources unavailable")
    code = ("import needle2.native as n; lib = n._library(); "
            "print(n.features()); print(n.sdot_available())")
    env = dict(os.environ, NEEDLE2_NATIVE_LIBRARY=str(lib_path), PYTHONPATH=str(ref))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, cwd=tmp_path)
    assert out.returncode == 0, out.stderr
    assert "cuda-sm100a" in out.stdout and "True" in out.stdout


def test_host_validation_mirrors_reference():
    from openneedle_b200.native import NativeCQ
    packed, norms, shape, cb, _ = example(2)
    with pytest.raises(ValueError, match="positive two-dimensional"):
        NativeCQ(packed, norms, (0, 257), 2, 128, cb)
    with pytest.raises(ValueError, match="storage bits"):
        NativeCQ(packed, norms, shape, 6, 128, cb)
    with pytest.raises(ValueError, match="power of two"):
        NativeCQ(packed, norms, shape, 2, 96, cb)
    for value in (-1.0, np.inf, np.nan):
        bad = norms.copy()
        bad[0, 0] = value
        with pytest.raises(ValueError, match="norms must be finite and nonnegative"):
            NativeCQ(packed, bad, shape, 2, 128, cb)
    for codebook in ([np.nan, 0, 1, 2], [-2, -1, 0, np.inf], [2, 1, 0, -1], [0, 0, 1, 2]):
        with pytest.raises(ValueError, match="codebook must be finite and strictly sorted"):
            NativeCQ(packed, norms, shape, 2, 128, codebook)
    with pytest.raises(ValueError, match="incorrect number of centroids"):
        NativeCQ(packed, norms, shape, 2, 128, cb[:3])
    tern, tn, ts, tcb, _ = example(5)
    bad = tern.copy()
    bad[0, 0] = 0b10
    with pytest.raises(ValueError, match="ternary crumb code 2"):
        NativeCQ(bad, tn, ts, 5, 128, tcb)


def test_create_fails_loudly_without_gpu():
    """No silent CPU fallback: on a machine without a GPU, construction raises."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from openneedle_b200.native import NativeCQ
    packed, norms, shape, cb, _ = example(4)
    with pytest.raises(MemoryError, match="Could not construct native CQ matrix"):
        NativeCQ(packed, norms, shape, 4, 128, cb)
