"""CPU ORACLE bindings — test infrastructure only.

ctypes access to two checker libraries built by ``oracle/Makefile``:

* ``_build/liboracle.so``: the plain-C restatement of OpenNeedle's CPU arithmetic
  (``cq_oracle.c``), the checker for every CUDA kernel;
* ``_ref/libneedle2_ref.so``: OpenNeedle's own CPU sources compiled unchanged plus
  ``ref_shim.cpp`` — used to pin the restatement and as bench.py's reference arm.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import
this module.  The product (``openneedle_b200``) never does.
"""
from __future__ import annotations

import ctypes as ct
import functools
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "_build" / "liboracle.so"
REF_LIB = HERE / "_ref" / "libneedle2_ref.so"
# Root of the reference project (the directory that holds needle2/):
# NEEDLE2_REFERENCE_SRC when set, else the copy that pip installed into
# baseline/_ref (git-ignored, it travels with the working tree).  Its
# needle2/csrc holds the C++ sources that `make ref` compiles, its needle2/ the
# Python (quantizer, NativeCQ/NativeEngine) that tests drive.
REF_ROOT = Path(os.environ.get("NEEDLE2_REFERENCE_SRC", str(HERE.parent / "baseline" / "_ref")))
REF_SRC = REF_ROOT / "needle2" / "csrc"


def reference_package():
    """The reference's own Python package root on sys.path, or None when absent."""
    import sys
    if not (REF_ROOT / "needle2" / "__init__.py").is_file():
        return None
    if str(REF_ROOT) not in sys.path:
        sys.path.insert(0, str(REF_ROOT))
    return REF_ROOT

_p = ct.c_void_p
_i = ct.c_int


def build(reference: bool | None = None) -> None:
    """Compile the restatement, and the reference shim when its sources exist."""
    targets = ["oracle"]
    if reference or (reference is None and (REF_SRC / "cq.cpp").is_file()):
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", str(HERE), f"REF_SRC={REF_SRC}", *targets], check=True)


@functools.lru_cache(maxsize=1)
def lib() -> ct.CDLL:
    if not ORACLE_LIB.is_file():
        build(reference=False)
    L = ct.CDLL(str(ORACLE_LIB))
    L.oracle_half_to_float.argtypes = [ct.c_uint16]
    L.oracle_half_to_float.restype = ct.c_float
    L.oracle_fwht.argtypes = [_p, _i]
    L.oracle_cq_transform.argtypes = [_p, _p, _i, _i]
    L.oracle_cq_linear.argtypes = [_p, _p, _i, _i, _i, _i, _p, _p, _p, _i]
    L.oracle_cq_rows.argtypes = [_p, _p, _i, _i, _i, _i, _p, _p, _p, _i]
    L.oracle_sdot_centroids.argtypes = [_p, _i, _p, _p]
    L.oracle_sdot_prepare.argtypes = [_p, _i, _i, _i, _p, _p]
    L.oracle_sdot_partials.argtypes = [_p, _i, _i, _i, _i, _p, _p, _i, _p]
    L.oracle_sdot_linear.argtypes = [_p, _p, _i, _i, _i, _i, _p, _p, _p, _i, _p, _p, _p]
    L.oracle_activation_quant.argtypes = [_p, _i, _i]
    L.oracle_argmax.argtypes = [_p, _i]
    L.oracle_argmax.restype = _i
    L.oracle_kv_quantize.argtypes = [_p, _p, _i, _i, _p, _p, _p, _p]
    L.oracle_cache_slot.argtypes = [_i, _i, _i]
    L.oracle_cache_slot.restype = _i
    L.oracle_attention_slots.argtypes = [_i, _i, _i, _p]
    L.oracle_attention_slots.restype = _i
    L.oracle_attention_i8.argtypes = [_p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _p, _p]
    L.oracle_attention_prefill_i8.argtypes = [_p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _p, _p, _p, _p]
    return L


def ref_available() -> bool:
    return REF_LIB.is_file()


@functools.lru_cache(maxsize=1)
def ref_lib() -> ct.CDLL:
    if not REF_LIB.is_file():
        raise FileNotFoundError(f"reference build missing: {REF_LIB} (run make -C oracle ref)")
    L = ct.CDLL(str(REF_LIB))
    L.needle2_cq_create.argtypes = [_p, _p, _i, _i, _i, _i, _p]
    L.needle2_cq_create.restype = _p
    L.needle2_cq_destroy.argtypes = [_p]
    L.needle2_cq_linear.argtypes = [_p, _p, _p, _i, _i]
    L.needle2_cq_rows.argtypes = [_p, _p, _p, _i]
    L.ref_sdot_prepare.argtypes = [_p, _p, _i, _i, _i, _i, _p, _p, _i, _p, _p]
    L.ref_sdot_centroids.argtypes = [_p, _p, _i, _i, _i, _i, _p, _p, _p, _p]
    L.ref_sdot_partials.argtypes = [_p, _p, _i, _i, _i, _i, _p, _p, _i, _p]
    L.ref_sdot_linear.argtypes = [_p, _p, _i, _i, _i, _i, _p, _p, _p, _i, _i]
    L.ref_sdot_new.argtypes = [_p, _p, _i, _i, _i, _i, _p]
    L.ref_sdot_new.restype = _p
    L.ref_sdot_run.argtypes = [_p, _p, _p, _i, _i]
    L.ref_sdot_free.argtypes = [_p]
    L.ref_kv_import.argtypes = [_i, _i, _i, _i, _i, _i, _p, _i, _p, _p, _p, _p, _p, _p]
    L.ref_kv_import.restype = _i
    L.ref_attention_i8.argtypes = [_i, _i, _i, _i, _i, _i, _p, _p, _p, _p, _i, _p, _p]
    return L


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def padded(dim: int, group: int) -> int:
    return (dim + group - 1) // group * group


# ---------------------------------------------------------------- restatement

def fwht(v):
    v = _c(v, np.float32).copy()
    lib().oracle_fwht(v.ctypes.data, v.size)
    return v


def cq_linear(packed, norms, shape, bits, group, cb, x):
    out, dim = shape
    packed, norms, cb = _c(packed, np.uint8), _c(norms, np.float16), _c(cb, np.float32)
    x = _c(x, np.float32)
    batch = x.size // dim
    y = np.empty(x.shape[:-1] + (out,), np.float32)
    lib().oracle_cq_linear(packed.ctypes.data, norms.ctypes.data, out, dim, bits, group,
                           cb.ctypes.data, x.ctypes.data, y.ctypes.data, batch)
    return y


def cq_rows(packed, norms, shape, bits, group, cb, ids):
    out, dim = shape
    ids = _c(ids, np.int64)
    packed, norms, cb = _c(packed, np.uint8), _c(norms, np.float16), _c(cb, np.float32)
    y = np.empty(ids.shape + (dim,), np.float32)
    lib().oracle_cq_rows(packed.ctypes.data, norms.ctypes.data, out, dim, bits, group,
                         cb.ctypes.data, ids.ctypes.data, y.ctypes.data, ids.size)
    return y


def sdot_centroids(cb, bits):
    cb = _c(cb, np.float32)
    c = np.zeros(16, np.int8)
    s = np.zeros(1, np.float32)
    lib().oracle_sdot_centroids(cb.ctypes.data, bits, c.ctypes.data, s.ctypes.data)
    return c, float(s[0])


def sdot_prepare(x, group):
    x = _c(x, np.float32)
    x2 = x.reshape(-1, x.shape[-1])
    rows, dim = x2.shape
    pad = padded(dim, group)
    q = np.empty((rows, pad), np.int8)
    s = np.empty((rows, pad // group), np.float32)
    lib().oracle_sdot_prepare(x2.ctypes.data, rows, dim, group, q.ctypes.data, s.ctypes.data)
    return q, s


def sdot_linear(packed, norms, shape, bits, group, cb, x):
    """Returns (y [rows,out], partials [rows,out,groups] int32, q, scales)."""
    out, dim = shape
    packed, norms, cb = _c(packed, np.uint8), _c(norms, np.float16), _c(cb, np.float32)
    x2 = _c(x, np.float32).reshape(-1, dim)
    rows = x2.shape[0]
    pad = padded(dim, group)
    groups = pad // group
    y = np.empty((rows, out), np.float32)
    d = np.empty((rows, out, groups), np.int32)
    q = np.empty((rows, pad), np.int8)
    s = np.empty((rows, groups), np.float32)
    lib().oracle_sdot_linear(packed.ctypes.data, norms.ctypes.data, out, dim, bits, group, cb.ctypes.data,
                             x2.ctypes.data, y.ctypes.data, rows, d.ctypes.data, q.ctypes.data, s.ctypes.data)
    return y, d, q, s


def activation_quant(x, bits=8):
    x = _c(x, np.float32).copy()
    lib().oracle_activation_quant(x.ctypes.data, x.size, bits)
    return x


def argmax(x):
    """Greedy token of each row of x (first maximum wins, NaNs never win)."""
    x = _c(x, np.float32)
    rows = x.reshape(-1, x.shape[-1])
    return np.array([lib().oracle_argmax(r.ctypes.data, r.size) for r in rows], np.int32)


def kv_quantize(k, v, kvheads, head_dim):
    """k, v: [tokens][kvheads*head_dim] -> (k_i8, v_i8, k_scale, v_scale)."""
    k, v = _c(k, np.float32).reshape(-1, kvheads * head_dim), _c(v, np.float32).reshape(-1, kvheads * head_dim)
    n = k.shape[0]
    ki, vi = np.empty((n, kvheads * head_dim), np.int8), np.empty((n, kvheads * head_dim), np.int8)
    ks, vs = np.empty((n, kvheads), np.float32), np.empty((n, kvheads), np.float32)
    for t in range(n):
        lib().oracle_kv_quantize(k[t].ctypes.data, v[t].ctypes.data, kvheads, head_dim,
                                 ki[t].ctypes.data, vi[t].ctypes.data, ks[t].ctypes.data, vs[t].ctypes.data)
    return ki, vi, ks, vs


def cache_slot(pos, prefix, window):
    return lib().oracle_cache_slot(pos, prefix, window)


def attention_i8(keys_i8, values_i8, k_scales, v_scales, heads, kvheads, head_dim, pos, prefix, window, q):
    """Cache arrays [capacity][kvheads*head_dim] / [capacity][kvheads]; q [heads*head_dim]."""
    ki, vi = _c(keys_i8, np.int8), _c(values_i8, np.int8)
    ks, vs = _c(k_scales, np.float32), _c(v_scales, np.float32)
    q = _c(q, np.float32)
    out = np.empty(heads * head_dim, np.float32)
    lib().oracle_attention_i8(ki.ctypes.data, vi.ctypes.data, ks.ctypes.data, vs.ctypes.data, heads, kvheads,
                              head_dim, pos, prefix, window, q.ctypes.data, out.ctypes.data)
    return out


def attention_prefill_i8(cache, heads, kvheads, head_dim, start_pos, prefix, window, q, k, v):
    """cache = dict of writable arrays keys_i8/values_i8/k_scales/v_scales (updated in place)."""
    q, k, v = _c(q, np.float32), _c(k, np.float32), _c(v, np.float32)
    count = q.size // (heads * head_dim)
    out = np.empty((count, heads * head_dim), np.float32)
    for name, dt in (("keys_i8", np.int8), ("values_i8", np.int8), ("k_scales", np.float32), ("v_scales", np.float32)):
        assert cache[name].dtype == dt and cache[name].flags.c_contiguous
    lib().oracle_attention_prefill_i8(cache["keys_i8"].ctypes.data, cache["values_i8"].ctypes.data,
                                      cache["k_scales"].ctypes.data, cache["v_scales"].ctypes.data,
                                      heads, kvheads, head_dim, start_pos, count, prefix, window,
                                      q.ctypes.data, k.ctypes.data, v.ctypes.data, out.ctypes.data)
    return out


# ------------------------------------------------------- reference (compiled)

def ref_cq_linear(packed, norms, shape, bits, group, cb, x, threads=1):
    out, dim = shape
    packed, norms, cb = _c(packed, np.uint8), _c(norms, np.float16), _c(cb, np.float32)
    x = _c(x, np.float32)
    L = ref_lib()
    h = L.needle2_cq_create(packed.ctypes.data, norms.ctypes.data, out, dim, bits, group, cb.ctypes.data)
    try:
        y = np.empty(x.shape[:-1] + (out,), np.float32)
        L.needle2_cq_linear(h, x.ctypes.data, y.ctypes.data, x.size // dim, threads)
    finally:
        L.needle2_cq_destroy(h)
    return y


def ref_cq_rows(packed, norms, shape, bits, group, cb, ids):
    out, dim = shape
    packed, norms, cb = _c(packed, np.uint8), _c(norms, np.float16), _c(cb, np.float32)
    ids = _c(ids, np.int64)
    L = ref_lib()
    h = L.needle2_cq_create(packed.ctypes.data, norms.ctypes.data, out, dim, bits, group, cb.ctypes.data)
    try:
        y = np.empty(ids.shape + (dim,), np.float32)
        L.needle2_cq_rows(h, ids.ctypes.data, y.ctypes.data, ids.size)
    finally:
        L.needle2_cq_destroy(h)
    return y


def sdot_unpermute(qperm, bits, group):
    """Undo the reference's bit-plane order (needle2/csrc/sdot.cpp:99-100)."""
    width = 4 if bits == 2 else 2
    chunk = width * 16
    pad = qperm.shape[-1]
    i = np.arange(pad)
    gi = i % group
    dest = (i - gi) + (gi // chunk) * chunk + (gi % width) * 16 + (gi % chunk) // width
    return qperm[..., dest]


def ref_sdot(packed, norms, shape, bits, group, cb, x, threads=1):
    """Reference SdotCQ: returns (y, partials, q in natural order, scales)."""
    out, dim = shape
    packed, norms, cb = _c(packed, np.uint8), _c(norms, np.float16), _c(cb, np.float32)
    x2 = _c(x, np.float32).reshape(-1, dim)
    rows = x2.shape[0]
    pad = padded(dim, group)
    groups = pad // group
    L = ref_lib()
    q = np.empty((rows, pad), np.int8)
    s = np.empty((rows, groups), np.float32)
    L.ref_sdot_prepare(packed.ctypes.data, norms.ctypes.data, out, dim, bits, group, cb.ctypes.data,
                       x2.ctypes.data, rows, q.ctypes.data, s.ctypes.data)
    d = np.empty((rows, out, groups), np.int32)
    L.ref_sdot_partials(packed.ctypes.data, norms.ctypes.data, out, dim, bits, group, cb.ctypes.data,
                        x2.ctypes.data, rows, d.ctypes.data)
    y = np.empty((rows, out), np.float32)
    L.ref_sdot_linear(packed.ctypes.data, norms.ctypes.data, out, dim, bits, group, cb.ctypes.data,
                      x2.ctypes.data, y.ctypes.data, rows, threads)
    return y, d, sdot_unpermute(q, bits, group), s


def ref_kv_import(heads, kvheads, head_dim, max_seq, window, prefix, positions, k, v):
    positions = _c(positions, np.int32)
    k, v = _c(k, np.float32), _c(v, np.float32)
    cap = window + prefix if window else max_seq
    K = kvheads * head_dim
    ki, vi = np.zeros((cap, K), np.int8), np.zeros((cap, K), np.int8)
    ks, vs = np.zeros((cap, kvheads), np.float32), np.zeros((cap, kvheads), np.float32)
    got = ref_lib().ref_kv_import(heads, kvheads, head_dim, max_seq, window, prefix, positions.ctypes.data,
                                  positions.size, k.ctypes.data, v.ctypes.data, ki.ctypes.data, vi.ctypes.data,
                                  ks.ctypes.data, vs.ctypes.data)
    assert got == cap
    return ki, vi, ks, vs


def ref_attention_i8(heads, kvheads, head_dim, max_seq, window, prefix, ki, vi, ks, vs, pos, q):
    ki, vi, ks, vs = _c(ki, np.int8), _c(vi, np.int8), _c(ks, np.float32), _c(vs, np.float32)
    q = _c(q, np.float32)
    out = np.empty(heads * head_dim, np.float32)
    ref_lib().ref_attention_i8(heads, kvheads, head_dim, max_seq, window, prefix, ki.ctypes.data, vi.ctypes.data,
                               ks.ctypes.data, vs.ctypes.data, pos, q.ctypes.data, out.ctypes.data)
    return out
