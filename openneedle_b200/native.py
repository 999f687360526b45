"""ctypes access to libneedle2_b200.so, mirroring OpenNeedle's ``needle2/native.py``.

``NativeCQ`` keeps the reference class's constructor, validation messages,
``linear``/``linear_sdot``/``rows``/``dequantize`` methods and error types
(needle2/native.py:165-279), so code written against the reference runs on
the GPU unchanged.  The compute runs in CUDA kernels only: when the library or
a GPU is missing, calls raise instead of falling back to any CPU path.
"""
from __future__ import annotations

import ctypes as ct
import functools
import os
from pathlib import Path

import numpy as np

from . import build as _build

_p = ct.c_void_p
_i = ct.c_int


def library_path() -> Path:
    override = os.environ.get("NEEDLE2_B200_LIBRARY")
    return Path(override).resolve() if override else _build.LIB


@functools.lru_cache(maxsize=1)
def _library() -> ct.CDLL:
    path = library_path()
    if not path.is_file():
        raise RuntimeError(f"libneedle2_b200.so not built ({path}); run python -m openneedle_b200.build")
    lib = ct.CDLL(str(path))
    lib.needle2_native_features.restype = ct.c_char_p
    lib.needle2_b200_error.restype = ct.c_char_p
    for name in ("needle2_cq_create", "needle2_sdot_create"):
        getattr(lib, name).argtypes = [_p, _p, _i, _i, _i, _i, _p]
        getattr(lib, name).restype = _p
    for name in ("needle2_cq_destroy", "needle2_sdot_destroy"):
        getattr(lib, name).argtypes = [_p]
        getattr(lib, name).restype = None
    for name in ("needle2_cq_linear", "needle2_sdot_linear"):
        getattr(lib, name).argtypes = [_p, _p, _p, _i, _i]
        getattr(lib, name).restype = None
    for name in ("needle2_cq_linear_checked", "needle2_sdot_linear_checked"):
        getattr(lib, name).argtypes = [_p, _p, _p, _i]
        getattr(lib, name).restype = _i
    for name in ("needle2_cq_linear_device", "needle2_sdot_linear_device"):
        getattr(lib, name).argtypes = [_p, _p, _p, _i, _p]
        getattr(lib, name).restype = _i
    for name in ("needle2_cq_prepare_device", "needle2_sdot_prepare_device"):
        getattr(lib, name).argtypes = [_p, _p, _i, _p]
        getattr(lib, name).restype = _i
    for name in ("needle2_cq_multiply_device", "needle2_sdot_multiply_device"):
        getattr(lib, name).argtypes = [_p, _p, _i, _p]
        getattr(lib, name).restype = _i
    lib.needle2_b200_set_int8_gemv.argtypes = [_i]
    lib.needle2_b200_set_int8_gemv.restype = _i
    lib.needle2_b200_set_f32_gemv.argtypes = [_i]
    lib.needle2_b200_set_f32_gemv.restype = _i
    lib.needle2_cq_linear_many_checked.argtypes = [ct.POINTER(_p), _i, _p, ct.POINTER(_p), _i, _i]
    lib.needle2_cq_linear_many_checked.restype = _i
    lib.needle2_cq_linear_many_device.argtypes = [ct.POINTER(_p), _i, _p, ct.POINTER(_p), _i, _i, _p]
    lib.needle2_cq_linear_many_device.restype = _i
    lib.needle2_cq_multiply_many_device.argtypes = [ct.POINTER(_p), _i, ct.POINTER(_p), _i, _i, _p]
    lib.needle2_cq_multiply_many_device.restype = _i
    lib.needle2_b200_device_fault.restype = _i
    lib.needle2_cq_linear_lookup.argtypes = [_p, _p, _p, _i, _i, _i]
    lib.needle2_cq_linear_lookup.restype = None
    lib.needle2_cq_linear_many.argtypes = [ct.POINTER(_p), _i, _p, ct.POINTER(_p), _i, _i]
    lib.needle2_cq_linear_many.restype = None
    lib.needle2_cq_rows.argtypes = [_p, _p, _p, _i]
    lib.needle2_cq_rows.restype = None
    lib.needle2_sdot_supported.restype = _i
    lib.needle2_sdot_debug.argtypes = [_p, _p, _i, _p, _p, _p, _p]
    lib.needle2_sdot_debug.restype = _i
    lib.needle2_cq_geometry.argtypes = [_p, ct.POINTER(_i)]
    lib.needle2_cq_geometry.restype = _i
    return lib


def available() -> bool:
    try:
        _library()
        return True
    except (OSError, RuntimeError):
        return False


def features() -> str:
    return _library().needle2_native_features().decode()


def sdot_available() -> bool:
    return bool(_library().needle2_sdot_supported())


def last_error() -> str:
    return _library().needle2_b200_error().decode()


def _check(status: int, what: str) -> None:
    if status:
        raise RuntimeError(f"{what}: {last_error()}")


def _check_void(what: str) -> None:
    msg = last_error()
    if msg:
        raise RuntimeError(f"{what}: {msg}")


def _stream_ptr(stream) -> int | None:
    if stream is None:
        return None
    return int(getattr(stream, "cuda_stream", stream))


class NativeCQ:
    """A packed ``[out, in]`` matrix held in device memory.

    The codebook must already include ``1/sqrt(group_size)`` as in a CACT header.
    ``bits=5`` denotes signed ternary crumb storage with 3 centroids.
    """

    def __init__(self, packed, norms, shape, bits, group_size, codebook):
        self.shape = tuple(int(v) for v in shape)
        if len(self.shape) != 2 or min(self.shape) <= 0:
            raise ValueError("NativeCQ requires a positive two-dimensional matrix shape")
        self.bits, self.group_size = int(bits), int(group_size)
        if self.bits not in (2, 3, 4, 5):
            raise ValueError("CQ storage bits must be 2, 3, 4, or ternary marker 5")
        if self.group_size < 8 or self.group_size & (self.group_size - 1):
            raise ValueError("CQ group size must be a power of two >= 8")
        out, dim = self.shape
        limit = np.iinfo(np.int32).max
        if max(out, dim, self.group_size) > limit or dim + self.group_size - 1 > limit:
            raise ValueError("CQ dimensions exceed the native int32 interface")
        padded = ((dim + self.group_size - 1) // self.group_size) * self.group_size
        storage_bits = 2 if self.bits == 5 else self.bits
        if padded * storage_bits > limit:
            raise ValueError("CQ row bit count exceeds the native int32 interface")
        self.padded = padded
        self.packed = np.ascontiguousarray(packed, dtype=np.uint8).reshape(out, padded * storage_bits // 8)
        self.norms = np.ascontiguousarray(norms, dtype=np.float16).reshape(out, padded // self.group_size)
        self.codebook = np.ascontiguousarray(codebook, dtype=np.float32)
        if self.codebook.shape != (3 if self.bits == 5 else 1 << self.bits,):
            raise ValueError("Codebook has incorrect number of centroids")
        if not np.isfinite(self.norms).all() or np.any(self.norms < 0):
            raise ValueError("CQ norms must be finite and nonnegative")
        if not np.isfinite(self.codebook).all() or not np.all(np.diff(self.codebook) > 0):
            raise ValueError("CQ codebook must be finite and strictly sorted")
        if self.bits == 5:
            for shift in (0, 2, 4, 6):
                if np.any(((self.packed >> shift) & 3) == 2):
                    raise ValueError("Invalid ternary crumb code 2")
        self._lib = _library()
        self._handle = self._lib.needle2_cq_create(self.packed.ctypes.data, self.norms.ctypes.data, out, dim,
                                                   self.bits, self.group_size, self.codebook.ctypes.data)
        if not self._handle:
            raise MemoryError(f"Could not construct native CQ matrix: {last_error()}")

    @classmethod
    def from_record(cls, record):
        cb = record.codebook
        if record.bits == 5 and cb is None:
            cb = (np.array([-1.2240064, 0., 1.2240064], np.float64) / np.sqrt(record.group_size)).astype(np.float32)
        return cls(record.packed, record.norms, record.shape, record.bits, record.group_size, cb)

    def __del__(self):
        if getattr(self, "_sdot_handle", None):
            self._lib.needle2_sdot_destroy(self._sdot_handle)
            self._sdot_handle = None
        if getattr(self, "_handle", None):
            self._lib.needle2_cq_destroy(self._handle)
            self._handle = None

    @property
    def groups(self) -> int:
        return self.padded // self.group_size

    def linear(self, x, threads: int = 1, *, lookup: int = 0):
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim < 1 or x.shape[-1] != self.shape[1]:
            raise ValueError(f"Expected input last dimension {self.shape[1]}; got {x.shape}")
        if not 1 <= int(threads) <= 256:
            raise ValueError("threads must be between 1 and 256")
        if (x.size // self.shape[1]) * self.shape[0] > np.iinfo(np.int32).max:
            raise ValueError("CQ batch output count exceeds the native int32 interface")
        y = np.empty(x.shape[:-1] + (self.shape[0],), dtype=np.float32)
        if lookup not in (0, 1, 2, 3):
            raise ValueError("lookup must be 0 (NEON), 1 (byte table), 2 (nibble table), or 3 (group byte table)")
        batch = x.size // self.shape[1]
        if batch:
            _check(self._lib.needle2_cq_linear_checked(self._handle, x.ctypes.data, y.ctypes.data, batch),
                   "needle2_cq_linear")
        return y

    def _sdot(self):
        if self.bits not in (2, 4) or not 64 <= self.group_size <= 131072:
            raise ValueError("SDOT requires CQ2/CQ4 and group size between 64 and 131072")
        if not getattr(self, "_sdot_handle", None):
            self._sdot_handle = self._lib.needle2_sdot_create(self.packed.ctypes.data, self.norms.ctypes.data,
                                                              *self.shape, self.bits, self.group_size,
                                                              self.codebook.ctypes.data)
            if not self._sdot_handle:
                raise RuntimeError(f"could not construct SDOT matrix: {last_error()}")
        return self._sdot_handle

    def _sdot_input(self, x, threads):
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim < 1 or x.shape[-1] != self.shape[1] or not np.isfinite(x).all():
            raise ValueError("SDOT input must have the expected last dimension and finite values")
        if not 1 <= int(threads) <= 256:
            raise ValueError("threads must be between 1 and 256")
        if (x.size // self.shape[1]) * self.shape[0] > np.iinfo(np.int32).max:
            raise ValueError("SDOT batch output count exceeds the native int32 interface")
        return x

    def linear_sdot(self, x, threads: int = 1):
        """int8 GEMV: rotated inputs and centroids rounded to INT8, exact int32 per group."""
        handle = self._sdot()
        x = self._sdot_input(x, threads)
        y = np.empty(x.shape[:-1] + (self.shape[0],), dtype=np.float32)
        batch = x.size // self.shape[1]
        if batch:
            _check(self._lib.needle2_sdot_linear_checked(handle, x.ctypes.data, y.ctypes.data, batch),
                   "needle2_sdot_linear")
        return y

    def sdot_debug(self, x):
        """(y, int32 partials [rows, out, groups], q int8 [rows, padded], scales [rows, groups])."""
        handle = self._sdot()
        x = self._sdot_input(x, 1).reshape(-1, self.shape[1])
        rows = x.shape[0]
        y = np.empty((rows, self.shape[0]), np.float32)
        d = np.empty((rows, self.shape[0], self.groups), np.int32)
        q = np.empty((rows, self.padded), np.int8)
        s = np.empty((rows, self.groups), np.float32)
        if rows:
            _check(self._lib.needle2_sdot_debug(handle, x.ctypes.data, rows, y.ctypes.data, d.ctypes.data,
                                                q.ctypes.data, s.ctypes.data), "needle2_sdot_debug")
        return y, d, q, s

    def linear_device(self, x, y, *, sdot: bool = False, stream=None) -> None:
        """y[batch, out] = W x[batch, in] on device tensors (torch CUDA float32, contiguous)."""
        handle = self._sdot() if sdot else self._handle
        batch = x.numel() // self.shape[1]
        if x.shape[-1] != self.shape[1] or y.shape[-1] != self.shape[0] or y.numel() != batch * self.shape[0]:
            raise ValueError("linear_device: shape mismatch")
        if not (x.is_contiguous() and y.is_contiguous()) or x.dtype != y.dtype:
            raise ValueError("linear_device: contiguous float32 tensors required")
        fn = self._lib.needle2_sdot_linear_device if sdot else self._lib.needle2_cq_linear_device
        _check(fn(handle, x.data_ptr(), y.data_ptr(), batch, _stream_ptr(stream)), "linear_device")

    def prepare_device(self, x, *, sdot: bool = False, stream=None) -> None:
        """Rotate (and for SDOT quantise) device activations into the handle's scratch."""
        handle = self._sdot() if sdot else self._handle
        fn = self._lib.needle2_sdot_prepare_device if sdot else self._lib.needle2_cq_prepare_device
        _check(fn(handle, x.data_ptr(), x.numel() // self.shape[1], _stream_ptr(stream)), "prepare_device")

    def multiply_device(self, y, batch: int, *, sdot: bool = False, stream=None) -> None:
        """y[batch, out] from the last prepare_device."""
        handle = self._sdot() if sdot else self._handle
        fn = self._lib.needle2_sdot_multiply_device if sdot else self._lib.needle2_cq_multiply_device
        _check(fn(handle, y.data_ptr(), int(batch), _stream_ptr(stream)), "multiply_device")

    def rows(self, ids):
        ids = np.asarray(ids)
        if ids.dtype.kind not in "iu":
            raise TypeError("row indices must be integers")
        ids_shape = ids.shape
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        if np.any((ids < 0) | (ids >= self.shape[0])):
            raise IndexError("CQ row index outside matrix")
        result = np.empty(ids_shape + (self.shape[1],), dtype=np.float32)
        if ids.size:
            self._lib.needle2_cq_rows(self._handle, ids.ctypes.data, result.ctypes.data, ids.size)
            _check_void("needle2_cq_rows")
        return result

    def dequantize(self):
        return self.rows(np.arange(self.shape[0], dtype=np.int64))


def linear_many(matrices, x, threads: int = 1, lookup: int = 0):
    """One activation row against several matrices (needle2/csrc/cq.cpp:360-366)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    outs = [np.empty(m.shape[0], np.float32) for m in matrices]
    handles = (_p * len(matrices))(*[m._handle for m in matrices])
    ys = (_p * len(matrices))(*[o.ctypes.data for o in outs])
    lib = _library()
    lib.needle2_cq_linear_many(handles, len(matrices), x.ctypes.data, ys, int(threads), int(lookup))
    _check_void("needle2_cq_linear_many")
    return outs


def linear_many_batch(matrices, x, *, sdot: bool = False):
    """x [batch, in] against several matrices sharing the input: returns a list of
    [batch, out_i] arrays; one fused launch when the geometry allows it."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, matrices[0].shape[1])
    batch = x.shape[0]
    outs = [np.empty((batch, m.shape[0]), np.float32) for m in matrices]
    hs = [m._sdot() if sdot else m._handle for m in matrices]
    handles = (_p * len(hs))(*hs)
    ys = (_p * len(outs))(*[o.ctypes.data for o in outs])
    _check(_library().needle2_cq_linear_many_checked(handles, len(hs), x.ctypes.data, ys, batch, int(sdot)),
           "linear_many")
    return outs


def device_fault() -> int:
    """1 if a kernel's bounded wait ran out since the last call (clears the flag)."""
    return int(_library().needle2_b200_device_fault())


def activation_quant(x, bits: int = 8):
    """The engine's fake activation quantiser (needle2/csrc/engine.cpp:185-191),
    row by row on a copy of x[rows][dim] (a 1-D x is one row), on the GPU."""
    lib = _library()
    fn = lib.needle2_b200_activation_quant
    fn.argtypes = [ct.c_void_p, ct.c_int, ct.c_int, ct.c_int]
    fn.restype = ct.c_int
    a = np.array(x, dtype=np.float32, copy=True, order="C")
    rows, dim = (1, a.size) if a.ndim == 1 else a.shape
    _check(fn(a.ctypes.data, int(rows), int(dim), int(bits)), "activation_quant")
    return a


def argmax_device(logits, out=None, stream=None):
    """Greedy token of each row of a CUDA float32 tensor logits[rows, vocab]
    (the decode loop's scan: first maximum wins, NaNs never chosen); returns an
    int32 CUDA tensor (or fills `out`)."""
    import torch
    lib = _library()
    fn = lib.needle2_b200_argmax_device
    fn.argtypes = [ct.c_void_p, ct.c_int, ct.c_int, ct.c_int, ct.c_void_p, ct.c_void_p]
    fn.restype = ct.c_int
    if logits.dtype != torch.float32 or logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be a float32 [rows, vocab] tensor with unit column stride")
    rows, vocab = logits.shape
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=logits.device)
    _check(fn(logits.data_ptr(), rows, vocab, logits.stride(0), out.data_ptr(), _stream_ptr(stream)), "argmax")
    return out


def set_f32_gemv(kind: int) -> int:
    """Select the FP32-mode GEMV kernel process-wide (0 automatic: the
    product-table cluster kernel for one row, the row-per-lane kernel for up to
    4 rows; 1 the slot-per-lane kernel; 2 the row-per-lane kernel without the
    product table); returns the previous setting."""
    prev = _library().needle2_b200_set_f32_gemv(int(kind))
    if prev < 0:
        raise ValueError(last_error())
    return prev


def set_int8_gemv(kind: int) -> int:
    """Select the int8 GEMV kernel process-wide (0 automatic, 1 diagonal warp
    MMA, 2 tcgen05, 3 fragment-order warp MMA); returns the previous setting."""
    prev = _library().needle2_b200_set_int8_gemv(int(kind))
    if prev < 0:
        raise ValueError(last_error())
    return prev
