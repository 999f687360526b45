"""ctypes access to libneedle2_b200.so for this package's own Python callers.

The reference's Python (needle2/native.py: NativeCQ, NativeEngine) binds the
same library unchanged through NEEDLE2_NATIVE_LIBRARY; this module adds what
that layer has no call for: device-pointer forms, the SDOT debug exports,
fused multi-matrix calls and the kernel switches.  The compute runs in CUDA
kernels only: when the library or a GPU is missing, calls raise instead of
falling back to any CPU path.
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


class Handle:
    """One library handle of a CQ matrix: the FP32-mode matrix
    (needle2_cq_create) or the int8 SDOT matrix (needle2_sdot_create).

    Host calls take numpy arrays whose last axis is the matrix's input width and
    return float32 arrays whose last axis is its output width; the ``*_device``
    calls take contiguous float32 CUDA tensors and enqueue on a stream.
    """

    def __init__(self, owner: "DeviceMatrix", sdot: bool):
        self.owner, self.sdot = owner, bool(sdot)
        lib = owner._lib
        create = lib.needle2_sdot_create if sdot else lib.needle2_cq_create
        out, inp = owner.shape
        self.ptr = create(owner._packed.ctypes.data, owner._norms.ctypes.data, out, inp, owner.bits, owner.group,
                          owner._codebook.ctypes.data)
        if not self.ptr:
            raise RuntimeError(f"{'needle2_sdot_create' if sdot else 'needle2_cq_create'}: {last_error()}")

    def close(self) -> None:
        if self.ptr:
            lib = self.owner._lib
            (lib.needle2_sdot_destroy if self.sdot else lib.needle2_cq_destroy)(self.ptr)
            self.ptr = None

    def __del__(self):
        self.close()

    def _rows(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim < 1 or x.shape[-1] != self.owner.shape[1]:
            raise ValueError(f"input last dimension must be {self.owner.shape[1]}, got shape {x.shape}")
        return x, x.size // self.owner.shape[1]

    def __call__(self, x) -> np.ndarray:
        """y = W x on the GPU from host memory (one synchronous call)."""
        x, batch = self._rows(x)
        y = np.empty(x.shape[:-1] + (self.owner.shape[0],), np.float32)
        if batch:
            fn = self.owner._lib.needle2_sdot_linear_checked if self.sdot else self.owner._lib.needle2_cq_linear_checked
            _check(fn(self.ptr, x.ctypes.data, y.ctypes.data, batch), "linear")
        return y

    def debug(self, x):
        """int8 mode only: (y, int32 group dots [rows, out, groups], int8 activations
        [rows, padded], activation scales [rows, groups])."""
        if not self.sdot:
            raise ValueError("debug exports exist for the int8 (SDOT) handle only")
        x, rows = self._rows(x)
        out, groups, padded = self.owner.shape[0], self.owner.groups, self.owner.padded
        y = np.empty((rows, out), np.float32)
        d = np.empty((rows, out, groups), np.int32)
        q = np.empty((rows, padded), np.int8)
        s = np.empty((rows, groups), np.float32)
        if rows:
            _check(self.owner._lib.needle2_sdot_debug(self.ptr, x.ctypes.data, rows, y.ctypes.data, d.ctypes.data,
                                                      q.ctypes.data, s.ctypes.data), "needle2_sdot_debug")
        return y, d, q, s

    def linear_device(self, x, y, stream=None) -> None:
        """y[batch, out] = W x[batch, in] for CUDA tensors."""
        out, inp = self.owner.shape
        batch = x.numel() // inp
        if x.shape[-1] != inp or y.shape[-1] != out or y.numel() != batch * out:
            raise ValueError("linear_device: shape mismatch")
        if not (x.is_contiguous() and y.is_contiguous()) or x.dtype != y.dtype:
            raise ValueError("linear_device: contiguous float32 tensors required")
        lib = self.owner._lib
        fn = lib.needle2_sdot_linear_device if self.sdot else lib.needle2_cq_linear_device
        _check(fn(self.ptr, x.data_ptr(), y.data_ptr(), batch, _stream_ptr(stream)), "linear_device")

    def prepare_device(self, x, stream=None) -> None:
        """Rotate (int8 mode: rotate and quantise) x into the handle's scratch."""
        lib = self.owner._lib
        fn = lib.needle2_sdot_prepare_device if self.sdot else lib.needle2_cq_prepare_device
        _check(fn(self.ptr, x.data_ptr(), x.numel() // self.owner.shape[1], _stream_ptr(stream)), "prepare_device")

    def multiply_device(self, y, batch: int, stream=None) -> None:
        """y[batch, out] from the last prepare_device."""
        lib = self.owner._lib
        fn = lib.needle2_sdot_multiply_device if self.sdot else lib.needle2_cq_multiply_device
        _check(fn(self.ptr, y.data_ptr(), int(batch), _stream_ptr(stream)), "multiply_device")


class DeviceMatrix:
    """A packed CQ matrix ``[out, in]`` uploaded to the GPU.

    ``fp32`` and ``sdot`` are its two library handles (FP32 dequant-accumulate
    and int8 SDOT arithmetic), each created on first use from the host arrays
    this object keeps.  ``codebook`` holds the stored centroids (bits 5:
    the three ternary centroids).  Argument checks are the library's: a
    create that fails raises with its message.  There is no CPU path.
    """

    def __init__(self, packed, norms, shape, bits: int, group: int, codebook):
        self.shape = (int(shape[0]), int(shape[1]))
        self.bits, self.group = int(bits), int(group)
        self._packed = np.ascontiguousarray(packed, dtype=np.uint8)
        self._norms = np.ascontiguousarray(norms, dtype=np.float16)
        self._codebook = np.ascontiguousarray(codebook, dtype=np.float32)
        self._lib = _library()
        self._handles = {}

    @property
    def padded(self) -> int:
        return -(-self.shape[1] // self.group) * self.group

    @property
    def groups(self) -> int:
        return self.padded // self.group

    def _handle(self, sdot: bool) -> Handle:
        h = self._handles.get(sdot)
        if h is None:
            h = self._handles[sdot] = Handle(self, sdot)
        return h

    @property
    def fp32(self) -> Handle:
        return self._handle(False)

    @property
    def sdot(self) -> Handle:
        return self._handle(True)

    def rows(self, ids) -> np.ndarray:
        """Dequantised rows ``[*ids.shape, in]`` (needle2_cq_rows)."""
        ids = np.asarray(ids)
        if ids.dtype.kind not in "iu":
            raise TypeError("row ids must be integers")
        flat = np.ascontiguousarray(ids, dtype=np.int64).reshape(-1)
        if flat.size and (flat.min() < 0 or flat.max() >= self.shape[0]):
            raise IndexError("row id outside the matrix")
        y = np.empty(ids.shape + (self.shape[1],), np.float32)
        if flat.size:
            self._lib.needle2_cq_rows(self.fp32.ptr, flat.ctypes.data, y.ctypes.data, flat.size)
            _check_void("needle2_cq_rows")
        return y

    def dense(self) -> np.ndarray:
        return self.rows(np.arange(self.shape[0]))

    def close(self) -> None:
        for h in self._handles.values():
            h.close()
        self._handles.clear()


def linear_many(matrices, x, threads: int = 1, lookup: int = 0):
    """One activation row against several matrices (needle2/csrc/cq.cpp:360-366)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    outs = [np.empty(m.shape[0], np.float32) for m in matrices]
    handles = (_p * len(matrices))(*[m.fp32.ptr for m in matrices])
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
    hs = [(m.sdot if sdot else m.fp32).ptr for m in matrices]
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
