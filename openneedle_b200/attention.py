"""Batched INT8 KV cache and attention on the GPU (ctypes over libneedle2_b200.so).

``KVCache`` holds ``sessions`` sequences of one attention layer that share one
read-only prefix (stored once on the device).  Its slot map, INT8 rule and
attention follow OpenNeedle's Engine (needle2/csrc/engine.cpp:500, 898-967,
1005-1021); ``export`` returns a session's cache in the reference's own
layout.  Host-array methods copy in and out; ``*_device`` methods take torch
CUDA tensors and do not synchronise.
"""
from __future__ import annotations

import ctypes as ct

import numpy as np

from .native import _check, _library, _stream_ptr, last_error

_p = ct.c_void_p
_i = ct.c_int


def _bind():
    lib = _library()
    if getattr(lib, "_kv_bound", False):
        return lib
    lib.needle2_kv_create.argtypes = [_i, _i, _i, _i, _i, _i, _i]
    lib.needle2_kv_create.restype = _p
    lib.needle2_kv_destroy.argtypes = [_p]
    lib.needle2_kv_destroy.restype = None
    lib.needle2_kv_storage_bytes.argtypes = [_p]
    lib.needle2_kv_storage_bytes.restype = ct.c_size_t
    lib.needle2_kv_set_prefix.argtypes = [_p, _p, _p]
    lib.needle2_kv_set_prefix_device.argtypes = [_p, _p, _p, _p]
    lib.needle2_kv_store.argtypes = [_p, _p, _p, _p, _p, _i]
    lib.needle2_kv_store_device.argtypes = [_p, _p, _p, _p, _p, _i, _p]
    lib.needle2_attention_query.argtypes = [_p, _p, _p, _p, _p, _i]
    lib.needle2_attention_query_device.argtypes = [_p, _p, _p, _p, _p, _i, _p]
    lib.needle2_attention_decode.argtypes = [_p, _p, _p, _p, _p, _p, _p, _i]
    lib.needle2_attention_decode_device.argtypes = [_p, _p, _p, _p, _p, _p, _p, _i, _p]
    lib.needle2_attention_prefill.argtypes = [_p, _p, _p, _i, _p, _p, _p, _p, _i]
    lib.needle2_attention_prefill_device.argtypes = [_p, _p, _p, _i, _p, _p, _p, _p, _i, _p]
    lib.needle2_kv_export.argtypes = [_p, _i, _p, _p, _p, _p]
    for name in ("needle2_kv_set_prefix", "needle2_kv_set_prefix_device", "needle2_kv_store",
                 "needle2_kv_store_device", "needle2_attention_query", "needle2_attention_query_device",
                 "needle2_attention_decode", "needle2_attention_decode_device", "needle2_attention_prefill",
                 "needle2_attention_prefill_device", "needle2_kv_export"):
        getattr(lib, name).restype = _i
    lib._kv_bound = True
    return lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32).reshape(-1)


class KVCache:
    """INT8 KV cache of one layer for ``sessions`` sequences sharing a prefix."""

    def __init__(self, sessions, heads, kvheads, head_dim, max_seq, window=0, prefix_len=0):
        self.sessions, self.heads, self.kvheads, self.head_dim = int(sessions), int(heads), int(kvheads), int(head_dim)
        self.max_seq, self.window, self.prefix_len = int(max_seq), int(window), int(prefix_len)
        if not 0 <= self.prefix_len <= self.max_seq:
            raise ValueError("prefix_len must lie between 0 and max_seq")
        if self.heads % self.kvheads:
            raise ValueError("heads must be a multiple of kvheads")
        self._lib = _bind()
        self._handle = self._lib.needle2_kv_create(self.sessions, self.heads, self.kvheads, self.head_dim,
                                                   self.max_seq, self.window, self.prefix_len)
        if not self._handle:
            raise MemoryError(f"could not create the KV cache: {last_error()}")

    def __del__(self):
        if getattr(self, "_handle", None):
            self._lib.needle2_kv_destroy(self._handle)
            self._handle = None

    @property
    def capacity(self) -> int:
        return self.window + self.prefix_len if self.window else self.max_seq

    @property
    def storage_bytes(self) -> int:
        return int(self._lib.needle2_kv_storage_bytes(self._handle))

    def _kv_width(self):
        return self.kvheads * self.head_dim

    def set_prefix(self, k, v) -> None:
        k, v = _f32(k), _f32(v)
        if k.shape != (self.prefix_len, self._kv_width()) or v.shape != k.shape:
            raise ValueError("prefix K/V must be [prefix_len, kvheads*head_dim]")
        _check(self._lib.needle2_kv_set_prefix(self._handle, k.ctypes.data, v.ctypes.data), "kv_set_prefix")

    def store(self, session_ids, positions, k, v) -> None:
        ids, pos = _i32(session_ids), _i32(positions)
        k, v = _f32(k), _f32(v)
        if k.shape != (ids.size, self._kv_width()) or v.shape != k.shape or pos.size != ids.size:
            raise ValueError("store: k, v must be [count, kvheads*head_dim]")
        _check(self._lib.needle2_kv_store(self._handle, ids.ctypes.data, pos.ctypes.data, k.ctypes.data,
                                          v.ctypes.data, ids.size), "kv_store")

    def query(self, session_ids, positions, q):
        ids, pos, q = _i32(session_ids), _i32(positions), _f32(q)
        if q.shape != (ids.size, self.heads * self.head_dim) or pos.size != ids.size:
            raise ValueError("query: q must be [count, heads*head_dim]")
        out = np.empty_like(q)
        _check(self._lib.needle2_attention_query(self._handle, ids.ctypes.data, pos.ctypes.data, q.ctypes.data,
                                                 out.ctypes.data, ids.size), "attention_query")
        return out

    def decode(self, session_ids, positions, q, k, v):
        ids, pos, q, k, v = _i32(session_ids), _i32(positions), _f32(q), _f32(k), _f32(v)
        n = ids.size
        if q.shape != (n, self.heads * self.head_dim) or k.shape != (n, self._kv_width()) or v.shape != k.shape:
            raise ValueError("decode: q [count, heads*hd], k/v [count, kvheads*hd]")
        out = np.empty_like(q)
        _check(self._lib.needle2_attention_decode(self._handle, ids.ctypes.data, pos.ctypes.data, q.ctypes.data,
                                                  k.ctypes.data, v.ctypes.data, out.ctypes.data, n),
               "attention_decode")
        return out

    def prefill(self, session_ids, start_positions, q, k, v):
        """q [count, tokens, heads*hd], k/v [count, tokens, kvheads*hd] -> out like q."""
        ids, pos, q, k, v = _i32(session_ids), _i32(start_positions), _f32(q), _f32(k), _f32(v)
        n = ids.size
        if q.ndim != 3 or q.shape[0] != n or q.shape[2] != self.heads * self.head_dim:
            raise ValueError("prefill: q must be [count, tokens, heads*head_dim]")
        t = q.shape[1]
        if k.shape != (n, t, self._kv_width()) or v.shape != k.shape:
            raise ValueError("prefill: k/v must be [count, tokens, kvheads*head_dim]")
        out = np.empty_like(q)
        _check(self._lib.needle2_attention_prefill(self._handle, ids.ctypes.data, pos.ctypes.data, t, q.ctypes.data,
                                                   k.ctypes.data, v.ctypes.data, out.ctypes.data, n),
               "attention_prefill")
        return out

    def export(self, session: int) -> dict:
        cap, w = self.capacity, self._kv_width()
        r = {"keys_i8": np.zeros((cap, w), np.int8), "values_i8": np.zeros((cap, w), np.int8),
             "k_scales": np.zeros((cap, self.kvheads), np.float32),
             "v_scales": np.zeros((cap, self.kvheads), np.float32)}
        _check(self._lib.needle2_kv_export(self._handle, int(session), r["keys_i8"].ctypes.data,
                                           r["values_i8"].ctypes.data, r["k_scales"].ctypes.data,
                                           r["v_scales"].ctypes.data), "kv_export")
        return r

    # ---- device tensors (torch CUDA, contiguous float32); ids/positions are host arrays
    def set_prefix_device(self, k, v, stream=None) -> None:
        _check(self._lib.needle2_kv_set_prefix_device(self._handle, k.data_ptr(), v.data_ptr(), _stream_ptr(stream)),
               "kv_set_prefix_device")

    def decode_device(self, session_ids, positions, q, k, v, out, stream=None) -> None:
        ids, pos = _i32(session_ids), _i32(positions)
        _check(self._lib.needle2_attention_decode_device(self._handle, ids.ctypes.data, pos.ctypes.data, q.data_ptr(),
                                                         k.data_ptr(), v.data_ptr(), out.data_ptr(), ids.size,
                                                         _stream_ptr(stream)), "attention_decode_device")

    def store_device(self, session_ids, positions, k, v, stream=None) -> None:
        ids, pos = _i32(session_ids), _i32(positions)
        _check(self._lib.needle2_kv_store_device(self._handle, ids.ctypes.data, pos.ctypes.data, k.data_ptr(),
                                                 v.data_ptr(), ids.size, _stream_ptr(stream)), "kv_store_device")

    def query_device(self, session_ids, positions, q, out, stream=None) -> None:
        ids, pos = _i32(session_ids), _i32(positions)
        _check(self._lib.needle2_attention_query_device(self._handle, ids.ctypes.data, pos.ctypes.data, q.data_ptr(),
                                                        out.data_ptr(), ids.size, _stream_ptr(stream)),
               "attention_query_device")

    def prefill_device(self, session_ids, start_positions, tokens, q, k, v, out, stream=None) -> None:
        ids, pos = _i32(session_ids), _i32(start_positions)
        _check(self._lib.needle2_attention_prefill_device(self._handle, ids.ctypes.data, pos.ctypes.data, int(tokens),
                                                          q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                                          ids.size, _stream_ptr(stream)), "attention_prefill_device")
