"""The Needle-2 forward on the GPU from Python: the engine ABI of
libneedle2_b200.so (needle2_engine_*, a drop-in for needle2/csrc/engine.cpp)
plus its batch extension (needle2_batch_*: many sequences in lockstep).

The reference's own ``needle2.native.NativeEngine`` drives the engine ABI
unchanged through NEEDLE2_NATIVE_LIBRARY; this module is for callers of the
batch extension (the throughput benchmark, multi-sequence tests).  It takes
any archive-like object: ``metadata`` (the .cact header fields) and
``tensors`` (name -> record with ``dtype``, ``shape`` and, for CQ records,
``packed``/``norms``/``bits``/``group_size``/``codebook``, else
``dequantize()``), as needle2/archive.py provides them.
"""
from __future__ import annotations

import ctypes as ct

import numpy as np

from .native import DeviceMatrix, _library

_p = ct.c_void_p
_i = ct.c_int

CQ_DTYPE = 3     # needle2/archive.py record dtype of a packed CQ matrix
LAYER_TENSORS = ("norm_in", "q_proj", "k_proj", "v_proj", "q_norm", "k_norm", "gate_proj", "out_proj", "post_norm",
                 "attn_gate", "pre_hada", "d1", "d2", "d3")
MHC_TENSORS = ("mhc_a_pre", "mhc_a_post", "mhc_a_res", "mhc_b_pre", "mhc_b_post", "mhc_b_res", "mhc_phi_pre",
               "mhc_phi_post", "mhc_phi_res")


class TensorDesc(ct.Structure):
    _fields_ = [("cq", _p), ("data", _p), ("rows", _i), ("cols", _i)]


class EngineConfig(ct.Structure):
    _fields_ = [(k, _i) for k in ("vocab", "dim", "heads", "kvheads", "layers", "head_dim", "max_seq", "hada",
                                  "lanes", "window", "slots", "subdim", "tables", "taps", "dilation", "num_orders")]
    _fields_ += [("orders", _i * 4), ("num_sites", _i), ("sites", _i * 4), ("rope_theta", ct.c_float)]


def tensor_names(m: dict) -> list[str]:
    """The engine's tensor order: embedding, per-layer tensors, mHC, engram sites, final norm."""
    names = ["embedding"]
    for layer in range(m["num_layers"]):
        names += [f"layer{layer:02d}.{t}" for t in LAYER_TENSORS]
    names += list(MHC_TENSORS)
    for site in range(len(m["engram_layers"])):
        names += [f"engram{site}.{t}" for t in ("tables", "key_proj", "value_proj", "taps")]
    names.append("final_norm")
    return names


def engine_config(m: dict) -> EngineConfig:
    c = EngineConfig()
    for field, key in (("vocab", "vocab_size"), ("dim", "d_model"), ("heads", "num_heads"),
                       ("kvheads", "num_kv_heads"), ("layers", "num_layers"), ("head_dim", "head_dim"),
                       ("max_seq", "max_seq_len"), ("hada", "hada_n"), ("lanes", "mhc_lanes"),
                       ("window", "kv_window"), ("slots", "engram_slots"), ("subdim", "engram_sub_dim"),
                       ("tables", "num_engram_tables"), ("taps", "engram_conv_taps"),
                       ("dilation", "engram_conv_dilation")):
        setattr(c, field, int(m[key]))
    orders, sites = list(m["engram_orders"]), list(m["engram_layers"])
    c.num_orders, c.num_sites = len(orders), len(sites)
    c.orders = (_i * 4)(*orders)
    c.sites = (_i * 4)(*sites)
    c.rope_theta = float(m["rope_theta"])
    return c


def _bind(lib):
    if getattr(lib, "_engine_bound", False):
        return lib
    lib.needle2_engine_create.argtypes = [ct.POINTER(EngineConfig), ct.POINTER(TensorDesc), _i, _i, _i]
    lib.needle2_engine_create.restype = _p
    lib.needle2_engine_destroy.argtypes = [_p]
    lib.needle2_engine_destroy.restype = None
    lib.needle2_engine_error.restype = ct.c_char_p
    lib.needle2_engine_set_sdot.argtypes = [_p]
    lib.needle2_engine_set_sdot.restype = _i
    lib.needle2_engine_set_int8_kv.argtypes = [_p, _i]
    lib.needle2_engine_set_int8_kv.restype = _i
    lib.needle2_batch_create.argtypes = [_p, _i, _i]
    lib.needle2_batch_create.restype = _p
    lib.needle2_batch_destroy.argtypes = [_p]
    lib.needle2_batch_destroy.restype = None
    lib.needle2_batch_kv_storage_bytes.argtypes = [_p]
    lib.needle2_batch_kv_storage_bytes.restype = ct.c_size_t
    lib.needle2_batch_set_prefix.argtypes = [_p, _p]
    lib.needle2_batch_set_prefix.restype = _i
    lib.needle2_batch_prefill.argtypes = [_p, _p, _i, _p, _p]
    lib.needle2_batch_prefill.restype = _i
    lib.needle2_batch_step.argtypes = [_p, _p, _p, _p]
    lib.needle2_batch_step.restype = _i
    lib.needle2_batch_decode_greedy.argtypes = [_p, _p, _i, _p]
    lib.needle2_batch_decode_greedy.restype = _i
    lib.needle2_batch_decode_greedy_device.argtypes = [_p, _p, _i, _p, _p]
    lib.needle2_batch_decode_greedy_device.restype = _i
    lib.needle2_batch_positions.argtypes = [_p, _p]
    lib.needle2_batch_positions.restype = _i
    lib.needle2_batch_step_kernels.argtypes = [_p]
    lib.needle2_batch_step_kernels.restype = _i
    lib.needle2_batch_set_graphs.argtypes = [_p, _i]
    lib.needle2_batch_set_graphs.restype = _i
    lib.needle2_batch_profile.argtypes = [_p, _i]
    lib.needle2_batch_profile.restype = _i
    lib.needle2_batch_profile_read.argtypes = [_p, _p, _i]
    lib.needle2_batch_profile_read.restype = _i
    lib._engine_bound = True
    return lib


class GpuModel:
    """A Needle-2 model resident on one GPU (the current CUDA device).

    matmul "fp32" (CQ dequant-accumulate) or "sdot" (int8 SDOT matmuls);
    kv_cache "int8" or "fp32"; activation_bits 0 or 8.  The mHC projections
    are uploaded as FP32 (dequantised when the archive stores them as CQ), as
    the reference's NativeEngine does (needle2/native.py:386-394)."""

    def __init__(self, archive, *, activation_bits: int = 0, matmul: str = "fp32", kv_cache: str = "int8"):
        if matmul not in ("fp32", "sdot") or kv_cache not in ("fp32", "int8") or activation_bits not in (0, 8):
            raise ValueError("matmul fp32|sdot, kv_cache fp32|int8, activation_bits 0|8")
        if matmul == "sdot" and activation_bits:
            raise ValueError("the SDOT mode quantises activations itself; use activation_bits=0")
        self.metadata = m = dict(archive.metadata)
        self._lib = _bind(_library())
        self._owners, descs = [], []
        for name in tensor_names(m):
            rec = archive.tensors[name]
            if rec.dtype == CQ_DTYPE and not name.startswith("mhc_"):
                mat = DeviceMatrix(rec.packed, rec.norms, rec.shape, rec.bits, rec.group_size,
                                   self._codebook(rec))
                self._owners.append(mat)
                descs.append(TensorDesc(mat.fp32.ptr, None, *rec.shape))
            else:
                a = np.ascontiguousarray(rec.dequantize(), dtype=np.float32)
                self._owners.append(a)
                rows, cols = (a.shape[0], int(np.prod(a.shape[1:]))) if a.ndim > 1 else (1, a.size)
                descs.append(TensorDesc(None, a.ctypes.data, rows, cols))
        self._descs = (TensorDesc * len(descs))(*descs)
        self._config = engine_config(m)
        self._h = self._lib.needle2_engine_create(ct.byref(self._config), self._descs, len(descs), 1,
                                                  int(activation_bits))
        if not self._h:
            raise RuntimeError(self._lib.needle2_engine_error().decode())
        if matmul == "sdot" and self._lib.needle2_engine_set_sdot(self._h):
            raise RuntimeError(self._lib.needle2_engine_error().decode())
        if self._lib.needle2_engine_set_int8_kv(self._h, int(kv_cache == "int8")):
            raise RuntimeError(self._lib.needle2_engine_error().decode())
        self.matmul, self.kv_cache, self.activation_bits = matmul, kv_cache, activation_bits

    @staticmethod
    def _codebook(rec):
        if rec.codebook is not None:
            return rec.codebook
        if rec.bits == 5:   # signed ternary crumbs: -c, 0, +c with c = 1.2240064 / sqrt(group)
            c = np.float64(1.2240064) / np.sqrt(rec.group_size)
            return np.array([-c, 0.0, c]).astype(np.float32)
        raise ValueError("CQ record without a codebook")

    @property
    def handle(self):
        return self._h

    def batch(self, sessions: int, prefix_len: int = 0) -> "GpuBatch":
        return GpuBatch(self, sessions, prefix_len)

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.needle2_engine_destroy(self._h)
            self._h = None
        for o in getattr(self, "_owners", []):
            if isinstance(o, DeviceMatrix):
                o.close()
        self._owners = []

    def __del__(self):
        self.close()


class GpuBatch:
    """`sessions` sequences of a GpuModel advancing in lockstep (needle2_batch_*)."""

    def __init__(self, model: GpuModel, sessions: int, prefix_len: int = 0):
        self.model, self.sessions, self.prefix_len = model, int(sessions), int(prefix_len)
        self._lib = model._lib
        self._h = self._lib.needle2_batch_create(model.handle, self.sessions, self.prefix_len)
        if not self._h:
            raise RuntimeError(self._lib.needle2_engine_error().decode())

    def _check(self, rc: int) -> None:
        if rc:
            raise RuntimeError(self._lib.needle2_engine_error().decode())

    @property
    def vocab(self) -> int:
        return int(self.model.metadata["vocab_size"])

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.needle2_batch_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def kv_storage_bytes(self) -> int:
        return int(self._lib.needle2_batch_kv_storage_bytes(self._h))

    STAGES = ("engrams+embedding", "mhc_routing", "qkvg_projections", "qk_norm_rope", "kv_store+attention",
              "out_projection", "mlp+mixing+next_routing", "final_norm+lm_head+greedy")

    def set_graphs(self, enable: bool = True) -> None:
        """Replay decode steps as a captured CUDA graph (default) or launch them one by one."""
        self._check(self._lib.needle2_batch_set_graphs(self._h, int(bool(enable))))

    def step_kernels(self) -> int:
        """Kernels of one decode step (from the last captured step graph)."""
        return int(self._lib.needle2_batch_step_kernels(self._h))

    def profile(self, enable: bool = True) -> None:
        """Per-stage CUDA-event timers of every forward pass (clears the totals)."""
        self._check(self._lib.needle2_batch_profile(self._h, int(bool(enable))))

    def profile_read(self) -> dict:
        """Milliseconds per stage since the last read (synchronises, clears)."""
        ms = np.zeros(len(self.STAGES), np.float64)
        self._check(self._lib.needle2_batch_profile_read(self._h, ms.ctypes.data, ms.size))
        return dict(zip(self.STAGES, ms.tolist()))

    def positions(self) -> np.ndarray:
        out = np.empty(self.sessions, np.int32)
        self._check(self._lib.needle2_batch_positions(self._h, out.ctypes.data))
        return out

    def set_prefix(self, tokens) -> None:
        t = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        if t.size != self.prefix_len:
            raise ValueError(f"the prefix has {self.prefix_len} tokens")
        self._check(self._lib.needle2_batch_set_prefix(self._h, t.ctypes.data))

    def prefill(self, tokens, *, logits: bool = True, greedy: bool = True):
        """tokens [sessions, n] -> (logits [sessions, vocab] of each last token or None,
        greedy next tokens [sessions] or None)."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        if t.ndim != 2 or t.shape[0] != self.sessions:
            raise ValueError(f"tokens must be [{self.sessions}, n]")
        lg = np.empty((self.sessions, self.vocab), np.float32) if logits else None
        nx = np.empty(self.sessions, np.int32) if greedy else None
        self._check(self._lib.needle2_batch_prefill(self._h, t.ctypes.data, t.shape[1],
                                                    lg.ctypes.data if lg is not None else None,
                                                    nx.ctypes.data if nx is not None else None))
        return lg, nx

    def step(self, tokens, *, logits: bool = True, greedy: bool = True):
        t = np.ascontiguousarray(tokens, dtype=np.int32).reshape(self.sessions)
        lg = np.empty((self.sessions, self.vocab), np.float32) if logits else None
        nx = np.empty(self.sessions, np.int32) if greedy else None
        self._check(self._lib.needle2_batch_step(self._h, t.ctypes.data, lg.ctypes.data if lg is not None else None,
                                                 nx.ctypes.data if nx is not None else None))
        return lg, nx

    def decode_greedy(self, first, steps: int) -> np.ndarray:
        """`steps` greedy steps from first[sessions]; returns the generated tokens [sessions, steps]."""
        f = np.ascontiguousarray(first, dtype=np.int32).reshape(self.sessions)
        out = np.empty((self.sessions, int(steps)), np.int32)
        self._check(self._lib.needle2_batch_decode_greedy(self._h, f.ctypes.data, int(steps), out.ctypes.data))
        return out

    def decode_greedy_device(self, first, steps: int, out, stream=None) -> None:
        """The same on int32 CUDA tensors first [sessions], out [sessions, steps]; no host sync."""
        s = None if stream is None else int(getattr(stream, "cuda_stream", stream))
        self._check(self._lib.needle2_batch_decode_greedy_device(self._h, first.data_ptr(), int(steps),
                                                                 out.data_ptr(), s))
