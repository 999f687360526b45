"""N-sharded SDOT matrices across the GPUs of one node (one process per GPU).

The packed rows of a CQ matrix are independent, so a matrix of `out` rows is
split into `world` shards of `ns` consecutive rows (`ns` = out / world rounded
up to a multiple of 4, the last shard padded with zero-norm rows, which give
zero outputs).  Every rank computes y[:, shard] for the whole batch; the full
y[batch][out] is then the all-gather of the shards.

Two forms of the exchange:

* ``forward``: the all-gather is fused into the int8 GEMM's epilogue.  Each rank
  holds a full [max_batch][world * ns] output buffer; the buffers are shared
  through CUDA IPC, and every rank's GEMM writes its output tiles into its
  columns of every rank's buffer (peer stores over NVLink) while the other
  tiles are still being computed.  A tiny NCCL all-reduce afterwards orders the
  ranks' kernels before anyone reads.
* ``forward_nccl``: the GEMM into a local [batch][ns] block, then NCCL's
  all_gather_into_tensor and a transpose (the baseline).

The reference has no multi-GPU path; shard results are bit-identical to the
single-GPU matrix because each output element depends only on its own row.
"""
from __future__ import annotations

import ctypes as ct

import numpy as np

from .native import _check, _library, _stream_ptr

_p = ct.c_void_p
_i = ct.c_int


def shard_layout(out: int, world: int, align: int = 4):
    """Rows per shard and each rank's [start, stop) rows of the original matrix."""
    if out <= 0 or world <= 0:
        raise ValueError("out and world must be positive")
    ns = -(-out // world)
    ns = -(-ns // align) * align
    return ns, [(min(out, r * ns), min(out, (r + 1) * ns)) for r in range(world)]


def shard_matrix(packed, norms, out: int, rank: int, world: int):
    """Packed rows and norm rows of `rank`'s shard, zero-padded to ns rows."""
    ns, spans = shard_layout(out, world)
    r0, r1 = spans[rank]
    p = np.zeros((ns, packed.shape[1]), packed.dtype)
    n = np.zeros((ns, norms.shape[1]), norms.dtype)
    p[: r1 - r0] = packed[r0:r1]
    n[: r1 - r0] = norms[r0:r1]
    return p, n


def assemble(gathered, out: int):
    """[world][batch][ns] shard outputs -> [batch][out] (numpy or torch)."""
    world, batch, ns = gathered.shape
    if hasattr(gathered, "permute"):
        return gathered.permute(1, 0, 2).reshape(batch, world * ns)[:, :out]
    return gathered.transpose(1, 0, 2).reshape(batch, world * ns)[:, :out]


def _bind():
    lib = _library()
    if getattr(lib, "_sharded_bound", False):
        return lib
    lib.needle2_sdot_create.argtypes = [_p, _p, _i, _i, _i, _i, _p]
    lib.needle2_sdot_create.restype = _p
    lib.needle2_sdot_destroy.argtypes = [_p]
    lib.needle2_sdot_destroy.restype = None
    lib.needle2_sdot_prepare_device.argtypes = [_p, _p, _i, _p]
    lib.needle2_sdot_prepare_device.restype = _i
    lib.needle2_sdot_multiply_device.argtypes = [_p, _p, _i, _p]
    lib.needle2_sdot_multiply_device.restype = _i
    lib.needle2_sdot_multiply_gather_device.argtypes = [_p, ct.POINTER(_p), _i, _i, _i, _p]
    lib.needle2_sdot_multiply_gather_device.restype = _i
    lib.needle2_b200_ipc_export.argtypes = [_p, _p, ct.POINTER(ct.c_ulonglong)]
    lib.needle2_b200_ipc_export.restype = _i
    lib.needle2_b200_ipc_import.argtypes = [_p, ct.c_ulonglong, ct.POINTER(_p)]
    lib.needle2_b200_ipc_import.restype = _i
    lib.needle2_b200_ipc_close.argtypes = [_p]
    lib.needle2_b200_ipc_close.restype = _i
    lib._sharded_bound = True
    return lib


class ShardedSdot:
    """This rank's shard of an SDOT (int8-mode) CQ matrix, with its share of the
    all-gather.  Collective: every rank of `process_group` constructs it with the
    same matrix and calls the same methods in the same order."""

    def __init__(self, packed, norms, shape, bits: int, group: int, codebook, max_batch: int,
                 process_group=None, device=None):
        import torch
        import torch.distributed as dist

        self._dist, self._torch = dist, torch
        self.group = process_group
        self.rank = dist.get_rank(process_group)
        self.world = dist.get_world_size(process_group)
        self.out, self.inp = int(shape[0]), int(shape[1])
        self.max_batch = int(max_batch)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.ns, self.spans = shard_layout(self.out, self.world)
        self._lib = _bind()
        p, n = shard_matrix(np.ascontiguousarray(packed), np.ascontiguousarray(norms), self.out, self.rank, self.world)
        cb = np.ascontiguousarray(codebook, dtype=np.float32)
        self._h = self._lib.needle2_sdot_create(p.ctypes.data, n.ctypes.data, self.ns, self.inp, int(bits), int(group),
                                                cb.ctypes.data)
        if not self._h:
            raise RuntimeError(f"sdot_create: {self._lib.needle2_b200_error().decode()}")
        # this rank's full output, shared with the other ranks
        self.full = torch.zeros(self.max_batch, self.world * self.ns, device=self.device)
        handle = ct.create_string_buffer(64)
        offset = ct.c_ulonglong(0)
        _check(self._lib.needle2_b200_ipc_export(self.full.data_ptr(), handle, ct.byref(offset)), "ipc_export")
        mine = (handle.raw, int(offset.value))
        table = [None] * self.world
        dist.all_gather_object(table, mine, group=process_group)
        self._imported = []
        ptrs = []
        for r, (h, off) in enumerate(table):
            if r == self.rank:
                ptrs.append(self.full.data_ptr())
                continue
            ptr = _p()
            _check(self._lib.needle2_b200_ipc_import(h, off, ct.byref(ptr)), "ipc_import")
            self._imported.append(ptr.value)
            ptrs.append(ptr.value)
        # every rank's buffer, at this shard's first column
        col = 4 * self.rank * self.ns
        self._dsts = (_p * self.world)(*[q + col for q in ptrs])
        self._flag = torch.zeros(1, device=self.device)
        self._local = None

    def close(self) -> None:
        if getattr(self, "_imported", None):
            for ptr in self._imported:
                self._lib.needle2_b200_ipc_close(ptr)
            self._imported = []
        if getattr(self, "_h", None):
            self._lib.needle2_sdot_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def _prepare(self, x, stream):
        batch = int(x.shape[0])
        if batch > self.max_batch:
            raise ValueError(f"batch {batch} exceeds max_batch {self.max_batch}")
        if x.shape[1] != self.inp or x.dtype != self._torch.float32 or not x.is_contiguous():
            raise ValueError(f"x must be a contiguous float32 [batch, {self.inp}] tensor")
        _check(self._lib.needle2_sdot_prepare_device(self._h, x.data_ptr(), batch, _stream_ptr(stream)), "prepare")
        return batch

    def _torch_stream(self, stream):
        """The torch stream that `stream` names (None: the current stream)."""
        torch = self._torch
        if stream is None:
            return torch.cuda.current_stream(self.device)
        if isinstance(stream, torch.cuda.Stream):
            return stream
        return torch.cuda.ExternalStream(int(stream), device=self.device)

    def barrier(self, stream=None) -> None:
        """Orders, on `stream`, everything every rank enqueued on its stream
        before this call ahead of anything any rank enqueues after it (a
        one-element all-reduce; its kernel cannot finish before every rank's
        stream has reached it)."""
        with self._torch.cuda.stream(self._torch_stream(stream)):
            self._dist.all_reduce(self._flag, group=self.group)

    def forward(self, x, stream=None):
        """y[batch][out] with the all-gather fused into the GEMM's epilogue.

        Returns a view of this rank's shared output buffer.  Every rank's next
        forward() overwrites every rank's buffer, so the view is valid until the
        next call on any rank; work that reads it must be enqueued on `stream`
        (or be ordered before the next forward() on it).  A barrier before the
        GEMM makes every rank's earlier reads of its buffer finish before any
        rank's epilogue stores into it; a barrier after it makes every rank's
        stores land before this rank's later work reads them."""
        batch = self._prepare(x, stream)
        self.barrier(stream)
        _check(self._lib.needle2_sdot_multiply_gather_device(self._h, self._dsts, self.world, self.world * self.ns,
                                                             batch, _stream_ptr(stream)), "multiply_gather")
        self.barrier(stream)
        return self.full[:batch, : self.out]

    def forward_local(self, x, stream=None):
        """This rank's shard only: [batch][ns] (no exchange)."""
        batch = self._prepare(x, stream)
        if self._local is None or self._local.shape[0] < batch:
            self._local = self._torch.empty(self.max_batch, self.ns, device=self.device)
        y = self._local[:batch]
        _check(self._lib.needle2_sdot_multiply_device(self._h, y.data_ptr(), batch, _stream_ptr(stream)), "multiply")
        return y

    def forward_nccl(self, x, stream=None):
        """The same y[batch][out] through a local GEMM and NCCL's all-gather."""
        y = self.forward_local(x, stream)
        g = self._torch.empty(self.world, y.shape[0], self.ns, device=self.device)
        with self._torch.cuda.stream(self._torch_stream(stream)):
            self._dist.all_gather_into_tensor(g, y.contiguous(), group=self.group)
            return assemble(g, self.out)
