"""CQ packing on the host: the weight format the kernels read.

A CQ matrix ``[out, in]`` is split along ``in`` into groups of ``group`` columns
(zero padded to a multiple of ``group``).  Each group is rotated by the
normalised Sylvester-Hadamard matrix, stored as its FP16 L2 norm plus one
``bits``-wide index per element into a sorted codebook, LSB-first
(needle2/quantize.py:54-108, docs/reference.md:98-133 of OpenNeedle).

This module builds such matrices for tests and benchmarks and decodes them for
checks.  It is format code: the kernels never call it.
"""
from __future__ import annotations

import functools
import math

import numpy as np

# The format's shared unit-sphere Lloyd-Max codebook for group 128 (CQ2 at
# [0:4], CQ3 at [4:12], CQ4 at [12:28]); archives carry these values in their
# headers, so packed indices are only meaningful against exactly these numbers
# (needle2/quantize.py:12-20).
_UNIT_CODEBOOK_G128 = np.array([
    -.1331721395254135, -.03990209102630615, .04003528133034706, .13346044719219208,
    -.18926136195659637, -.11788499355316162, -.06614968925714493, -.02101346105337143,
    .022101031616330147, .06678506731987, .11826207488775253, .18982602655887604,
    -.23953154683113098, -.18070605397224426, -.14095793664455414, -.10901255160570145,
    -.08151296526193619, -.056527651846408844, -.03293915092945099, -.010116109624505043,
    .012710800394415855, .03570791706442833, .059458255767822266, .08497702330350876,
    .112741619348526, .1446969211101532, .184239000082016, .2422737032175064,
], dtype=np.float32)
_CODEBOOK_OFFSET = {2: 0, 3: 4, 4: 12}


def check_group(group: int) -> None:
    if group < 8 or group & (group - 1):
        raise ValueError("group_size must be a power of two >= 8")


def codebook(bits: int, group: int = 128) -> np.ndarray:
    """Sorted FP32 centroids for ``bits`` in {2,3,4}, scaled by sqrt(128/group)."""
    if bits not in _CODEBOOK_OFFSET:
        raise ValueError("CQ supports 2, 3, or 4 bits")
    check_group(group)
    start = _CODEBOOK_OFFSET[bits]
    return _UNIT_CODEBOOK_G128[start:start + (1 << bits)].copy() * np.float32(math.sqrt(128 / group))


@functools.lru_cache(maxsize=8)
def hadamard_matrix(n: int) -> np.ndarray:
    """Normalised Sylvester-Hadamard matrix H_n / sqrt(n), float32."""
    check_group(n)
    h = np.array([[1.0]], dtype=np.float32)
    while h.shape[0] < n:
        h = np.concatenate([np.concatenate([h, h], 1), np.concatenate([h, -h], 1)], 0)
    return h * np.float32(1 / math.sqrt(n))


def pack_indices(indices: np.ndarray, bits: int) -> np.ndarray:
    """[rows, cols] indices (cols % 8 == 0) -> LSB-first bitstream bytes."""
    idx = np.asarray(indices)
    if bits not in (2, 3, 4) or idx.ndim != 2 or idx.shape[1] % 8:
        raise ValueError("indices must be [rows, multiple of 8], bits in 2/3/4")
    if idx.size and (idx.min() < 0 or idx.max() >= 1 << bits):
        raise ValueError("index outside codebook")
    # eight fields of `bits` bits fill exactly `bits` bytes
    fields = idx.astype(np.uint64).reshape(idx.shape[0], -1, 8)
    word = np.zeros(fields.shape[:-1], np.uint64)
    for j in range(8):
        word |= fields[..., j] << np.uint64(j * bits)
    out = np.empty(fields.shape[:-1] + (bits,), np.uint8)
    for b in range(bits):
        out[..., b] = ((word >> np.uint64(8 * b)) & np.uint64(0xFF)).astype(np.uint8)
    return out.reshape(idx.shape[0], -1)


def unpack_indices(packed: np.ndarray, bits: int, cols: int) -> np.ndarray:
    """Inverse of pack_indices for ``cols`` columns."""
    p = np.asarray(packed, dtype=np.uint8)
    if bits not in (2, 3, 4) or cols % 8 or p.ndim != 2 or p.shape[1] != cols * bits // 8:
        raise ValueError("invalid packed CQ geometry")
    chunks = p.reshape(p.shape[0], -1, bits).astype(np.uint64)
    word = np.zeros(chunks.shape[:-1], np.uint64)
    for b in range(bits):
        word |= chunks[..., b] << np.uint64(8 * b)
    mask = np.uint64((1 << bits) - 1)
    fields = [((word >> np.uint64(j * bits)) & mask).astype(np.uint8) for j in range(8)]
    return np.stack(fields, -1).reshape(p.shape[0], cols)


def quantize_matrix(weight, bits: int = 2, group: int = 128, cb=None, chunk_rows: int = 256):
    """Pack an FP32 matrix: per group rotate (dense Hadamard, float32), take the
    L2 norm, pick the nearest centroid of the unit vector (ties to the lower
    index) and store the norm as FP16.  Returns (packed uint8, norms float16).

    Same numerics as the format's exporter, needle2/quantize.py:78-108.
    """
    check_group(group)
    w = np.asarray(weight, dtype=np.float32)
    if w.ndim != 2 or not all(w.shape) or not np.isfinite(w).all():
        raise ValueError("weight must be a finite nonempty matrix")
    if bits not in (2, 3, 4):
        raise ValueError("only CQ2/3/4 packing is supported")
    cb = codebook(bits, group) if cb is None else np.asarray(cb, dtype=np.float32)
    if cb.shape != (1 << bits,) or not np.isfinite(cb).all() or not np.all(np.diff(cb) > 0):
        raise ValueError("invalid sorted codebook")
    rows, cols = w.shape
    pad = (-cols) % group
    width = cols + pad
    groups = width // group
    packed = np.empty((rows, width * bits // 8), np.uint8)
    norms = np.empty((rows, groups), np.float16)
    h = hadamard_matrix(group)
    for r0 in range(0, rows, chunk_rows):
        blk = np.pad(w[r0:r0 + chunk_rows], ((0, 0), (0, pad))).reshape(-1, groups, group)
        rot = blk @ h
        norm = np.sqrt(np.sum(rot ** 2, axis=-1, keepdims=True))
        unit = rot / np.maximum(norm, 1e-12)
        hi = np.clip(np.searchsorted(cb, unit), 1, cb.size - 1)
        take_lo = np.abs(unit - cb[hi - 1]) <= np.abs(unit - cb[hi])
        idx = np.where(take_lo, hi - 1, hi)
        packed[r0:r0 + len(blk)] = pack_indices(idx.reshape(len(blk), width), bits)
        with np.errstate(over="ignore"):
            n16 = norm[..., 0].astype(np.float16)
        if not np.isfinite(n16).all():
            raise ValueError("group norm overflows FP16; rescale the weights")
        norms[r0:r0 + len(blk)] = n16
    return packed, norms


def dequantize_matrix(packed, norms, shape, bits: int = 2, group: int = 128, cb=None) -> np.ndarray:
    """Dense FP32 reconstruction (dense Hadamard), for checks."""
    cb = codebook(bits, group) if cb is None else np.asarray(cb, dtype=np.float32)
    rows, cols = shape
    width = -(-cols // group) * group
    idx = unpack_indices(packed, bits, width)
    rot = cb[idx].reshape(rows, -1, group) * np.asarray(norms, dtype=np.float32)[..., None]
    return (rot @ hadamard_matrix(group)).reshape(rows, width)[:, :cols].copy()


def synthetic_matrix(rows: int, cols: int, bits: int, group: int = 128, seed: int = 0, std: float = 0.02):
    """W ~ N(0, std) from default_rng(seed), packed: the benchmark weights."""
    w = np.random.default_rng(seed).normal(0.0, std, (rows, cols)).astype(np.float32)
    packed, norms = quantize_matrix(w, bits, group)
    return packed, norms, codebook(bits, group)
