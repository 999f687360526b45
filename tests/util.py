"""Shared helpers for the parity tests."""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def ref_quantize():
    """The reference's own CQ packer (needle2/quantize.py), from the reference
    package (NEEDLE2_REFERENCE_SRC, default the pip install in baseline/_ref)."""
    from oracle import oracle as O
    if O.reference_package() is None:
        raise RuntimeError(f"reference package not found under {O.REF_ROOT}: install it into baseline/_ref "
                           "or set NEEDLE2_REFERENCE_SRC")
    from needle2 import quantize
    return quantize


def synthetic_matrix(rows: int, cols: int, bits: int, group: int = 128, seed: int = 0, std: float = 0.02):
    """W ~ N(0, std) from default_rng(seed), packed by the reference's quantizer:
    (packed, norms, codebook)."""
    q = ref_quantize()
    w = np.random.default_rng(seed).normal(0.0, std, (rows, cols)).astype(np.float32)
    packed, norms = q.quantize_matrix(w, bits, group)
    return packed, norms, q.codebook(bits, group)


def golden(name: str) -> dict:
    with np.load(GOLDEN / name) as z:
        return {k: z[k] for k in z.files}


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def rel_err(actual, expected) -> float:
    """max |actual - expected| / max |expected| (0 when both are all zero)."""
    actual, expected = np.asarray(actual, np.float64), np.asarray(expected, np.float64)
    scale = np.max(np.abs(expected)) if expected.size else 0.0
    diff = np.max(np.abs(actual - expected)) if expected.size else 0.0
    return float(diff / scale) if scale else float(diff)


# FP32-mode tolerance: outputs within 1e-4 of max|y_ref| (the path's stated bar).
FP32_REL_TOL = 1e-4


def example(bits, rows=9, dim=257, group=128, seed=None):
    """Random packed matrix with zero-norm row 0, as the reference's own test
    builds it (tests/test_native.py:9-29 of OpenNeedle): returns packed, norms,
    shape, codebook, dense reconstruction."""
    rng = np.random.default_rng(104 + bits if seed is None else seed)
    padded = (dim + group - 1) // group * group
    storage = 2 if bits == 5 else bits
    cb = np.linspace(-2, 2, 3 if bits == 5 else 1 << bits, dtype=np.float32) / np.sqrt(np.float32(group))
    indices = rng.integers(0, len(cb), (rows, padded), dtype=np.uint8)
    crumbs = np.where(indices == 0, 3, indices - 1).astype(np.uint8) if bits == 5 else indices
    packed = np.zeros((rows, padded * storage // 8), dtype=np.uint8)
    for col in range(padded):
        bit = col * storage
        packed[:, bit // 8] |= (crumbs[:, col] << (bit % 8)).astype(np.uint8)
        if bit % 8 + storage > 8:
            packed[:, bit // 8 + 1] |= (crumbs[:, col] >> (8 - bit % 8)).astype(np.uint8)
    norms = rng.uniform(0.1, 2, (rows, padded // group)).astype(np.float16)
    norms[0] = 0
    h = np.ones((1, 1), dtype=np.float32)
    while len(h) < group:
        h = np.block([[h, h], [h, -h]])
    h /= np.sqrt(np.float32(group))
    dense = ((cb[indices].reshape(rows, -1, group) * norms.astype(np.float32)[..., None]) @ h).reshape(rows, padded)[:, :dim]
    return packed, norms, (rows, dim), cb, dense
