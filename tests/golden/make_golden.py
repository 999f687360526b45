"""Generates the golden fixtures in this directory from the reference itself.

Run where the reference is available (NEEDLE2_REFERENCE_SRC, default the copy
installed into baseline/_ref):

    make -C oracle ref && python tests/golden/make_golden.py

The weights are packed by the reference's own ``needle2.quantize.quantize_matrix``
and every expected output comes from the reference's CPU code compiled from its
sources (oracle/_ref): ``needle2_cq_linear``/``needle2_cq_rows`` of its C ABI,
``SdotCQ`` through the shim, ``Engine::import_state`` and
``Engine::compute_attention`` through the shim.  Inputs follow the seeded
synthetic configurations of the benchmark (seed 0 weights N(0, 0.02),
seed 1 activations N(0, 1)).
"""
from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from oracle import oracle as O  # noqa: E402

if O.reference_package() is None:
    raise SystemExit(f"reference package not found under {O.REF_ROOT}; set NEEDLE2_REFERENCE_SRC")
from needle2 import quantize as ref_quantize  # noqa: E402  (the reference's packer)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def matrices():
    w = np.random.default_rng(0).normal(0.0, 0.02, (2048, 512)).astype(np.float32)
    out = {}
    for bits in (2, 4):
        packed, norms = ref_quantize.quantize_matrix(w, bits, 128)
        out[bits] = (packed, norms, ref_quantize.codebook(bits, 128))
    return out


def main() -> None:
    O.build(reference=True)
    mats = matrices()
    x64 = np.random.default_rng(1).normal(size=(64, 512)).astype(np.float32)
    for bits, (packed, norms, cb) in mats.items():
        shape = (2048, 512)
        # config 1: FP32 matvec, x 1x512
        y1 = O.ref_cq_linear(packed, norms, shape, bits, 128, cb, x64[:1])
        y4 = O.ref_cq_linear(packed, norms, shape, bits, 128, cb, x64[:4])
        rows = O.ref_cq_rows(packed, norms, shape, bits, 128, cb, np.array([0, 1, 777, 2047]))
        # config 2: SDOT int8 mode at M in {1,4,16,64}
        ys, ds, qs, ss = O.ref_sdot(packed, norms, shape, bits, 128, cb, x64)
        fields = dict(packed=packed, norms=norms, codebook=cb, x=x64, y_fp32_m1=y1, y_fp32_m4=y4,
                      rows_ids=np.array([0, 1, 777, 2047]), rows=rows,
                      sdot_q=qs, sdot_scales=ss, sdot_partials_m1=ds[:1], sdot_y_m4=ys[:4])
        for m in (1, 4, 16, 64):
            fields[f"sdot_partials_sha_m{m}"] = np.array(sha(ds[:m]))
            fields[f"sdot_y_sha_m{m}"] = np.array(sha(ys[:m]))
        np.savez_compressed(HERE / f"cq{bits}_2048x512.npz", **fields)

    # INT8 KV attention: 8 heads, 4 KV heads, head_dim 64, sinks + sliding window,
    # and a plain causal cache; K/V imported through the reference rule.
    rng = np.random.default_rng(7)
    att = {}
    for tag, (maxseq, window, prefix, n) in {"win": (64, 16, 8, 40), "full": (48, 0, 5, 48)}.items():
        H, KV, HD = 8, 4, 64
        pos = np.arange(n, dtype=np.int32)
        k = rng.normal(size=(n, KV * HD)).astype(np.float32)
        v = rng.normal(size=(n, KV * HD)).astype(np.float32)
        ki, vi, ks, vs = O.ref_kv_import(H, KV, HD, maxseq, window, prefix, pos, k, v)
        qpos = np.array([n - 1, n - 2, prefix, 3], np.int32) if window else np.array([n - 1, 20, 0], np.int32)
        q = rng.normal(size=(len(qpos), H * HD)).astype(np.float32)
        outs = np.stack([O.ref_attention_i8(H, KV, HD, maxseq, window, prefix, ki, vi, ks, vs, int(p), q[i])
                         for i, p in enumerate(qpos)])
        att.update({f"{tag}_geom": np.array([H, KV, HD, maxseq, window, prefix, n]), f"{tag}_k": k, f"{tag}_v": v,
                    f"{tag}_keys_i8": ki, f"{tag}_values_i8": vi, f"{tag}_k_scales": ks, f"{tag}_v_scales": vs,
                    f"{tag}_qpos": qpos, f"{tag}_q": q, f"{tag}_out": outs})
    np.savez_compressed(HERE / "attention_i8.npz", **att)
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
