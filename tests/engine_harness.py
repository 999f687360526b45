"""Runs engine plans (tests/engine_child.py) in child processes against the
reference's CPU build or this repository's GPU library (test infrastructure)."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent


def run_plan(archive_path, plan, library, workdir, tag, timeout=1800):
    """Executes `plan` with NEEDLE2_NATIVE_LIBRARY=library; returns its outputs."""
    from oracle import oracle as O
    workdir = Path(workdir)
    plan_path = workdir / f"{tag}_plan.json"
    out_path = workdir / f"{tag}_out.npz"
    plan_path.write_text(json.dumps(plan))
    env = dict(os.environ, NEEDLE2_NATIVE_LIBRARY=str(library), NEEDLE2_FRONTEND_LIBRARY=str(O.REF_LIB),
               PYTHONPATH=os.pathsep.join([str(O.REF_ROOT), str(ROOT), str(HERE)]),
               OMP_NUM_THREADS=os.environ.get("OMP_NUM_THREADS", "8"))
    proc = subprocess.run([sys.executable, str(HERE / "engine_child.py"), str(archive_path), str(plan_path),
                           str(out_path)], env=env, capture_output=True, text=True, timeout=timeout)
    if proc.returncode:
        raise RuntimeError(f"{tag} plan failed:\n{proc.stdout[-2000:]}\n{proc.stderr[-4000:]}")
    with np.load(out_path) as z:
        return {k: z[k] for k in z.files}


def rel(a, b) -> float:
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    scale = np.max(np.abs(b)) if b.size else 0.0
    return float(np.max(np.abs(a - b)) / scale) if scale else float(np.max(np.abs(a - b)))


def top2_margin(logits) -> float:
    """Gap between the two largest logits of a row (greedy ties are fragile below it)."""
    s = np.sort(np.asarray(logits, np.float64))
    return float(s[-1] - s[-2])
