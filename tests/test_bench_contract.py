"""The reference arm of bench.py on the host: the reference's own engine
(NativeEngine on its CPU library built from its sources) decoding config 5,
printed as the bench contract's JSON line.  It must run without the CUDA
library of this package (a missing library path cannot stop it) and, under
torchrun, only on rank 0."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _run(extra_env):
    env = dict(os.environ)
    env.update(extra_env)
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "2",
                           "--warmup", "3"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_json_line():
    from oracle import oracle as O
    r = _run({"NEEDLE2_B200_LIBRARY": str(ROOT / "no_such_library.so"), "CUDA_VISIBLE_DEVICES": ""})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    if not O.ref_available():
        assert "unavailable" in d
        pytest.skip("the reference's CPU build is missing here")
    assert d["metric"] == "batched_decode_tokens_per_s" and d["unit"] == "tokens/s"
    assert d["higher_is_better"] is True and d["value"] > 0 and d["n_gpus"] == 1
    assert d["config"]["workload"] == "needle2_config5_decode_1024x256"
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_print_nothing():
    r = _run({"WORLD_SIZE": "2", "RANK": "1", "LOCAL_RANK": "1", "CUDA_VISIBLE_DEVICES": ""})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]
