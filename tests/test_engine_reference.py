"""The engine-parity harness on CPU: the reference's own NativeEngine, built
from its sources (oracle/_ref), runs the plans that the GPU tests compare
against, and shows the properties those comparisons rely on (prefill equals
token-by-token steps within FP32 tolerance, a restored prefix reproduces its
continuation bit for bit, the SDOT hook runs).  Needs the reference package
(NEEDLE2_REFERENCE_SRC, default baseline/_ref) and oracle/_ref."""
import numpy as np
import pytest

from engine_harness import rel, run_plan

pytestmark = pytest.mark.reference


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    from oracle import oracle as O
    if O.reference_package() is None or not O.ref_available():
        pytest.skip("reference package or oracle/_ref unavailable")
    from engine_models import build_archive, save_archive, tiny_config
    d = tmp_path_factory.mktemp("engine")
    meta, records = build_archive(tiny_config(window=5), seed=117)
    path = d / "tiny.npz"
    save_archive(path, meta, records)
    return path, d, O.REF_LIB


def test_reference_engine_plan_properties(tiny):
    path, d, lib = tiny
    ids = [int(t) for t in np.random.default_rng(3).integers(1, 61, 20)]
    plan = [{"op": "engine", "kv": "fp32"}, {"op": "reset", "prefix": 3},
            {"op": "prefill", "tokens": ids}, {"op": "reset", "prefix": 3},
            {"op": "prefill", "tokens": ids[:3]}, {"op": "cache_prefix"}]
    plan += [{"op": "step", "token": int(t)} for t in ids[3:]]
    plan += [{"op": "reset_to_prefix"}] + [{"op": "step", "token": int(t)} for t in ids[3:]]
    plan += [{"op": "engine", "kv": "int8", "matmul": "sdot"}, {"op": "prefill", "tokens": ids, "last_only": True},
             {"op": "decode", "first": 5, "max_new": 4}]
    r = run_plan(path, plan, lib, d, "ref")
    full = r["2_logits"]
    steps = np.stack([r[f"{6 + j}_logits"] for j in range(len(ids) - 3)])
    assert rel(steps, full[3:]) <= 1e-4                       # prefill == steps within FP32 rounding
    again = np.stack([r[f"{7 + len(ids) - 3 + j}_logits"] for j in range(len(ids) - 3)])
    np.testing.assert_array_equal(again, steps)               # restored prefix: bit for bit
    n = len(plan)
    assert r[f"{n - 1}_tokens"][0] == 5 and len(r[f"{n - 1}_tokens"]) <= 4
    assert np.isfinite(r[f"{n - 2}_logits"]).all()
