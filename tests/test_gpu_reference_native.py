"""The reference's own Python layer (needle2/native.py, NativeCQ) computing on
this library: NEEDLE2_NATIVE_LIBRARY points the reference's loader at
libneedle2_b200.so (needle2/native.py:76-84), and its unchanged NativeCQ.linear,
linear(lookup=1..3), linear_sdot, rows and dequantize run on the GPU against
the golden fixtures that the reference's CPU build produced.

The reference package comes from NEEDLE2_REFERENCE_SRC, by default the copy
pip installed into baseline/_ref; without it the test skips.  It runs in a
child process because the reference's loader caches its library choice."""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from util import FP32_REL_TOL, golden, rel_err, sha

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]

CHILD = r"""
import sys
import numpy as np
from needle2.native import NativeCQ, build_native, sdot_available
out = {}
assert sdot_available()
for bits in (2, 4):
    with np.load(sys.argv[1] + f"/cq{bits}_2048x512.npz") as z:
        g = {k: z[k] for k in z.files}
    q = NativeCQ(g["packed"], g["norms"], (2048, 512), bits, 128, g["codebook"])
    for m in (1, 4, 16, 64):
        out[f"cq{bits}_fp32_m{m}"] = q.linear(g["x"][:m])
        out[f"cq{bits}_sdot_m{m}"] = q.linear_sdot(g["x"][:m])
    for mode in (1, 2, 3):
        out[f"cq{bits}_lookup{mode}"] = q.linear(g["x"][:4], lookup=mode)
    out[f"cq{bits}_rows"] = q.rows(g["rows_ids"])
    out[f"cq{bits}_dense"] = q.dequantize()[:64]
print(build_native())
np.savez(sys.argv[2], **out)
"""


@pytest.fixture(scope="module")
def reference_results(tmp_path_factory):
    from oracle import oracle as O
    from openneedle_b200 import build
    if O.reference_package() is None:
        pytest.skip(f"reference package unavailable under {O.REF_ROOT}")
    lib = build.build()
    dst = tmp_path_factory.mktemp("refnative") / "out.npz"
    env = dict(os.environ, NEEDLE2_NATIVE_LIBRARY=str(lib), PYTHONPATH=str(O.REF_ROOT))
    proc = subprocess.run([sys.executable, "-c", CHILD, str(ROOT / "tests" / "golden"), str(dst)], env=env,
                          capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-3000:]
    assert Path(proc.stdout.strip().splitlines()[-1]).resolve() == Path(lib).resolve()
    with np.load(dst) as z:
        return {k: z[k] for k in z.files}


@pytest.mark.parametrize("bits", [2, 4])
def test_reference_nativecq_runs_on_this_library(reference_results, oracle_lib, bits):
    r = reference_results
    g = golden(f"cq{bits}_2048x512.npz")
    assert rel_err(r[f"cq{bits}_fp32_m1"], g["y_fp32_m1"]) <= FP32_REL_TOL
    assert rel_err(r[f"cq{bits}_fp32_m4"], g["y_fp32_m4"]) <= FP32_REL_TOL
    for mode in (1, 2, 3):
        assert rel_err(r[f"cq{bits}_lookup{mode}"], g["y_fp32_m4"]) <= FP32_REL_TOL
    for m in (1, 4, 16, 64):
        # the reference's SDOT y is bit-exact (golden SHA-256 from its SdotCQ)
        assert sha(r[f"cq{bits}_sdot_m{m}"]) == str(g[f"sdot_y_sha_m{m}"])
        ref = oracle_lib.cq_linear(g["packed"], g["norms"], (2048, 512), bits, 128, g["codebook"], g["x"][:m])
        assert rel_err(r[f"cq{bits}_fp32_m{m}"], ref) <= FP32_REL_TOL
    np.testing.assert_array_equal(r[f"cq{bits}_rows"], g["rows"])
    dense = oracle_lib.cq_rows(g["packed"], g["norms"], (2048, 512), bits, 128, g["codebook"], np.arange(64))
    np.testing.assert_array_equal(r[f"cq{bits}_dense"], dense)
