"""The engine's fake activation quantiser (A8 mode, needle2/csrc/engine.cpp:185-191)
on the GPU against the oracle, bit for bit."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def native():
    from openneedle_b200 import build, native
    build.build()
    return native


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("rows,dim", [(1, 512), (7, 100), (64, 4096), (3, 1)])
def test_activation_quant_matches_oracle(native, oracle_lib, bits, rows, dim):
    rng = np.random.default_rng(rows * 1000 + dim + bits)
    x = rng.normal(size=(rows, dim)).astype(np.float32) * rng.uniform(0.01, 100, size=(rows, 1)).astype(np.float32)
    if rows > 2:
        x[1] = 0                       # unchanged
        x[2, ::3] = x[2, ::3] * 1e-6   # tiny values round to zero
    y = native.activation_quant(x, bits)
    ref = np.stack([oracle_lib.activation_quant(r.copy(), bits) for r in x])
    np.testing.assert_array_equal(y, ref)


def test_activation_quant_zero_bits_is_identity(native):
    x = np.random.default_rng(0).normal(size=(2, 33)).astype(np.float32)
    np.testing.assert_array_equal(native.activation_quant(x, 0), x)
