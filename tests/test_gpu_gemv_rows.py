"""GPU parity of the FP32-mode decode GEMVs against the oracle's CQ::linear,
within the FP32 tolerance max|y - y_ref| / max|y_ref| <= 1e-4: the
product-table cluster kernel (one activation row), the row-per-lane kernel
(up to 4 rows) and the slot-per-lane kernel, also against one another.
Shapes cover row counts that leave a partial 32-row block, group counts that
split over 1, 2, 4 and 8 warps or cluster CTAs (including a count that is not
a power of two), 2- and 4-bit storage and group sizes 64, 128 and 256."""
import numpy as np
import pytest

from util import FP32_REL_TOL, example, rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def native():
    from openneedle_b200 import build, native
    build.build()
    return native


@pytest.fixture
def f32_kind(native):
    prev = native.set_f32_gemv(0)
    yield
    native.set_f32_gemv(prev)


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("group,dim", [(64, 64), (64, 448), (128, 300), (128, 384), (128, 512), (128, 768), (128, 4096),
                                       (128, 5120), (256, 2048), (256, 8192)])
@pytest.mark.parametrize("rows", [33, 100])
def test_rows_kernel_against_oracle(native, oracle_lib, f32_kind, bits, group, dim, rows):
    packed, norms, shape, cb, dense = example(bits, rows=rows, dim=dim, group=group, seed=7 * dim + rows)
    q = native.DeviceMatrix(packed, norms, shape, bits, group, cb)
    x = np.random.default_rng(dim + bits).normal(size=(4, dim)).astype(np.float32)
    for m in (1, 2, 3, 4):
        ref = oracle_lib.cq_linear(packed, norms, shape, bits, group, cb, x[:m])
        # automatic choice, slot-per-lane, row-per-lane without the table: the
        # same sums in different orders
        ys = []
        for kind in (0, 1, 2):
            native.set_f32_gemv(kind)
            ys.append(q.fp32(x[:m]))
            native.set_f32_gemv(0)
            assert rel_err(ys[-1], ref) <= FP32_REL_TOL, (m, kind, rel_err(ys[-1], ref))
        assert rel_err(ys[0], ys[1]) <= FP32_REL_TOL
        assert rel_err(ys[2], ys[1]) <= FP32_REL_TOL
        # repeated calls give identical results (no atomics, fixed order)
        np.testing.assert_array_equal(q.fp32(x[:m]), ys[0])
    assert native.device_fault() == 0


@pytest.mark.parametrize("bits", [2, 4])
def test_rows_kernel_large_and_fused(native, oracle_lib, f32_kind, bits):
    """A K = 4096 matrix (32 groups, eight warps per row block) against the
    oracle, and a fused launch over matrices of different heights giving the
    single-matrix results exactly."""
    from util import synthetic_matrix
    p, nrm, cb = synthetic_matrix(2080, 4096, bits, seed=21)
    big = native.DeviceMatrix(p, nrm, (2080, 4096), bits, 128, cb)
    x = np.random.default_rng(5).normal(size=(2, 4096)).astype(np.float32)
    assert rel_err(big.fp32(x[:1]), oracle_lib.cq_linear(p, nrm, (2080, 4096), bits, 128, cb, x[:1])) \
        <= FP32_REL_TOL
    mats = [big]
    for i, n in enumerate((31, 32, 4097)):
        pi, ni, _ = synthetic_matrix(n, 4096, bits, seed=60 + i)
        mats.append(native.DeviceMatrix(pi, ni, (n, 4096), bits, 128, cb))
    for m in (1, 2):
        outs = native.linear_many_batch(mats, x[:m], sdot=False)
        for mat, o in zip(mats, outs):
            np.testing.assert_array_equal(o, mat.fp32(x[:m]))
    assert native.device_fault() == 0
