"""GPU parity of the CQ matrix kernels against the oracle and the golden vectors.

FP32 mode: max|y - y_ref| / max|y_ref| <= 1e-4 (FP32_REL_TOL), the path's
stated tolerance; row dequantisation is bit-exact.  SDOT mode: int32
per-group dots, int8 activations and scales bit-exact, and y bit-exact (the
per-group terms are added in the reference's order).
"""
import numpy as np
import pytest

from util import FP32_REL_TOL, example, golden, ref_quantize, rel_err, sha, synthetic_matrix

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def native():
    from openneedle_b200 import build, native
    build.build()
    return native


@pytest.mark.parametrize("bits", [2, 4])
def test_config1_fp32_matches_golden(native, bits):
    g = golden(f"cq{bits}_2048x512.npz")
    q = native.DeviceMatrix(g["packed"], g["norms"], (2048, 512), bits, 128, g["codebook"])
    assert rel_err(q.fp32(g["x"][:1]), g["y_fp32_m1"]) <= FP32_REL_TOL
    assert rel_err(q.fp32(g["x"][:4]), g["y_fp32_m4"]) <= FP32_REL_TOL
    np.testing.assert_allclose(q.fp32(g["x"][:4]), g["y_fp32_m4"], atol=2e-5, rtol=1e-3)
    np.testing.assert_array_equal(q.rows(g["rows_ids"]), g["rows"])


@pytest.mark.parametrize("bits", [2, 4])
def test_config2_sdot_bit_exact_against_golden(native, bits):
    g = golden(f"cq{bits}_2048x512.npz")
    q = native.DeviceMatrix(g["packed"], g["norms"], (2048, 512), bits, 128, g["codebook"])
    for m in (1, 4, 16, 64):
        y, d, qa, s = q.sdot.debug(g["x"][:m])
        assert sha(d) == str(g[f"sdot_partials_sha_m{m}"]), f"int32 partials differ at M={m}"
        assert sha(y) == str(g[f"sdot_y_sha_m{m}"]), f"y differs at M={m}"
        np.testing.assert_array_equal(qa, g["sdot_q"][:m])
        np.testing.assert_array_equal(s, g["sdot_scales"][:m])
        np.testing.assert_array_equal(q.sdot(g["x"][:m]), y)
    np.testing.assert_array_equal(q.sdot.debug(g["x"][:1])[1], g["sdot_partials_m1"])


@pytest.mark.parametrize("bits", [2, 3, 4, 5])
@pytest.mark.parametrize("group", [8, 16, 32, 64, 128, 256, 1024, 2048])
def test_fp32_random_against_oracle(native, oracle_lib, bits, group):
    packed, norms, shape, cb, dense = example(bits, rows=9, dim=257, group=group)
    q = native.DeviceMatrix(packed, norms, shape, bits, group, cb)
    x = np.random.default_rng(9).normal(size=(2, 3, 257)).astype(np.float32)
    y = q.fp32(x)
    ref = oracle_lib.cq_linear(packed, norms, shape, bits, group, cb, x)
    assert y.shape == (2, 3, 9)
    assert rel_err(y, ref) <= FP32_REL_TOL
    np.testing.assert_allclose(y, x @ dense.T, atol=3e-5, rtol=1e-3)
    ids = np.array([[8, 2], [0, 2]])
    np.testing.assert_array_equal(q.rows(ids), oracle_lib.cq_rows(packed, norms, shape, bits, group, cb, ids))
    np.testing.assert_allclose(q.dense(), dense, atol=2e-7, rtol=3e-5)


def test_fp32_empty_and_shape_errors(native):
    packed, norms, shape, cb, _ = example(2)
    q = native.DeviceMatrix(packed, norms, shape, 2, 128, cb)
    assert q.fp32(np.empty((0, 257))).shape == (0, 9)
    with pytest.raises(ValueError):
        q.fp32(np.ones(256))
    with pytest.raises(IndexError):
        q.rows([9])


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("group", [64, 128, 256, 1024, 2048])
def test_sdot_random_against_oracle(native, oracle_lib, bits, group):
    packed, norms, shape, cb, _ = example(bits, rows=129, dim=257, group=group)
    q = native.DeviceMatrix(packed, norms, shape, bits, group, cb)
    x = np.random.default_rng(315).normal(size=(5, 257)).astype(np.float32)
    x[0] = 0
    x[1] = 0
    x[1, 0] = 1
    y, d, qa, s = q.sdot.debug(x)
    ry, rd, rq, rs = oracle_lib.sdot_linear(packed, norms, shape, bits, group, cb, x)
    np.testing.assert_array_equal(qa, rq)
    np.testing.assert_array_equal(s, rs)
    np.testing.assert_array_equal(d, rd)
    np.testing.assert_array_equal(y, ry)


@pytest.mark.parametrize("bits", [2, 4])
def test_sdot_rows_independent_of_block(native, bits):
    """A row's output does not depend on which other rows share the launch
    (the property of tests/test_sdot_row4.py in OpenNeedle)."""
    Q = ref_quantize()
    rng = np.random.default_rng(42)
    w = rng.normal(size=(129, 129)).astype(np.float32) * np.arange(1, 130, dtype=np.float32)[:, None]
    packed, norms = Q.quantize_matrix(w, bits, 64)
    cb = Q.codebook(bits, 64)
    block = native.DeviceMatrix(packed, norms, w.shape, bits, 64, cb)
    for x in (rng.normal(size=129).astype(np.float32), np.zeros(129, np.float32), np.eye(1, 129, dtype=np.float32)[0]):
        whole = block.sdot(x)
        singles = np.concatenate([native.DeviceMatrix(packed[i:i + 1], norms[i:i + 1], (1, 129), bits, 64, cb).sdot(x)
                                  for i in (0, 1, 64, 127, 128)])
        np.testing.assert_array_equal(whole[[0, 1, 64, 127, 128]], singles)


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("n,k", [(8192, 4096), (11008, 4096), (32768, 512)])
def test_large_shapes_against_oracle(native, oracle_lib, bits, n, k):
    packed, norms, cb = synthetic_matrix(n, k, bits, seed=1000 + n)
    q = native.DeviceMatrix(packed, norms, (n, k), bits, 128, cb)
    x = np.random.default_rng(1).normal(size=(3, k)).astype(np.float32)
    assert rel_err(q.fp32(x), oracle_lib.cq_linear(packed, norms, (n, k), bits, 128, cb, x)) <= FP32_REL_TOL
    y, d, _, _ = q.sdot.debug(x)
    ry, rd, _, _ = oracle_lib.sdot_linear(packed, norms, (n, k), bits, 128, cb, x)
    np.testing.assert_array_equal(d, rd)
    np.testing.assert_array_equal(y, ry)


def test_device_entry_points_match_host(native):
    import torch
    g = golden("cq4_2048x512.npz")
    q = native.DeviceMatrix(g["packed"], g["norms"], (2048, 512), 4, 128, g["codebook"])
    x = torch.from_numpy(g["x"][:16]).cuda()
    y = torch.empty(16, 2048, device="cuda")
    q.fp32.linear_device(x, y)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y.cpu().numpy(), q.fp32(g["x"][:16]))
    q.sdot.linear_device(x, y)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y.cpu().numpy(), q.sdot(g["x"][:16]))


def test_linear_many_matches_single(native):
    g = golden("cq2_2048x512.npz")
    a = native.DeviceMatrix(g["packed"], g["norms"], (2048, 512), 2, 128, g["codebook"])
    b = native.DeviceMatrix(g["packed"][:100], g["norms"][:100], (100, 512), 2, 128, g["codebook"])
    ya, yb = native.linear_many([a, b], g["x"][0])
    np.testing.assert_array_equal(ya, a.fp32(g["x"][0]))
    np.testing.assert_array_equal(yb, b.fp32(g["x"][0]))


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("sdot", [False, True])
def test_fused_many_matches_single(native, bits, sdot):
    """Several matrices sharing one input in one fused launch give exactly the
    single-matrix results (the per-row arithmetic does not depend on fusion)."""
    mats = []
    for i, (n, k) in enumerate([(1536, 512), (512, 512), (33, 512), (2048, 512)]):
        p, nrm, cb = synthetic_matrix(n, k, bits, seed=50 + i)
        mats.append(native.DeviceMatrix(p, nrm, (n, k), bits, 128, cb))
    x = np.random.default_rng(3).normal(size=(5, 512)).astype(np.float32)
    outs = native.linear_many_batch(mats, x, sdot=sdot)
    for m, o in zip(mats, outs):
        np.testing.assert_array_equal(o, m.sdot(x) if sdot else m.fp32(x))
    # more matrices than one launch holds
    many = [mats[i % 4] for i in range(37)]
    outs = native.linear_many_batch(many, x[:1], sdot=sdot)
    for m, o in zip(many, outs):
        np.testing.assert_array_equal(o, m.sdot(x[:1]) if sdot else m.fp32(x[:1]))
    assert native.device_fault() == 0
