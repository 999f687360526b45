"""GPU parity of the CQ matrix kernels against the oracle and the golden vectors.

FP32 mode: max|y - y_ref| / max|y_ref| <= 1e-4 (FP32_REL_TOL), the path's
stated tolerance; row dequantisation is bit-exact.  SDOT mode: int32
per-group dots, int8 activations and scales bit-exact, and y bit-exact (the
per-group terms are added in the reference's order).
"""
import numpy as np
import pytest

from util import FP32_REL_TOL, example, golden, rel_err, sha

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def native():
    from openneedle_b200 import build, native
    build.build()
    return native


@pytest.fixture(params=[1, 2, 3], ids=["diag_mma", "tcgen05", "frag_mma"])
def int8_kernel(request, native):
    """Run an SDOT test once per int8 GEMV kernel (both must be bit-exact)."""
    prev = native.set_int8_gemv(request.param)
    yield request.param
    native.set_int8_gemv(prev)


@pytest.mark.parametrize("bits", [2, 4])
def test_config1_fp32_matches_golden(native, bits):
    g = golden(f"cq{bits}_2048x512.npz")
    q = native.NativeCQ(g["packed"], g["norms"], (2048, 512), bits, 128, g["codebook"])
    assert rel_err(q.linear(g["x"][:1]), g["y_fp32_m1"]) <= FP32_REL_TOL
    assert rel_err(q.linear(g["x"][:4]), g["y_fp32_m4"]) <= FP32_REL_TOL
    np.testing.assert_allclose(q.linear(g["x"][:4]), g["y_fp32_m4"], atol=2e-5, rtol=1e-3)
    np.testing.assert_array_equal(q.rows(g["rows_ids"]), g["rows"])


@pytest.mark.parametrize("bits", [2, 4])
def test_config2_sdot_bit_exact_against_golden(native, int8_kernel, bits):
    g = golden(f"cq{bits}_2048x512.npz")
    q = native.NativeCQ(g["packed"], g["norms"], (2048, 512), bits, 128, g["codebook"])
    for m in (1, 4, 16, 64):
        y, d, qa, s = q.sdot_debug(g["x"][:m])
        assert sha(d) == str(g[f"sdot_partials_sha_m{m}"]), f"int32 partials differ at M={m}"
        assert sha(y) == str(g[f"sdot_y_sha_m{m}"]), f"y differs at M={m}"
        np.testing.assert_array_equal(qa, g["sdot_q"][:m])
        np.testing.assert_array_equal(s, g["sdot_scales"][:m])
        np.testing.assert_array_equal(q.linear_sdot(g["x"][:m]), y)
    np.testing.assert_array_equal(q.sdot_debug(g["x"][:1])[1], g["sdot_partials_m1"])


@pytest.mark.parametrize("bits", [2, 3, 4, 5])
@pytest.mark.parametrize("group", [8, 16, 32, 64, 128, 256, 1024, 2048])
def test_fp32_random_against_oracle(native, oracle_lib, bits, group):
    packed, norms, shape, cb, dense = example(bits, rows=9, dim=257, group=group)
    q = native.NativeCQ(packed, norms, shape, bits, group, cb)
    x = np.random.default_rng(9).normal(size=(2, 3, 257)).astype(np.float32)
    y = q.linear(x)
    ref = oracle_lib.cq_linear(packed, norms, shape, bits, group, cb, x)
    assert y.shape == (2, 3, 9)
    assert rel_err(y, ref) <= FP32_REL_TOL
    np.testing.assert_allclose(y, x @ dense.T, atol=3e-5, rtol=1e-3)
    for lookup in (1, 2, 3):
        assert rel_err(q.linear(x, lookup=lookup), ref) <= FP32_REL_TOL
    ids = np.array([[8, 2], [0, 2]])
    np.testing.assert_array_equal(q.rows(ids), oracle_lib.cq_rows(packed, norms, shape, bits, group, cb, ids))
    np.testing.assert_allclose(q.dequantize(), dense, atol=2e-7, rtol=3e-5)


def test_fp32_empty_and_shape_errors(native):
    packed, norms, shape, cb, _ = example(2)
    q = native.NativeCQ(packed, norms, shape, 2, 128, cb)
    assert q.linear(np.empty((0, 257))).shape == (0, 9)
    with pytest.raises(ValueError):
        q.linear(np.ones(256))
    with pytest.raises(IndexError):
        q.rows([9])


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("group", [64, 128, 256, 1024, 2048])
def test_sdot_random_against_oracle(native, oracle_lib, int8_kernel, bits, group):
    packed, norms, shape, cb, _ = example(bits, rows=129, dim=257, group=group)
    q = native.NativeCQ(packed, norms, shape, bits, group, cb)
    x = np.random.default_rng(315).normal(size=(5, 257)).astype(np.float32)
    x[0] = 0
    x[1] = 0
    x[1, 0] = 1
    y, d, qa, s = q.sdot_debug(x)
    ry, rd, rq, rs = oracle_lib.sdot_linear(packed, norms, shape, bits, group, cb, x)
    np.testing.assert_array_equal(qa, rq)
    np.testing.assert_array_equal(s, rs)
    np.testing.assert_array_equal(d, rd)
    np.testing.assert_array_equal(y, ry)


@pytest.mark.parametrize("bits", [2, 4])
def test_sdot_rows_independent_of_block(native, int8_kernel, bits):
    """A row's output does not depend on which other rows share the launch
    (the property of tests/test_sdot_row4.py in OpenNeedle)."""
    from openneedle_b200.quantize import codebook, quantize_matrix
    rng = np.random.default_rng(42)
    w = rng.normal(size=(129, 129)).astype(np.float32) * np.arange(1, 130, dtype=np.float32)[:, None]
    packed, norms = quantize_matrix(w, bits, 64)
    cb = codebook(bits, 64)
    block = native.NativeCQ(packed, norms, w.shape, bits, 64, cb)
    for x in (rng.normal(size=129).astype(np.float32), np.zeros(129, np.float32), np.eye(1, 129, dtype=np.float32)[0]):
        whole = block.linear_sdot(x)
        singles = np.concatenate([native.NativeCQ(packed[i:i + 1], norms[i:i + 1], (1, 129), bits, 64, cb).linear_sdot(x)
                                  for i in (0, 1, 64, 127, 128)])
        np.testing.assert_array_equal(whole[[0, 1, 64, 127, 128]], singles)


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("n,k", [(8192, 4096), (11008, 4096), (32768, 512)])
def test_large_shapes_against_oracle(native, oracle_lib, int8_kernel, bits, n, k):
    from openneedle_b200.quantize import synthetic_matrix
    packed, norms, cb = synthetic_matrix(n, k, bits, seed=1000 + n)
    q = native.NativeCQ(packed, norms, (n, k), bits, 128, cb)
    x = np.random.default_rng(1).normal(size=(3, k)).astype(np.float32)
    assert rel_err(q.linear(x), oracle_lib.cq_linear(packed, norms, (n, k), bits, 128, cb, x)) <= FP32_REL_TOL
    y, d, _, _ = q.sdot_debug(x)
    ry, rd, _, _ = oracle_lib.sdot_linear(packed, norms, (n, k), bits, 128, cb, x)
    np.testing.assert_array_equal(d, rd)
    np.testing.assert_array_equal(y, ry)


def test_device_entry_points_match_host(native, int8_kernel):
    import torch
    g = golden("cq4_2048x512.npz")
    q = native.NativeCQ(g["packed"], g["norms"], (2048, 512), 4, 128, g["codebook"])
    x = torch.from_numpy(g["x"][:16]).cuda()
    y = torch.empty(16, 2048, device="cuda")
    q.linear_device(x, y)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y.cpu().numpy(), q.linear(g["x"][:16]))
    q.linear_device(x, y, sdot=True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y.cpu().numpy(), q.linear_sdot(g["x"][:16]))


def test_linear_many_matches_single(native):
    g = golden("cq2_2048x512.npz")
    a = native.NativeCQ(g["packed"], g["norms"], (2048, 512), 2, 128, g["codebook"])
    b = native.NativeCQ(g["packed"][:100], g["norms"][:100], (100, 512), 2, 128, g["codebook"])
    ya, yb = native.linear_many([a, b], g["x"][0])
    np.testing.assert_array_equal(ya, a.linear(g["x"][0]))
    np.testing.assert_array_equal(yb, b.linear(g["x"][0]))


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("sdot", [False, True])
def test_fused_many_matches_single(native, int8_kernel, bits, sdot):
    """Several matrices sharing one input in one fused launch give exactly the
    single-matrix results (the per-row arithmetic does not depend on fusion)."""
    from openneedle_b200.quantize import synthetic_matrix
    mats = []
    for i, (n, k) in enumerate([(1536, 512), (512, 512), (33, 512), (2048, 512)]):
        p, nrm, cb = synthetic_matrix(n, k, bits, seed=50 + i)
        mats.append(native.NativeCQ(p, nrm, (n, k), bits, 128, cb))
    x = np.random.default_rng(3).normal(size=(5, 512)).astype(np.float32)
    outs = native.linear_many_batch(mats, x, sdot=sdot)
    for m, o in zip(mats, outs):
        np.testing.assert_array_equal(o, m.linear_sdot(x) if sdot else m.linear(x))
    # more matrices than one launch holds
    many = [mats[i % 4] for i in range(37)]
    outs = native.linear_many_batch(many, x[:1], sdot=sdot)
    for m, o in zip(many, outs):
        np.testing.assert_array_equal(o, m.linear_sdot(x[:1]) if sdot else m.linear(x[:1]))
    assert native.device_fault() == 0
