"""The int8 (SDOT) prefill GEMM on the tensor cores (batches of 64+ rows, group
128) against the oracle and against the GEMV path: outputs bit-exact."""
import ctypes as ct

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def native():
    from openneedle_b200 import build, native
    build.build()
    return native


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("n,k,m", [(300, 512, 64), (301, 512, 130), (1000, 1024, 257), (2048, 512, 2048)])
def test_prefill_gemm_matches_oracle(native, oracle_lib, bits, n, k, m):
    from util import synthetic_matrix
    packed, norms, cb = synthetic_matrix(n, k, bits, seed=700 + n + bits)
    q = native.DeviceMatrix(packed, norms, (n, k), bits, 128, cb)
    x = np.random.default_rng(m + k).normal(size=(m, k)).astype(np.float32)
    x[3] = 0                                   # an all-zero row (scale 1)
    y = q.sdot(x)
    ry, _, _, _ = oracle_lib.sdot_linear(packed, norms, (n, k), bits, 128, cb, x)
    np.testing.assert_array_equal(y, ry)


@pytest.mark.parametrize("bits", [2, 4])
def test_prefill_gemm_matches_gemv_at_config3_width(native, bits):
    """Config-3 width (N = 8192, K = 4096): the GEMM and the GEMV path (the
    no-allocation entry always runs the GEMV) agree bit for bit."""
    import torch
    from util import synthetic_matrix
    n, k, m = 8192, 4096, 512
    packed, norms, cb = synthetic_matrix(n, k, bits, seed=91 + bits)
    q = native.DeviceMatrix(packed, norms, (n, k), bits, 128, cb)
    h = q.sdot.ptr
    lib = native._library()
    lib.needle2_sdot_linear_device_noalloc.argtypes = [ct.c_void_p] * 3 + [ct.c_int, ct.c_void_p]
    lib.needle2_sdot_linear_device_noalloc.restype = ct.c_int
    x = torch.from_numpy(np.random.default_rng(5).normal(size=(m, k)).astype(np.float32)).cuda()
    y_gemm = torch.empty(m, n, device="cuda")
    y_gemv = torch.empty(m, n, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.needle2_sdot_linear_device(h, x.data_ptr(), y_gemm.data_ptr(), m, s) == 0
    for r0 in range(0, m, 256):
        assert lib.needle2_sdot_linear_device_noalloc(h, x[r0:].data_ptr(), y_gemv[r0:].data_ptr(), 256, s) == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y_gemm.cpu().numpy(), y_gemv.cpu().numpy())
    assert native.device_fault() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("n,k,m,group", [(300, 512, 64, 128), (301, 512, 130, 128), (1000, 1024, 257, 128),
                                         (2048, 512, 2048, 128), (520, 640, 96, 64)])
def test_fp32_prefill_gemm_matches_oracle(native, oracle_lib, bits, n, k, m, group):
    """FP32 mode from 64 rows on runs the bf16 hi/lo tensor-core GEMM; it must stay
    within the FP32 tolerance of the reference's per-group FP32 sums."""
    from util import FP32_REL_TOL, rel_err, synthetic_matrix
    packed, norms, cb = synthetic_matrix(n, k, bits, group, seed=900 + n + bits)
    q = native.DeviceMatrix(packed, norms, (n, k), bits, group, cb)
    x = np.random.default_rng(m + k + 1).normal(size=(m, k)).astype(np.float32)
    x[5] = 0
    y = q.fp32(x)
    ref = oracle_lib.cq_linear(packed, norms, (n, k), bits, group, cb, x)
    assert rel_err(y, ref) <= FP32_REL_TOL
    # rows are independent of the batch they run in: the GEMV's result for the
    # first 16 rows agrees within the same tolerance
    assert rel_err(y[:16], q.fp32(x[:16])) <= FP32_REL_TOL


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("n,k", [(8192, 2048), (8192, 4096), (11008, 2048), (11008, 4096)])
def test_fp32_prefill_gemm_config3_sizes(native, oracle_lib, bits, n, k):
    """Config 3's FP32-mode shapes (M = 2048 activation rows, K up to 4096, N up
    to 11008): the bf16 hi/lo GEMM's error grows with K, so it is checked at the
    full widths.  The oracle runs on a sample of 24 activation rows (all N
    outputs of each), spread over the batch and its tiles, including an
    all-zero row; the bar is max|y - y_ref| / max|y_ref| <= 1e-4 per tensor."""
    from util import FP32_REL_TOL, rel_err, synthetic_matrix
    m = 2048
    packed, norms, cb = synthetic_matrix(n, k, bits, 128, seed=30 + n + k + bits)
    q = native.DeviceMatrix(packed, norms, (n, k), bits, 128, cb)
    x = np.random.default_rng(n + k).normal(size=(m, k)).astype(np.float32)
    x[1000] = 0
    y = q.fp32(x)
    sample = np.array([0, 1, 127, 128, 255, 511, 640, 777, 1000, 1023, 1024, 1151, 1200, 1337, 1500, 1535,
                       1536, 1663, 1800, 1919, 1920, 2000, 2046, 2047])
    ref = oracle_lib.cq_linear(packed, norms, (n, k), bits, 128, cb, x[sample])
    err = rel_err(y[sample], ref)
    print(f"config-3 FP32 GEMM CQ{bits} N={n} K={k}: max rel err {err:.3e}")
    assert err <= FP32_REL_TOL
    assert not y[1000].any()


@pytest.mark.gpu
@pytest.mark.parametrize("m", [64, 128, 200, 1024])
def test_fp32_decode_gemm_fused_projections(native, oracle_lib, m):
    """Decode-sized FP32 GEMMs (a few hundred rows, K = 512): config 5's fused
    Q/K/V/gate projections (N = 512, 256, 256, 512, CQ2) and its out
    projection.  These launches split K over a cluster of CTAs and add the
    partial tiles in a fixed order; outputs stay within the FP32 tolerance of
    the oracle on every matrix and are identical from call to call."""
    from util import FP32_REL_TOL, rel_err, synthetic_matrix
    from openneedle_b200.native import linear_many_batch
    k = 512
    shapes = [512, 256, 256, 512]
    mats, raw = [], []
    for i, n in enumerate(shapes):
        packed, norms, cb = synthetic_matrix(n, k, 2, 128, seed=4000 + 17 * i + n)
        mats.append(native.DeviceMatrix(packed, norms, (n, k), 2, 128, cb))
        raw.append((packed, norms, cb, n))
    x = np.random.default_rng(m).normal(size=(m, k)).astype(np.float32)
    x[m // 2] = 0
    ys = linear_many_batch(mats, x)
    again = linear_many_batch(mats, x)
    sample = np.unique(np.array([0, 1, 31, 63, m // 2, m - 2, m - 1]))
    for (packed, norms, cb, n), y, y2 in zip(raw, ys, again):
        ref = oracle_lib.cq_linear(packed, norms, (n, k), 2, 128, cb, x[sample])
        assert rel_err(y[sample], ref) <= FP32_REL_TOL
        np.testing.assert_array_equal(y, y2)
        assert not y[m // 2].any()
    # the out projection alone (one 512-wide matrix: a wider K split)
    packed, norms, cb, n = raw[0]
    y = mats[0].fp32(x)
    ref = oracle_lib.cq_linear(packed, norms, (n, k), 2, 128, cb, x[sample])
    assert rel_err(y[sample], ref) <= FP32_REL_TOL
