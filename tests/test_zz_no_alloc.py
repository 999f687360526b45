"""needle2_sdot_linear_device_noalloc (no device allocation, fixed per-device
scratch) against needle2_sdot_linear_device on the same inputs.  Both run the
same quantiser and int8 GEMV, so outputs must agree exactly (tolerance 0)."""
import ctypes as ct

import numpy as np
import pytest

from util import golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    from openneedle_b200 import build, native
    build.build()
    lib = native._library()
    lib.needle2_sdot_linear_device_noalloc.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_void_p, ct.c_int, ct.c_void_p]
    lib.needle2_sdot_linear_device_noalloc.restype = ct.c_int
    return lib


def _sdot_handle(native, bits):
    g = golden(f"cq{bits}_2048x512.npz")
    q = native.DeviceMatrix(g["packed"], g["norms"], (2048, 512), bits, 128, g["codebook"])
    return q, q.sdot.ptr, g


@pytest.mark.parametrize("bits", [2, 4])
def test_noalloc_matches_device_entry_twice(lib, bits):
    import torch
    from openneedle_b200 import native
    q, handle, g = _sdot_handle(native, bits)
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(77 + bits)
    for batch in (16, 3):   # two calls in a row, different batches and inputs
        x = torch.from_numpy(rng.normal(size=(batch, 512)).astype(np.float32)).cuda()
        ref = torch.empty(batch, 2048, device="cuda")
        got = torch.full((batch, 2048), float("nan"), device="cuda")
        assert lib.needle2_sdot_linear_device(handle, x.data_ptr(), ref.data_ptr(), batch, stream) == 0
        assert lib.needle2_sdot_linear_device_noalloc(handle, x.data_ptr(), got.data_ptr(), batch, stream) == 0, \
            lib.needle2_b200_error().decode()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(got.cpu().numpy(), ref.cpu().numpy())
    # the golden activations give the golden SDOT outputs as well
    x = torch.from_numpy(g["x"][:4]).cuda()
    got = torch.empty(4, 2048, device="cuda")
    assert lib.needle2_sdot_linear_device_noalloc(handle, x.data_ptr(), got.data_ptr(), 4, stream) == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(got.cpu().numpy(), q.sdot(g["x"][:4]))


def test_noalloc_rejects_oversized_batch(lib):
    import torch
    from openneedle_b200 import native
    _, handle, _ = _sdot_handle(native, 4)
    batch = (1 << 20) // 512 + 1   # one row beyond the 1 MiB activation scratch
    x = torch.zeros(batch, 512, device="cuda")
    y = torch.zeros(batch, 2048, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.needle2_sdot_linear_device_noalloc(handle, x.data_ptr(), y.data_ptr(), batch, stream) == -1
    assert b"no-allocation scratch" in lib.needle2_b200_error()
    assert lib.needle2_sdot_linear_device_noalloc(handle, x.data_ptr(), y.data_ptr(), 0, stream) == 0
