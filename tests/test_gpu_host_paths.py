"""The host-pointer fused call (needle2_cq_linear_many_checked) gives the same
bits whether its buffers are pageable (staged through the library's pinned
buffer) or page-locked (the kernels store the outputs straight into them)."""
import ctypes as ct

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    from openneedle_b200 import build
    from openneedle_b200.native import _library
    build.build()
    return _library()


@pytest.mark.parametrize("sdot", [1, 0])
@pytest.mark.parametrize("batch", [1, 64])
def test_pinned_and_pageable_outputs_agree(lib, sdot, batch):
    import torch
    from util import synthetic_matrix
    mats = [synthetic_matrix(1000 + 8 * i, 512, 4, 128, seed=40 + i) for i in range(3)]
    create = lib.needle2_sdot_create if sdot else lib.needle2_cq_create
    destroy = lib.needle2_sdot_destroy if sdot else lib.needle2_cq_destroy
    hs = [create(p.ctypes.data, n.ctypes.data, p.shape[0], 512, 4, 128, cb.ctypes.data) for p, n, cb in mats]
    assert all(hs)
    try:
        hp = (ct.c_void_p * 3)(*hs)
        x = np.random.default_rng(batch).normal(size=(batch, 512)).astype(np.float32)
        outs = [m[0].shape[0] for m in mats]
        ys_np = [np.empty((batch, o), np.float32) for o in outs]
        assert lib.needle2_cq_linear_many_checked(hp, 3, x.ctypes.data, (ct.c_void_p * 3)(*[a.ctypes.data for a in ys_np]),
                                                  batch, sdot) == 0
        xp = torch.from_numpy(x).pin_memory()
        ys_p = [torch.empty(batch, o, pin_memory=True) for o in outs]
        assert lib.needle2_cq_linear_many_checked(hp, 3, xp.data_ptr(), (ct.c_void_p * 3)(*[t.data_ptr() for t in ys_p]),
                                                  batch, sdot) == 0
        for a, t in zip(ys_np, ys_p):
            np.testing.assert_array_equal(a, t.numpy())
    finally:
        for h in hs:
            destroy(h)
