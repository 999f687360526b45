"""The decode loop's greedy token (needle2/csrc/engine.cpp:1434-1442) on the GPU
against the oracle's sequential scan: first maximum wins, NaNs never chosen,
0 when the first logit is NaN."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def native():
    from openneedle_b200 import build, native
    build.build()
    return native


@pytest.mark.parametrize("rows,vocab,ld", [(1, 32768, 32768), (7, 1000, 1003), (64, 5, 5), (3, 1, 1),
                                         (8, 1000, 1000), (16, 32768, 32768), (5, 4, 8)])
def test_argmax_matches_oracle(native, oracle_lib, rows, vocab, ld):
    import torch
    rng = np.random.default_rng(rows * 7 + vocab)
    x = rng.normal(size=(rows, ld)).astype(np.float32)
    if rows >= 3 and vocab >= 10:
        x[0, [3, vocab - 1]] = 50.0                 # tie: the first wins
        x[1, 0] = np.nan                            # NaN first: 0
        x[2, 1:vocab:2] = np.nan                    # NaNs never chosen
    if rows >= 4 and vocab >= 10:
        x[3, :] = -np.inf; x[3, 4] = -0.0; x[3, 8] = 0.0   # equal zeros: the first
    if rows >= 5 and vocab >= 10:
        x[4, :] = -np.inf                           # all -inf: 0
    xd = torch.from_numpy(x).cuda()[:, :vocab]
    got = native.argmax_device(xd).cpu().numpy()
    ref = oracle_lib.argmax(np.ascontiguousarray(x[:, :vocab]))
    np.testing.assert_array_equal(got, ref)
