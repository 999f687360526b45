"""Pins the CPU oracle to the reference (CPU only).

The oracle (oracle/cq_oracle.c) restates the reference's x86 arithmetic in the
same operation order, so it must reproduce the golden vectors — produced by
the reference itself — bit for bit.  When the reference sources are present
(oracle/_ref), randomized cases modelled on the reference's own tests are
compared as well.
"""
import numpy as np
import pytest

from util import example, golden, sha



@pytest.mark.parametrize("bits", [2, 4])
def test_oracle_fp32_matches_golden(oracle_lib, bits):
    g = golden(f"cq{bits}_2048x512.npz")
    shape = (2048, 512)
    y1 = oracle_lib.cq_linear(g["packed"], g["norms"], shape, bits, 128, g["codebook"], g["x"][:1])
    y4 = oracle_lib.cq_linear(g["packed"], g["norms"], shape, bits, 128, g["codebook"], g["x"][:4])
    np.testing.assert_array_equal(y1, g["y_fp32_m1"])
    np.testing.assert_array_equal(y4, g["y_fp32_m4"])
    rows = oracle_lib.cq_rows(g["packed"], g["norms"], shape, bits, 128, g["codebook"], g["rows_ids"])
    np.testing.assert_array_equal(rows, g["rows"])


@pytest.mark.parametrize("bits", [2, 4])
def test_oracle_sdot_matches_golden(oracle_lib, bits):
    g = golden(f"cq{bits}_2048x512.npz")
    y, d, q, s = oracle_lib.sdot_linear(g["packed"], g["norms"], (2048, 512), bits, 128, g["codebook"], g["x"])
    np.testing.assert_array_equal(q, g["sdot_q"])
    np.testing.assert_array_equal(s, g["sdot_scales"])
    np.testing.assert_array_equal(d[:1], g["sdot_partials_m1"])
    np.testing.assert_array_equal(y[:4], g["sdot_y_m4"])
    for m in (1, 4, 16, 64):
        assert sha(d[:m]) == str(g[f"sdot_partials_sha_m{m}"])
        assert sha(y[:m]) == str(g[f"sdot_y_sha_m{m}"])


@pytest.mark.parametrize("tag", ["win", "full"])
def test_oracle_kv_and_attention_match_golden(oracle_lib, tag):
    g = golden("attention_i8.npz")
    H, KV, HD, maxseq, window, prefix, n = (int(v) for v in g[f"{tag}_geom"])
    ki, vi, ks, vs = oracle_lib.kv_quantize(g[f"{tag}_k"], g[f"{tag}_v"], KV, HD)
    cap = window + prefix if window else maxseq
    cache = {"keys_i8": np.zeros((cap, KV * HD), np.int8), "values_i8": np.zeros((cap, KV * HD), np.int8),
             "k_scales": np.zeros((cap, KV), np.float32), "v_scales": np.zeros((cap, KV), np.float32)}
    for t in range(n):
        s = oracle_lib.cache_slot(t, prefix, window)
        cache["keys_i8"][s], cache["values_i8"][s], cache["k_scales"][s], cache["v_scales"][s] = ki[t], vi[t], ks[t], vs[t]
    np.testing.assert_array_equal(cache["keys_i8"], g[f"{tag}_keys_i8"])
    np.testing.assert_array_equal(cache["values_i8"], g[f"{tag}_values_i8"])
    np.testing.assert_array_equal(cache["k_scales"], g[f"{tag}_k_scales"])
    np.testing.assert_array_equal(cache["v_scales"], g[f"{tag}_v_scales"])
    for i, p in enumerate(g[f"{tag}_qpos"]):
        out = oracle_lib.attention_i8(cache["keys_i8"], cache["values_i8"], cache["k_scales"], cache["v_scales"],
                                      H, KV, HD, int(p), prefix, window, g[f"{tag}_q"][i])
        np.testing.assert_array_equal(out, g[f"{tag}_out"][i])


def test_oracle_prefill_is_store_then_attend(oracle_lib):
    """Prefill = per token store, then attend (engine.cpp:1170-1210): equal to
    importing the whole cache up to each token and attending there."""
    g = golden("attention_i8.npz")
    H, KV, HD, maxseq, window, prefix, n = (int(v) for v in g["win_geom"])
    cap = window + prefix
    cache = {"keys_i8": np.zeros((cap, KV * HD), np.int8), "values_i8": np.zeros((cap, KV * HD), np.int8),
             "k_scales": np.zeros((cap, KV), np.float32), "v_scales": np.zeros((cap, KV), np.float32)}
    rng = np.random.default_rng(5)
    q = rng.normal(size=(n, H * HD)).astype(np.float32)
    out = oracle_lib.attention_prefill_i8(cache, H, KV, HD, 0, prefix, window, q, g["win_k"], g["win_v"])
    np.testing.assert_array_equal(cache["keys_i8"], g["win_keys_i8"])
    # last token attends over the final cache state
    last = oracle_lib.attention_i8(g["win_keys_i8"], g["win_values_i8"], g["win_k_scales"], g["win_v_scales"],
                                   H, KV, HD, n - 1, prefix, window, q[-1])
    np.testing.assert_array_equal(out[-1], last)


def test_activation_quant_a8(oracle_lib):
    x = np.random.default_rng(3).normal(size=512).astype(np.float32)
    y = oracle_lib.activation_quant(x, 8)
    a = np.max(np.abs(x))
    scale = np.float32(a / np.float32(127))
    np.testing.assert_array_equal(y, np.clip(np.rint(x / scale), -128, 127).astype(np.float32) * scale)
    np.testing.assert_array_equal(oracle_lib.activation_quant(np.zeros(8, np.float32), 8), np.zeros(8, np.float32))


# ---------------------------------------------------------------- reference

from oracle import oracle as _O  # noqa: E402

needs_ref = pytest.mark.skipif(not _O.ref_available(), reason="reference build (oracle/_ref) unavailable")


@needs_ref
@pytest.mark.reference
@pytest.mark.parametrize("bits", [2, 3, 4, 5])
@pytest.mark.parametrize("group", [8, 64, 128])
def test_oracle_fp32_matches_reference_random(oracle_lib, bits, group):
    packed, norms, shape, cb, dense = example(bits, dim=257, group=group)
    x = np.random.default_rng(9).normal(size=(2, 3, 257)).astype(np.float32)
    ref = oracle_lib.ref_cq_linear(packed, norms, shape, bits, group, cb, x)
    np.testing.assert_array_equal(oracle_lib.cq_linear(packed, norms, shape, bits, group, cb, x), ref)
    np.testing.assert_allclose(ref, x @ dense.T, atol=3e-6, rtol=2e-5)
    ids = np.array([8, 2, 0, 2])
    np.testing.assert_array_equal(oracle_lib.cq_rows(packed, norms, shape, bits, group, cb, ids),
                                  oracle_lib.ref_cq_rows(packed, norms, shape, bits, group, cb, ids))


@needs_ref
@pytest.mark.reference
@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("group", [64, 128])
def test_oracle_sdot_matches_reference_random(oracle_lib, bits, group):
    packed, norms, shape, cb, _ = example(bits, dim=257, group=group)
    x = np.random.default_rng(315).normal(size=(5, 257)).astype(np.float32)
    x[0] = 0
    x[1] = 0
    x[1, 0] = 1
    mine = oracle_lib.sdot_linear(packed, norms, shape, bits, group, cb, x)
    ref = oracle_lib.ref_sdot(packed, norms, shape, bits, group, cb, x)
    for a, b in zip(mine, ref):
        np.testing.assert_array_equal(a, b)


def test_argmax_first_max_and_nans(oracle_lib):
    """The oracle's greedy scan against the reference loop written out in Python
    (engine.cpp:1434-1442): ties, NaNs, infinities and signed zeros."""
    def loop(row):
        best, max_v = 0, row[0]
        for i in range(1, len(row)):
            if row[i] > max_v:
                max_v, best = row[i], i
        return best
    rng = np.random.default_rng(8)
    rows = [rng.normal(size=1000).astype(np.float32) for _ in range(4)]
    rows[0][[10, 500]] = 9.0                        # a tie: the first wins
    rows[1][0] = np.nan                             # NaN first: stays 0
    rows[2][[3, 7]] = np.nan; rows[2][900] = np.inf # later NaNs skipped
    rows[3][:] = -np.inf; rows[3][5] = -0.0; rows[3][6] = 0.0   # +0 is not > -0
    for r in rows:
        assert oracle_lib.argmax(r)[0] == loop(r.tolist())
