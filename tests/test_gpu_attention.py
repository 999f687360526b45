"""GPU parity of the INT8 KV store and attention kernels.

Caches are compared bit for bit (int8 values and FP32 scales, in the
reference's own layout via KVCache.export); attention outputs within the FP32
tolerance max|out - ref| / max|ref| <= 1e-4 (FP32_REL_TOL) against the oracle
restatement of Engine::compute_attention and against golden vectors produced
by the reference itself.
"""
import numpy as np
import pytest

from util import FP32_REL_TOL, golden, rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def attention():
    from openneedle_b200 import attention, build
    build.build()
    return attention


def oracle_cache(cap, kvheads, hd):
    return {"keys_i8": np.zeros((cap, kvheads * hd), np.int8), "values_i8": np.zeros((cap, kvheads * hd), np.int8),
            "k_scales": np.zeros((cap, kvheads), np.float32), "v_scales": np.zeros((cap, kvheads), np.float32)}


def oracle_store(O, cache, k, v, positions, kvheads, hd, prefix, window):
    ki, vi, ks, vs = O.kv_quantize(k, v, kvheads, hd)
    for t, p in enumerate(positions):
        s = O.cache_slot(int(p), prefix, window)
        cache["keys_i8"][s], cache["values_i8"][s] = ki[t], vi[t]
        cache["k_scales"][s], cache["v_scales"][s] = ks[t], vs[t]


def assert_cache_equal(got, want):
    for name in ("keys_i8", "values_i8", "k_scales", "v_scales"):
        np.testing.assert_array_equal(got[name], want[name], err_msg=name)


@pytest.mark.parametrize("tag", ["win", "full"])
def test_golden_cache_and_attention(attention, tag):
    g = golden("attention_i8.npz")
    H, KV, HD, maxseq, window, prefix, n = (int(v) for v in g[f"{tag}_geom"])
    kv = attention.KVCache(3, H, KV, HD, maxseq, window, prefix)
    kv.set_prefix(g[f"{tag}_k"][:prefix], g[f"{tag}_v"][:prefix])
    for t in range(prefix, n):
        kv.store([1], [t], g[f"{tag}_k"][t:t + 1], g[f"{tag}_v"][t:t + 1])
    assert_cache_equal(kv.export(1), {k: g[f"{tag}_{k}"] for k in ("keys_i8", "values_i8", "k_scales", "v_scales")})
    for i, p in enumerate(g[f"{tag}_qpos"]):
        out = kv.query([1], [int(p)], g[f"{tag}_q"][i:i + 1])[0]
        assert rel_err(out, g[f"{tag}_out"][i]) <= FP32_REL_TOL


@pytest.mark.parametrize("heads,kvheads,hd,window,prefix", [
    (8, 4, 64, 0, 24), (8, 4, 64, 16, 7), (8, 8, 64, 0, 5), (6, 2, 38, 17, 7), (6, 2, 32, 0, 0), (4, 1, 128, 9, 3),
    (4, 2, 128, 0, 5), (8, 2, 64, 12, 5), (16, 2, 64, 0, 3)])
def test_decode_sessions_against_oracle(attention, oracle_lib, heads, kvheads, hd, window, prefix):
    O = oracle_lib
    rng = np.random.default_rng(11)
    S, steps, maxseq = 3, 40, 96
    kv = attention.KVCache(S, heads, kvheads, hd, maxseq, window, prefix)
    cap = kv.capacity
    pk = rng.normal(size=(prefix, kvheads * hd)).astype(np.float32)
    pv = rng.normal(size=(prefix, kvheads * hd)).astype(np.float32)
    if prefix:
        kv.set_prefix(pk, pv)
    caches = [oracle_cache(cap, kvheads, hd) for _ in range(S)]
    for c in caches:
        oracle_store(O, c, pk, pv, range(prefix), kvheads, hd, prefix, window)
    for step in range(steps):
        pos = prefix + step
        ids = [s for s in range(S) if (step + s) % 4 != 3]   # sessions skip steps: positions differ
        positions = [prefix + sum(1 for t in range(step) if (t + s) % 4 != 3) for s in ids]
        q = rng.normal(size=(len(ids), heads * hd)).astype(np.float32)
        k = rng.normal(size=(len(ids), kvheads * hd)).astype(np.float32) * (1 + step % 3)
        v = rng.normal(size=(len(ids), kvheads * hd)).astype(np.float32)
        if step == 5:
            k[0] = 0   # an all-zero head: scale 1, codes 0
        out = kv.decode(ids, positions, q, k, v)
        for j, s in enumerate(ids):
            oracle_store(O, caches[s], k[j:j + 1], v[j:j + 1], [positions[j]], kvheads, hd, prefix, window)
            ref = O.attention_i8(caches[s]["keys_i8"], caches[s]["values_i8"], caches[s]["k_scales"],
                                 caches[s]["v_scales"], heads, kvheads, hd, positions[j], prefix, window, q[j])
            assert rel_err(out[j], ref) <= FP32_REL_TOL, (step, s)
        del pos
    for s in range(S):
        assert_cache_equal(kv.export(s), caches[s])


@pytest.mark.parametrize("window,tokens", [(0, 20), (16, 20), (16, 7), (40, 33)])
def test_prefill_against_oracle(attention, oracle_lib, window, tokens):
    O = oracle_lib
    H, KV, HD, prefix, maxseq = 8, 4, 64, 6, 128
    rng = np.random.default_rng(5)
    S = 3
    kv = attention.KVCache(S, H, KV, HD, maxseq, window, prefix)
    pk = rng.normal(size=(prefix, KV * HD)).astype(np.float32)
    pv = rng.normal(size=(prefix, KV * HD)).astype(np.float32)
    kv.set_prefix(pk, pv)
    caches = [oracle_cache(kv.capacity, KV, HD) for _ in range(S)]
    for c in caches:
        oracle_store(O, c, pk, pv, range(prefix), KV, HD, prefix, window)
    starts = np.array([prefix] * S, np.int32)
    for chunk in range(2):
        q = rng.normal(size=(S, tokens, H * HD)).astype(np.float32)
        k = rng.normal(size=(S, tokens, KV * HD)).astype(np.float32)
        v = rng.normal(size=(S, tokens, KV * HD)).astype(np.float32)
        out = kv.prefill(np.arange(S), starts, q, k, v)
        for s in range(S):
            ref = O.attention_prefill_i8(caches[s], H, KV, HD, int(starts[s]), prefix, window, q[s], k[s], v[s])
            assert rel_err(out[s], ref) <= FP32_REL_TOL, (chunk, s)
        starts += tokens
    for s in range(S):
        assert_cache_equal(kv.export(s), caches[s])


def test_config4_scale_prefix_prefill_decode(attention, oracle_lib):
    """256 sessions sharing a 384-token prefix: a 128-token prefill on top of it,
    then decode steps; sampled sessions against the oracle, and one session's
    decode at 4096 positions."""
    O = oracle_lib
    H, KV, HD, P, S, T, maxseq = 8, 4, 64, 384, 256, 128, 4096
    rng = np.random.default_rng(0)
    kv = attention.KVCache(S, H, KV, HD, maxseq, 0, P)
    pk = rng.normal(size=(P, KV * HD)).astype(np.float32)
    pv = rng.normal(size=(P, KV * HD)).astype(np.float32)
    kv.set_prefix(pk, pv)
    q = rng.normal(size=(S, T, H * HD)).astype(np.float32)
    k = rng.normal(size=(S, T, KV * HD)).astype(np.float32)
    v = rng.normal(size=(S, T, KV * HD)).astype(np.float32)
    out = kv.prefill(np.arange(S), np.full(S, P, np.int32), q, k, v)
    sample = [0, 1, 127, 255]
    caches = {}
    for s in sample:
        c = oracle_cache(maxseq, KV, HD)
        oracle_store(O, c, pk, pv, range(P), KV, HD, P, 0)
        ref = O.attention_prefill_i8(c, H, KV, HD, P, P, 0, q[s], k[s], v[s])
        assert rel_err(out[s], ref) <= FP32_REL_TOL, s
        caches[s] = c
    # decode 4 steps for all sessions
    for step in range(4):
        pos = np.full(S, P + T + step, np.int32)
        qd = rng.normal(size=(S, H * HD)).astype(np.float32)
        kd = rng.normal(size=(S, KV * HD)).astype(np.float32)
        vd = rng.normal(size=(S, KV * HD)).astype(np.float32)
        od = kv.decode(np.arange(S), pos, qd, kd, vd)
        for s in sample:
            oracle_store(O, caches[s], kd[s:s + 1], vd[s:s + 1], [int(pos[s])], KV, HD, P, 0)
            ref = O.attention_i8(caches[s]["keys_i8"], caches[s]["values_i8"], caches[s]["k_scales"],
                                 caches[s]["v_scales"], H, KV, HD, int(pos[s]), P, 0, qd[s])
            assert rel_err(od[s], ref) <= FP32_REL_TOL
    for s in sample:
        assert_cache_equal(kv.export(s), caches[s])
    # long context: fill session 7 to 4095 positions and query at 4095
    n = maxseq - P - 1
    kl = rng.normal(size=(1, n, KV * HD)).astype(np.float32)
    vl = rng.normal(size=(1, n, KV * HD)).astype(np.float32)
    ql = rng.normal(size=(1, n, H * HD)).astype(np.float32)
    kv.prefill([7], [P], ql, kl, vl)
    c = oracle_cache(maxseq, KV, HD)
    oracle_store(O, c, pk, pv, range(P), KV, HD, P, 0)
    oracle_store(O, c, kl[0], vl[0], range(P, P + n), KV, HD, P, 0)
    qq = rng.normal(size=(1, H * HD)).astype(np.float32)
    kk = rng.normal(size=(1, KV * HD)).astype(np.float32)
    od = kv.decode([7], [maxseq - 1], qq, kk, kk)
    oracle_store(O, c, kk, kk, [maxseq - 1], KV, HD, P, 0)
    ref = O.attention_i8(c["keys_i8"], c["values_i8"], c["k_scales"], c["v_scales"], H, KV, HD, maxseq - 1, P, 0, qq[0])
    assert rel_err(od[0], ref) <= FP32_REL_TOL
    assert_cache_equal(kv.export(7), c)


def test_validation_errors(attention):
    kv = attention.KVCache(2, 8, 4, 64, 32, 0, 4)
    z = np.zeros((1, 256), np.float32)
    with pytest.raises(RuntimeError, match="shared prefix not set"):
        kv.store([0], [4], z, z)
    kv.set_prefix(np.zeros((4, 256), np.float32), np.zeros((4, 256), np.float32))
    with pytest.raises(RuntimeError, match="inside the shared prefix"):
        kv.store([0], [3], z, z)
    with pytest.raises(RuntimeError, match="session id outside"):
        kv.store([2], [4], z, z)
    with pytest.raises(RuntimeError, match="maximum context"):
        kv.store([0], [32], z, z)
    with pytest.raises(RuntimeError, match="twice"):
        kv.store([0, 0], [4, 5], np.zeros((2, 256), np.float32), np.zeros((2, 256), np.float32))
    with pytest.raises(MemoryError, match="multiple of kvheads|at most 8"):
        attention.KVCache(1, 18, 2, 64, 8)
