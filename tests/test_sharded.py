"""Host logic of the N-sharded matrix (openneedle_b200/sharded.py) on CPU:
row spans, zero-norm padding, and reassembly of gathered shards, with two
gloo ranks standing in for GPUs (each rank's shard computed as a dense
product of its dequantised rows)."""
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from util import ref_quantize, synthetic_matrix
from openneedle_b200.sharded import assemble, shard_layout, shard_matrix


@pytest.mark.parametrize("out,world", [(14336, 8), (14336, 2), (1000, 2), (1001, 4), (5, 8), (4096, 3)])
def test_shard_layout_covers_rows(out, world):
    ns, spans = shard_layout(out, world)
    assert ns % 4 == 0 and ns * world >= out
    assert spans[0][0] == 0 and spans[-1][1] == out
    for (a, b), (c, d) in zip(spans, spans[1:]):
        assert b == c and 0 <= b - a <= ns
    if out == 14336 and world == 8:
        assert ns == 1792


def test_shard_padding_rows_are_zero():
    packed, norms, cb = synthetic_matrix(1001, 256, 4, 128, seed=2)
    ns, spans = shard_layout(1001, 4)
    p, n = shard_matrix(packed, norms, 1001, 3, 4)
    r0, r1 = spans[3]
    assert p.shape == (ns, packed.shape[1]) and n.shape == (ns, norms.shape[1])
    np.testing.assert_array_equal(p[: r1 - r0], packed[r0:r1])
    assert not p[r1 - r0:].any() and not n[r1 - r0:].astype(np.float32).any()
    w = ref_quantize().dequantize_matrix(p, n, (ns, 256), 4, 128, cb)
    assert not w[r1 - r0:].any()   # zero norms give zero rows


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out, k, q):
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        packed, norms, cb = synthetic_matrix(out, k, 4, 128, seed=3)
        x = np.random.default_rng(9).normal(size=(6, k)).astype(np.float64)
        p, n = shard_matrix(packed, norms, out, rank, world)
        ns = p.shape[0]
        y = x @ ref_quantize().dequantize_matrix(p, n, (ns, k), 4, 128, cb).astype(np.float64).T
        parts = [torch.empty(6, ns, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(y)))
        full = assemble(torch.stack(parts), out).numpy()
        ref = x @ ref_quantize().dequantize_matrix(packed, norms, (out, k), 4, 128, cb).astype(np.float64).T
        q.put((rank, full.shape == ref.shape and bool(np.allclose(full, ref, rtol=1e-12, atol=1e-12))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("out,world", [(1000, 2), (1001, 2)])
def test_gloo_two_ranks_gather_equals_full_matrix(out, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, out, 256, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = dict(q.get(timeout=5) for _ in range(world))
    assert all(p.exitcode == 0 for p in procs)
    assert all(results[r] for r in range(world))
