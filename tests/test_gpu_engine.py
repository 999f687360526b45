"""The whole Needle-2 forward on the GPU against the reference engine.

Each plan runs twice through the reference's unchanged Python layer
(needle2/native.py NativeEngine): once on the reference's own CPU build
(oracle/_ref, compiled from its sources) and once on libneedle2_b200.so.  The
bar for logits and hidden states is max|y - y_ref| / max|y_ref| <= 1e-4 per
tensor; greedy tokens must be identical (the top-2 margin of a diverging step
is reported, since ties below FP32 rounding cannot be decided).  Weights are
the reference's NeedleModel default init packed by its quantizer
(tests/engine_models.py)."""
import numpy as np
import pytest

from engine_harness import rel, run_plan, top2_margin

pytestmark = pytest.mark.gpu
TOL = 1e-4


@pytest.fixture(scope="module")
def env(tmp_path_factory):
    from oracle import oracle as O
    if O.reference_package() is None or not O.ref_available():
        pytest.skip("reference package or oracle/_ref unavailable")
    from openneedle_b200 import build
    lib = build.build()
    return tmp_path_factory.mktemp("engine"), O.REF_LIB, lib


def _archive(env, name, cfg, seed):
    from engine_models import build_archive, save_archive
    path = env[0] / f"{name}.npz"
    if not path.exists():
        meta, records = build_archive(cfg, seed=seed)
        save_archive(path, meta, records)
    return path


def _both(env, path, plan, tag):
    d, ref_lib, lib = env
    return run_plan(path, plan, ref_lib, d, f"{tag}_ref"), run_plan(path, plan, lib, d, f"{tag}_gpu")


def _compare(ref, gpu, tol=TOL, what=""):
    worst = 0.0
    for key, a in ref.items():
        if key == "library":
            continue
        b = gpu[key]
        if key.endswith("_tokens"):
            if not np.array_equal(a, b):
                raise AssertionError(f"{what} {key}: greedy tokens differ {a} vs {b}")
            continue
        e = rel(b, a)
        worst = max(worst, e)
        assert e <= tol, f"{what} {key}: rel err {e:.3e}"
    return worst


def _tokens(n, vocab, seed):
    return [int(t) for t in np.random.default_rng(seed).integers(1, vocab, n)]


@pytest.mark.parametrize("window", [0, 5])
@pytest.mark.parametrize("kv", ["fp32", "int8"])
@pytest.mark.parametrize("abits", [0, 8])
def test_engine_matches_reference(env, window, kv, abits):
    from engine_models import tiny_config
    path = _archive(env, f"tiny_w{window}", tiny_config(window), 117)
    ids = _tokens(24, 61, 5 + window)
    plan = [{"op": "engine", "kv": kv, "abits": abits}]
    for prefix in (0, 3):
        plan += [{"op": "reset", "prefix": prefix}, {"op": "prefill", "tokens": ids[:18]}]
        plan += [{"op": "step", "token": t, "hidden": True} for t in ids[18:]]
        plan += [{"op": "decode", "first": ids[-1], "max_new": 6}, {"op": "kv_bytes"}]
    ref, gpu = _both(env, path, plan, f"w{window}_{kv}_{abits}")
    for k in [k for k in ref if k.endswith("_kv_bytes")]:
        ref.pop(k), gpu.pop(k)
    worst = _compare(ref, gpu, what=f"window {window} kv {kv} abits {abits}")
    print(f"engine window={window} kv={kv} abits={abits}: max rel err {worst:.3e}")


def test_engine_prefix_snapshot_and_candidates(env):
    from engine_models import tiny_config
    path = _archive(env, "tiny_w5", tiny_config(5), 117)
    ids = _tokens(20, 61, 9)
    plan = [{"op": "engine", "kv": "int8"}, {"op": "reset", "prefix": 4}, {"op": "prefill", "tokens": ids[:4]},
            {"op": "cache_prefix"}, {"op": "prefill", "tokens": ids[4:14]}, {"op": "reset_to_prefix"},
            {"op": "prefill", "tokens": ids[4:14]}, {"op": "reset_to_prefix"},
            {"op": "step_candidates", "token": ids[4], "candidates": [3, 7, 11, 60, 2]},
            {"op": "step", "token": ids[5]}]
    ref, gpu = _both(env, path, plan, "snapshot")
    _compare(ref, gpu, what="snapshot")
    np.testing.assert_array_equal(gpu["4_logits"], gpu["6_logits"])   # restored prefix: bit for bit


def test_engine_torch_prefill_import(env):
    from engine_models import tiny_config
    path = _archive(env, "tiny_w0", tiny_config(0), 117)
    ids = _tokens(16, 61, 13)
    plan = [{"op": "engine", "kv": "int8"}, {"op": "reset", "prefix": 0},
            {"op": "prefill", "tokens": ids[:12], "last_only": True, "backend": "torch"}]
    plan += [{"op": "step", "token": t} for t in ids[12:]]
    ref, gpu = _both(env, path, plan, "import")
    _compare(ref, gpu, what="torch-prefill import")


def test_engine_sdot_matches_reference(env):
    """int8 matmuls (per-group int8 activations, exact int32 dots) across the whole forward."""
    from engine_models import tiny_config
    path = _archive(env, "tiny_w0", tiny_config(0), 117)
    ids = _tokens(20, 61, 21)
    plan = [{"op": "engine", "kv": "int8", "matmul": "sdot"}, {"op": "prefill", "tokens": ids[:16]}]
    plan += [{"op": "step", "token": t} for t in ids[16:]]
    ref, gpu = _both(env, path, plan, "sdot")
    worst = _compare(ref, gpu, what="sdot")
    print(f"engine sdot: max rel err {worst:.3e}")


def test_batch_matches_reference_per_sequence(env):
    """The batch extension: three sequences sharing a 5-token prefix, each equal
    to the reference engine run on that sequence alone."""
    from engine_models import tiny_config
    d, ref_lib, lib = env
    path = _archive(env, "tiny_w0", tiny_config(0), 117)
    prefix = _tokens(5, 61, 30)
    prompts = [_tokens(9, 61, 31 + s) for s in range(3)]
    teacher = [_tokens(4, 61, 41 + s) for s in range(3)]
    op = {"op": "batch", "sessions": 3, "prefix": prefix, "prompts": prompts, "teacher": teacher, "kv": "int8",
          "steps": 6}
    gpu = run_plan(path, [op, dict(op, graphs=False)], lib, d, "batch_gpu")
    for s in range(3):
        plan = [{"op": "engine", "kv": "int8"}, {"op": "reset", "prefix": 5},
                {"op": "prefill", "tokens": prefix + prompts[s], "last_only": True}]
        plan += [{"op": "step", "token": t} for t in teacher[s]]
        plan += [{"op": "decode", "first": int(gpu["0_first"][s]), "max_new": 7}]
        ref = run_plan(path, plan, ref_lib, d, f"batch_ref{s}")
        assert rel(gpu["0_prefill_logits"][s], ref["2_logits"]) <= TOL
        assert int(gpu["0_first"][s]) == int(np.argmax(ref["2_logits"]))
        for j in range(4):
            assert rel(gpu["0_teacher_logits"][s, j], ref[f"{3 + j}_logits"]) <= TOL
        np.testing.assert_array_equal(gpu["0_tokens"][s], ref["7_tokens"][1:])   # greedy decode, graph replay
    np.testing.assert_array_equal(gpu["0_positions"], [5 + 9 + 4 + 6] * 3)
    # the captured-graph steps and the launch-by-launch steps agree bit for bit
    np.testing.assert_array_equal(gpu["0_tokens"], gpu["1_tokens"])
    np.testing.assert_array_equal(gpu["0_teacher_logits"], gpu["1_teacher_logits"])


@pytest.mark.parametrize("kv", ["fp32", "int8"])
def test_config5_geometry_matches_reference(env, kv):
    """BASELINE config 5's decoder (d 512, 12 layers, 8/4 heads x 64, vocab
    32768, CQ4 embedding, CQ2 projections and tables): a 48-token prompt and 6
    teacher-forced steps.  With the FP32 cache the logits stay within the
    1e-4 bar.  With the INT8 cache, a K or V element whose scaled value lies
    within FP32 rounding of a half-integer can round to the neighbouring int8
    code here and not there (the quantiser is discontinuous); such isolated
    one-code differences move the logits by up to a few 1e-4 of their
    maximum, so that case is held to 1e-3, and greedy tokens must agree
    wherever the reference's top-2 margin exceeds that bar."""
    from engine_models import config5
    d, ref_lib, lib = env
    path = _archive(env, "config5", config5(), 0)
    ids = _tokens(54, 32768, 77)
    plan = [{"op": "engine", "kv": kv}, {"op": "prefill", "tokens": ids[:48], "last_only": True}]
    plan += [{"op": "step", "token": t} for t in ids[48:]]
    ref, gpu = _both(env, path, plan, f"config5_{kv}")
    bar = TOL if kv == "fp32" else 1e-3
    worst = 0.0
    for key in [k for k in ref if k.endswith("_logits")]:
        e = rel(gpu[key], ref[key])
        worst = max(worst, e)
        margin = top2_margin(ref[key]) / np.max(np.abs(ref[key]))
        if int(np.argmax(gpu[key])) != int(np.argmax(ref[key])):
            assert margin <= bar, f"{key}: greedy differs with top-2 margin {margin:.3e}"
        assert e <= bar, f"{key}: rel err {e:.3e}"
    print(f"config-5 decoder kv={kv}: max rel err {worst:.3e}")


def test_decode_compiled_matches_reference(env):
    """needle2_engine_decode_compiled (frontend.cpp:1057-1079) through the
    reference's needle2/frontend.py decode_native: unconstrained greedy decoding
    from the prompt's own logits, and grammar-constrained decoding of a tool
    call (logits whose maximum is <tool_call>, then the compiled tool schema's
    token automaton: candidate projections, single-candidate steps and the
    terminal state).  The tokenizer and grammar compiler are the reference's,
    reached through this library's forwarding entry points."""
    from engine_models import tiny_config
    path = _archive(env, "tiny_v269", tiny_config(0, vocab=269), 31)
    tools = [{"name": "fn", "parameters": {"type": "object",
                                           "properties": {"a": {"type": "integer"}, "b": {"type": "boolean"}},
                                           "required": ["a", "b"]}}]
    prompt = _tokens(9, 269, 77)
    plan = [{"op": "engine", "kv": "fp32"},
            {"op": "decode_compiled", "prompt": prompt, "max_new": 12, "tools": None},
            {"op": "decode_compiled", "prompt": prompt, "max_new": 40, "tools": tools, "first": 10},
            {"op": "decode_compiled", "prompt": prompt[:4], "max_new": 40, "tools": tools, "first": 10}]
    ref, gpu = _both(env, path, plan, "compiled")
    _compare(ref, gpu, what="decode_compiled")
    assert ref["2_tokens"][0] == 10 and len(ref["2_tokens"]) > 1


@pytest.mark.parametrize("kv", ["fp32", "int8"])
def test_config5_batch_decode_kernels_match_reference(env, kv):
    """Config 5's decoder batched over 512 sessions, the row count at which a
    decode step runs the layer-boundary kernel and the tensor-core projections
    fed by its rotated bf16 operands; with the FP32 cache the projections'
    fused norm / RoPE / KV-store epilogue, with the INT8 cache the
    warp-per-query attention that norms, ropes and stores the new token itself
    (max_seq_len 256 keeps the caches small).  Sessions spread over the batch
    and its 128-row tiles, each against the reference engine run on that
    session alone: prefill and teacher-forced logits within 1e-4 (1e-3 with the
    INT8 cache: see test_config5_geometry_matches_reference), greedy tokens
    equal where the top-2 margin exceeds that bar."""
    from engine_models import config5
    d, ref_lib, lib = env
    path = _archive(env, "config5_s256", config5(256), 0)
    S, keep = 512, [0, 1, 130, 511]
    rng = np.random.default_rng(5)
    prompts = rng.integers(3, 32768, (S, 16)).tolist()
    teacher = rng.integers(3, 32768, (S, 3)).tolist()
    op = {"op": "batch", "sessions": S, "prompts": prompts, "teacher": teacher, "kv": kv, "steps": 3,
          "keep": keep}
    gpu = run_plan(path, [op], lib, d, f"c5batch_gpu_{kv}")
    bar = TOL if kv == "fp32" else 1e-3
    for i, s in enumerate(keep):
        plan = [{"op": "engine", "kv": kv}, {"op": "prefill", "tokens": prompts[s], "last_only": True}]
        plan += [{"op": "step", "token": t} for t in teacher[s]]
        plan += [{"op": "decode", "first": int(gpu["0_first"][s]), "max_new": 4}]
        ref = run_plan(path, plan, ref_lib, d, f"c5batch_ref_{kv}_{s}")
        pairs = [(gpu["0_prefill_logits"][i], ref["1_logits"])]
        pairs += [(gpu["0_teacher_logits"][i, j], ref[f"{2 + j}_logits"]) for j in range(3)]
        for n, (a, b) in enumerate(pairs):
            assert rel(a, b) <= bar, f"session {s}, logits {n}: rel err {rel(a, b):.3e}"
        if int(gpu["0_first"][s]) != int(np.argmax(ref["1_logits"])):
            assert top2_margin(ref["1_logits"]) / np.max(np.abs(ref["1_logits"])) <= bar
        else:
            np.testing.assert_array_equal(gpu["0_tokens"][s], ref["5_tokens"][1:])


@pytest.mark.parametrize("kv,S,prompt_len", [("fp32", 96, 260), ("int8", 64, 260), ("int8", 96, 260),
                                             ("int8", 96, 16)])
def test_config5_small_batch_matches_reference(env, kv, S, prompt_len):
    """Config 5's decoder batched over 64-96 sessions: the per-GPU share of an
    8-GPU run.  Decode steps here take the one-CTA-per-SM layer boundary and
    the K-split projections (their parts added by the RoPE / KV-store kernel
    and by the layer boundary).  Attention writes the out projection's rotated
    operands: at 64 sessions and 260-token prompts it splits the context and
    rotates while combining the splits; at 96 sessions it runs unsplit and
    rotates inside the attention kernel.  Two sessions against the reference
    engine run on each alone: logits within 1e-4 (1e-3 with the INT8 cache,
    whose quantiser is discontinuous: see test_config5_geometry_matches_reference),
    greedy tokens equal where the top-2 margin exceeds that bar."""
    from engine_models import config5
    d, ref_lib, lib = env
    path = _archive(env, "config5_s512", config5(512), 0)
    keep = [0, S - 1]
    rng = np.random.default_rng(11)
    prompts = rng.integers(3, 32768, (S, prompt_len)).tolist()
    teacher = rng.integers(3, 32768, (S, 2)).tolist()
    op = {"op": "batch", "sessions": S, "prompts": prompts, "teacher": teacher, "kv": kv, "steps": 3,
          "keep": keep}
    gpu = run_plan(path, [op], lib, d, f"c5small_gpu_{kv}_{S}_{prompt_len}")
    for i, s in enumerate(keep):
        plan = [{"op": "engine", "kv": kv}, {"op": "prefill", "tokens": prompts[s], "last_only": True}]
        plan += [{"op": "step", "token": t} for t in teacher[s]]
        plan += [{"op": "decode", "first": int(gpu["0_first"][s]), "max_new": 4}]
        ref = run_plan(path, plan, ref_lib, d, f"c5small_ref_{kv}_{S}_{prompt_len}_{s}")
        pairs = [(gpu["0_prefill_logits"][i], ref["1_logits"])]
        pairs += [(gpu["0_teacher_logits"][i, j], ref[f"{2 + j}_logits"]) for j in range(2)]
        bar = TOL if kv == "fp32" else 1e-3
        for n, (a, b) in enumerate(pairs):
            assert rel(a, b) <= bar, f"session {s}, logits {n}: rel err {rel(a, b):.3e}"
        if int(gpu["0_first"][s]) == int(np.argmax(ref["1_logits"])):
            np.testing.assert_array_equal(gpu["0_tokens"][s], ref["4_tokens"][1:])
        else:
            assert top2_margin(ref["1_logits"]) / np.max(np.abs(ref["1_logits"])) <= bar
