"""Runs an engine plan through the reference's unchanged Python layer
(needle2/native.py NativeEngine) on whichever library NEEDLE2_NATIVE_LIBRARY
names -- the reference's CPU build (oracle/_ref) or libneedle2_b200.so -- and
saves every output (test infrastructure; one process per library, because the
reference's loader caches its choice).

    python tests/engine_child.py ARCHIVE.npz PLAN.json OUT.npz

A plan is a list of operations:
  {"op": "engine", "kv": "int8"|"fp32", "abits": 0|8, "matmul": "fp32"|"sdot"}
  {"op": "reset", "prefix": P}
  {"op": "prefill", "tokens": [...], "last_only": bool, "backend": "native"|"torch"}
  {"op": "step", "token": t, "hidden": bool}
  {"op": "step_candidates", "token": t, "candidates": [...]}
  {"op": "cache_prefix"} / {"op": "reset_to_prefix"}
  {"op": "decode", "first": t, "max_new": n}
  {"op": "decode_compiled", "prompt": [...], "max_new": n, "tools": [...] | null, "first": t | null}
    (needle2/frontend.py decode_native through NativeEngine.decode_from_logits: the
    prompt's prefill logits, or logits whose maximum is `first`; the grammar is
    compiled from `tools` with the tokenizer of engine_models.tokenizer_blob)
  {"op": "kv_bytes"}
  {"op": "batch", "sessions": S, "prefix": [...], "prompts": [[...]...], "steps": n, "kv": ..., "matmul": ...}
    (GPU library only: this repository's batch extension through openneedle_b200.engine;
    "keep": [...] saves only those sessions' logits)
Outputs are saved as "<index>_<name>".
"""
from __future__ import annotations

import ctypes as ct
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE))


def main(archive_path: str, plan_path: str, out_path: str) -> int:
    from engine_models import load_archive
    from needle2.native import NativeEngine, build_native

    archive = load_archive(archive_path)
    plan = json.loads(Path(plan_path).read_text())
    lib_path = str(build_native())
    on_reference = "libneedle2_ref" in Path(lib_path).name
    out = {"library": np.frombuffer(lib_path.encode(), np.uint8)}
    engine = None
    for i, op in enumerate(plan):
        kind = op["op"]
        if kind == "engine":
            matmul = op.get("matmul", "fp32")
            engine = NativeEngine(archive, activation_bits=op.get("abits", 0), kv_cache=op.get("kv", "fp32"),
                                  matmul="fp32" if (matmul == "sdot" and on_reference) else matmul)
            if matmul == "sdot" and on_reference:
                # the reference refuses SDOT off ARM64; its portable branches compute the same integers
                lib = ct.CDLL(lib_path)
                lib.ref_engine_force_sdot.argtypes = [ct.c_void_p]
                assert lib.ref_engine_force_sdot(engine._handle) == 0
        elif kind == "reset":
            engine.reset(prefix_len=op.get("prefix", 0))
        elif kind == "prefill":
            out[f"{i}_logits"] = engine.prefill(np.asarray(op["tokens"]), last_only=op.get("last_only", False),
                                                backend=op.get("backend", "native"))
        elif kind == "step":
            r = engine.step(int(op["token"]), return_hidden=op.get("hidden", False))
            if op.get("hidden", False):
                out[f"{i}_logits"], out[f"{i}_hidden"] = r
            else:
                out[f"{i}_logits"] = r
        elif kind == "step_candidates":
            out[f"{i}_logits"] = engine.step_candidates(int(op["token"]), op["candidates"])
        elif kind == "cache_prefix":
            engine.cache_prefix()
        elif kind == "reset_to_prefix":
            engine.reset_to_prefix()
        elif kind == "decode":
            out[f"{i}_tokens"] = np.asarray(engine.decode(int(op["first"]), int(op["max_new"])), np.int32)
        elif kind == "decode_compiled":
            from needle2.frontend import CompiledGrammar, NativeTokenizer
            from engine_models import tokenizer_blob
            grammar = None
            if op.get("tools") is not None:
                tok = NativeTokenizer(tokenizer_blob())
                grammar = CompiledGrammar(tok, json.dumps(op["tools"], separators=(",", ":")))
            engine.reset()
            logits = engine.prefill(np.asarray(op["prompt"]), last_only=True)
            if op.get("first") is not None:
                logits = np.full_like(logits, -1.0)
                logits[int(op["first"])] = 1.0
            out[f"{i}_tokens"] = np.asarray(engine.decode_from_logits(logits, int(op["max_new"]), grammar), np.int32)
        elif kind == "kv_bytes":
            out[f"{i}_kv_bytes"] = np.array([engine.kv_storage_bytes], np.int64)
        elif kind == "batch":
            if on_reference:
                raise SystemExit("the batch extension exists only in libneedle2_b200.so")
            from openneedle_b200.engine import GpuModel
            model = GpuModel(archive, matmul=op.get("matmul", "fp32"), kv_cache=op.get("kv", "int8"),
                             activation_bits=op.get("abits", 0))
            prefix = op.get("prefix", [])
            b = model.batch(op["sessions"], len(prefix))
            b.set_graphs(op.get("graphs", True))
            if prefix:
                b.set_prefix(prefix)
            keep = op.get("keep")
            pick = (lambda a: a[keep]) if keep is not None else (lambda a: a)
            logits, nxt = b.prefill(np.asarray(op["prompts"], np.int32))
            out[f"{i}_prefill_logits"] = pick(logits)
            out[f"{i}_first"] = nxt
            if op.get("teacher"):
                steps = []
                for tok in np.asarray(op["teacher"], np.int32).T:
                    lg, _ = b.step(tok, greedy=False)
                    steps.append(pick(lg))
                out[f"{i}_teacher_logits"] = np.stack(steps, 1)
            if op.get("steps"):
                out[f"{i}_tokens"] = b.decode_greedy(nxt, op["steps"])
            out[f"{i}_positions"] = b.positions()
            b.close()
            model.close()
        else:
            raise SystemExit(f"unknown op {kind}")
    np.savez(out_path, **out)
    return 0


if __name__ == "__main__":
    sys.exit(main(*sys.argv[1:4]))
