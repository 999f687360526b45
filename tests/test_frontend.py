"""The frontend entry points of libneedle2_b200.so (needle2/csrc/frontend.h:15-35)
driven by the reference's own needle2/frontend.py, in child processes (the
reference's loader caches its library choice): the tokenizer and grammar
compiler forward to the reference's native library named by
NEEDLE2_FRONTEND_LIBRARY, so tokens and token automata equal the reference's
Python tokenizer and grammar compiler; without that variable they fail with a
message that names it.  No GPU is used."""
import os
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent

CHILD = textwrap.dedent(r'''
    import json, sys
    from needle2.frontend import CompiledGrammar, NativeTokenizer
    from needle2.grammar import compile_tool_dfa
    from needle2.tokenizer import RefTokenizer, parse_tokenizer_blob
    from engine_models import tokenizer_blob

    blob = tokenizer_blob()
    try:
        native = NativeTokenizer(blob)
    except Exception as e:
        print("ERROR", e)
        sys.exit(0)
    ref = RefTokenizer(parse_tokenizer_blob(blob))
    for text in ["", "abab", " ba ab", "中文!", "a</tools>b", "{\"a\": 1}"]:
        assert native.encode(text) == ref.encode(text), text
        assert native.decode(native.encode(text)) == ref.decode(ref.encode(text)), text
    tools = [{"name": "fn", "parameters": {"type": "object",
                                          "properties": {"a": {"type": "integer"}, "s": {"type": "string"},
                                                         "e": {"enum": ["ab", None, True]}},
                                          "required": ["a"]}}]
    grammar = CompiledGrammar(native, json.dumps(tools, separators=(",", ":")))
    desc = grammar._lib.needle2_grammar_dfa(grammar._handle).contents
    py = compile_tool_dfa(tools, ref)
    # walk both automata from their start states in lockstep
    todo, seen = [(0, 0)], set()
    while todo:
        x, y = todo.pop()
        if (x, y) in seen:
            continue
        seen.add((x, y))
        assert desc.state_types[x] == py.state_types[y]
        a = {desc.candidate_tokens[i]: desc.next_states[i]
             for i in range(desc.candidate_offsets[x], desc.candidate_offsets[x + 1])}
        lo, hi = py.candidate_offsets[y:y + 2]
        b = dict(zip(py.candidate_tokens[lo:hi], py.next_states[lo:hi]))
        assert a.keys() == b.keys()
        todo.extend((a[t], b[t]) for t in a)
    print("OK", len(seen))
''')


def _run(env_extra):
    from oracle import oracle as O
    env = {k: v for k, v in os.environ.items() if k != "NEEDLE2_FRONTEND_LIBRARY"}
    env.update(env_extra, PYTHONPATH=os.pathsep.join([str(O.REF_ROOT), str(ROOT), str(HERE)]))
    proc = subprocess.run([sys.executable, "-c", CHILD], env=env, capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stderr[-3000:]
    return proc.stdout


@pytest.fixture(scope="module")
def libs():
    from oracle import oracle as O
    if O.reference_package() is None or not O.ref_available():
        pytest.skip("reference package or oracle/_ref unavailable")
    from openneedle_b200 import build
    return str(build.build()), str(O.REF_LIB)


def test_frontend_forwards_to_reference_library(libs):
    lib, ref = libs
    out = _run({"NEEDLE2_NATIVE_LIBRARY": lib, "NEEDLE2_FRONTEND_LIBRARY": ref})
    assert out.startswith("OK"), out


def test_frontend_without_library_fails_loudly(libs):
    lib, _ = libs
    out = _run({"NEEDLE2_NATIVE_LIBRARY": lib})
    assert out.startswith("ERROR") and "NEEDLE2_FRONTEND_LIBRARY" in out, out
