"""Synthetic Needle-2 archives for the engine parity tests and the decoder
benchmark (test infrastructure).

Models are the reference's own NeedleModel with its default random init
(needle2/model.py:266-287) under a fixed torch seed; matrices are packed by
the reference's quantizer into its TensorRecord objects (needle2/archive.py),
exactly as OpenNeedle's tests build in-memory archives
(tests/test_native.py:75-88 there).  Archives are saved to .npz so that a
reference process and a GPU process can load identical weights.
"""
from __future__ import annotations

import json
from types import SimpleNamespace

import numpy as np


def _ref():
    from oracle import oracle as O
    if O.reference_package() is None:
        raise RuntimeError(f"reference package not found under {O.REF_ROOT}")
    import needle2.archive as A
    import needle2.model as M
    import needle2.quantize as Q
    return A, M, Q


def tiny_config(window: int = 0, vocab: int = 61) -> dict:
    """A few-layer model exercising GQA, two lanes, two engram sites with
    nonidentity taps, a sliding window when window > 0."""
    return dict(vocab_size=vocab, d_model=32, num_heads=4, num_kv_heads=2, num_layers=3, head_dim=8, mhc_lanes=2,
                engram_layers=(0, 2), engram_orders=(2, 3), engram_slots=19, engram_sub_dim=8, num_engram_tables=4,
                engram_conv_taps=4, engram_conv_dilation=3, max_seq_len=96, kv_window=window)


def tokenizer_blob() -> bytes:
    """A small tokenizer in the .cact tokenizer record format (needle2/
    tokenizer.py:13-27: header <IIIIIBBH = pieces, pad, eos, bos, unk,
    add_dummy_prefix, byte_fallback, reserved; then per piece <fBH = score,
    type, byte length, UTF-8 bytes): control tokens, the grammar's special
    markers at the ids the grammar compiler looks for (<stop> 5,
    <tool_call> 10, </tool_call> 11), a few text pieces and all 256 byte
    pieces, 269 in all."""
    import struct
    normal, unknown, control, user, byte = 0, 1, 2, 3, 4
    pieces = [("<pad>", control), ("</s>", control), ("<s>", control), ("<unk>", unknown), ("\u2581", normal),
              ("<stop>", user), ("a", normal), ("b", normal), ("ab", normal), ("ba", normal),
              ("<tool_call>", user), ("</tool_call>", user), ("</tools>", user)]
    pieces += [(f"<0x{v:02X}>", byte) for v in range(256)]
    out = bytearray(struct.pack("<IIIIIBBH", len(pieces), 0, 1, 2, 3, 1, 1, 0))
    for text, kind in pieces:
        raw = text.encode("utf-8")
        out += struct.pack("<fBH", -float(len(raw)), kind, len(raw)) + raw
    return bytes(out)


def config5(max_seq_len: int = 4096) -> dict:
    """d 512, 12 layers, 8 heads x 64 (4 KV heads), vocab
    32768, max_seq 4096 (smaller values shrink only the KV capacity), no
    window, engram sites at layers 2 and 9."""
    return dict(vocab_size=32768, d_model=512, num_heads=8, num_kv_heads=4, num_layers=12, head_dim=64,
                max_seq_len=max_seq_len, kv_window=0, engram_layers=(2, 9))


def build_archive(cfg: dict, seed: int = 0, *, taps_noise: float = 0.1, embedding_bits: int = 4,
                  mhc_bits: int = 4, default_bits: int = 2, group: int = 128):
    """(metadata, records): NeedleModel(cfg) under torch.manual_seed(seed),
    CQ for the embedding (embedding_bits), the mHC projections (mhc_bits; the
    engine uses them dequantised) and every other projection / engram table
    (default_bits), FP32 elsewhere -- the release scheme of the reference's
    docs (embedding=4, mhc=4, default=2)."""
    import torch
    A, M, Q = _ref()
    torch.manual_seed(seed)
    model = M.NeedleModel(M.NeedleConfig(**cfg))
    with torch.no_grad():
        for site in range(len(model.config.engram_layers)):
            if taps_noise:
                getattr(model, f"engram{site}").taps[1:].normal_(0, taps_noise)
    records = {}
    for name, tensor in model.canonical_state_dict().items():
        a = tensor.detach().numpy().astype(np.float32)
        is_matrix = a.ndim == 2 and (name == "embedding" or name.startswith("mhc_phi") or
                                     name.endswith("_proj") or name.endswith(".tables"))
        if is_matrix:
            bits = embedding_bits if name == "embedding" else mhc_bits if name.startswith("mhc_phi") else default_bits
            packed, norms = Q.quantize_matrix(a, bits, group)
            records[name] = A.TensorRecord(name, A.CQ, a.shape, packed.tobytes() + norms.tobytes(), group, bits,
                                           Q.codebook(bits, group))
        else:
            records[name] = A.TensorRecord(name, A.FP32, a.shape, a.tobytes())
    meta = model.config.to_dict()
    meta["hada_n"] = 1 << (meta["d_model"] - 1).bit_length()
    meta["engram_orders"] = list(meta["engram_orders"])
    meta["engram_layers"] = list(meta["engram_layers"])
    return meta, records


def save_archive(path, meta: dict, records: dict) -> None:
    arrays = {"__meta__": np.frombuffer(json.dumps(meta).encode(), np.uint8)}
    for name, r in records.items():
        arrays[f"{name}|blob"] = np.frombuffer(r.blob, np.uint8)
        info = {"dtype": r.dtype, "shape": list(r.shape), "group": r.group_size, "bits": r.bits}
        arrays[f"{name}|info"] = np.frombuffer(json.dumps(info).encode(), np.uint8)
        if r.codebook is not None:
            arrays[f"{name}|cb"] = np.asarray(r.codebook, np.float32)
    np.savez(path, **arrays)


def load_archive(path):
    """SimpleNamespace(metadata, tensors) of reference TensorRecords, the
    in-memory archive form the reference's NativeEngine accepts."""
    A, _, _ = _ref()
    z = np.load(path)
    meta = json.loads(bytes(z["__meta__"]).decode())
    records = {}
    for key in z.files:
        if not key.endswith("|info"):
            continue
        name = key[:-5]
        info = json.loads(bytes(z[key]).decode())
        cb = z[f"{name}|cb"] if f"{name}|cb" in z.files else None
        records[name] = A.TensorRecord(name, info["dtype"], tuple(info["shape"]), z[f"{name}|blob"].tobytes(),
                                       info["group"], info["bits"], cb)
    return SimpleNamespace(metadata=meta, tensors=records)
