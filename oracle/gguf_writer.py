"""Minimal GGUF v3 writer for seeded synthetic models (test infrastructure).

TEST INFRASTRUCTURE ONLY: it exists so that the reference's own runner
(GGUF + FastRunner, inferencer.cu:204-340, :1182-1531, built unmodified into
oracle/_ref/) can load the same random-init weights the B200 engine and the
CPU oracle use.  Used by tests/, tests/golden/make_ref_runner_golden.py and
bench.py's reference-CUDA baseline leg; never by the product.

Layout written (what GGUF's reader expects, inferencer.cu:216-292):
  "GGUF", u32 version 3, u64 tensor count, u64 key/value count;
  key/values: u64-length string key, u32 type, value (u32 = 4, f32 = 6,
  string = 8);
  tensor infos: name, u32 n_dims, u64 dims (dims[0] = row length), u32 GGML
  type (0 F32, 12 Q4_K, 14 Q6_K), u64 offset from the data start;
  zero padding to the 32-byte alignment, then each tensor's bytes at its
  offset (offsets 32-byte aligned).
"""
from __future__ import annotations

import struct

import numpy as np

ALIGN = 32


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, value) -> bytes:
    if isinstance(value, str):
        return _str(key) + struct.pack("<I", 8) + _str(value)
    if isinstance(value, float):
        return _str(key) + struct.pack("<If", 6, value)
    return _str(key) + struct.pack("<II", 4, int(value))


def llama_metadata(cfg) -> dict:
    """The keys FastRunner reads (inferencer.cu:1205-1214)."""
    return {
        "general.architecture": "llama",
        "llama.embedding_length": cfg.dim,
        "llama.block_count": cfg.layers,
        "llama.attention.head_count": cfg.heads,
        "llama.attention.head_count_kv": cfg.kv_heads,
        "llama.feed_forward_length": cfg.hidden,
        "llama.vocab_size": cfg.vocab,
        "llama.attention.layer_norm_rms_epsilon": float(cfg.eps),
        "llama.rope.freq_base": float(cfg.rope_base),
    }


def tensor_table(cfg, weights: dict):
    """(name, dims, ggml type, array) for every tensor of a synth model."""
    shapes = {n: (t, r, c) for n, t, r, c in cfg.matrices()}
    out = []
    for name, arr in weights.items():
        if name in shapes:
            t, rows, cols = shapes[name]
            out.append((name, (cols, rows), t, arr))
        elif name == "output.weight":
            per_block = arr.shape[1] // (cfg.dim // 256)
            out.append((name, (cfg.dim, cfg.vocab), {144: 12, 210: 14}[per_block], arr))
        else:
            out.append((name, (arr.size,), 0, np.ascontiguousarray(arr, np.float32)))
    return out


def write_gguf(path: str, cfg, weights: dict) -> int:
    """Writes `weights` (synth.make_model output) as a GGUF v3 file; returns
    the byte size of the tensor data."""
    table = tensor_table(cfg, weights)
    meta = llama_metadata(cfg)
    head = b"GGUF" + struct.pack("<IQQ", 3, len(table), len(meta))
    head += b"".join(_kv(k, v) for k, v in meta.items())
    offset = 0
    offsets = []
    for name, dims, t, arr in table:
        offsets.append(offset)
        head += _str(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
        head += struct.pack("<IQ", t, offset)
        offset += (arr.nbytes + ALIGN - 1) // ALIGN * ALIGN
    pad = (-len(head)) % ALIGN
    with open(path, "wb") as f:
        f.write(head + b"\0" * pad)
        for (name, dims, t, arr), off in zip(table, offsets):
            data = np.ascontiguousarray(arr).tobytes()
            f.write(data)
            f.write(b"\0" * ((-len(data)) % ALIGN))
    return offset


def _str_array(key: str, values) -> bytes:
    """A GGUF array of strings (type 9 of element type 8), as the reader's
    tokenizer keys expect (inferencer.cu:227-232)."""
    return _str(key) + struct.pack("<IIQ", 9, 8, len(values)) + b"".join(_str(v) for v in values)


def write_vocab_gguf(path: str, tokens, merges) -> None:
    """A GGUF v3 file holding only tokenizer.ggml.tokens and
    tokenizer.ggml.merges (no tensors), for the reference's Tokenizer; 32 bytes
    of padding follow the header, since the reader wants data after it."""
    head = b"GGUF" + struct.pack("<IQQ", 3, 0, 2)
    head += _str_array("tokenizer.ggml.tokens", tokens) + _str_array("tokenizer.ggml.merges", merges)
    with open(path, "wb") as f:
        f.write(head + b"\0" * ((-len(head)) % ALIGN) + b"\0" * ALIGN)

