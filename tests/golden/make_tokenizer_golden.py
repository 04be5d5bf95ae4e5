"""Captures tests/golden/tokenizer_golden.npz: the reference's own Tokenizer
(inferencer.cu:361-451, built unmodified into oracle/_ref/libref_harness.so
by oracle/Makefile.ref) run on the host over a synthetic Llama-3-sized
vocabulary, on seeded texts and edge cases.

Run from the repository root after `make -C oracle -f Makefile.ref REF_DIR=...`:
    python tests/golden/make_tokenizer_golden.py
The vocabulary is trained here (ijb200.synth_vocab: byte-level BPE over seeded
text, 128256 tokens with fillers and the Llama 3 special tokens) and stored in
the fixture as its merge pairs; the tests rebuild the same token and merge
lists from them with synth_vocab.synthetic_vocab.  The oracle restatement
(oracle/bpe.py) is compared on the way.
"""
import ctypes
import json
import os
import random
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "inferencer-jetson_b200"))
import bpe  # noqa: E402
from gguf_writer import write_vocab_gguf  # noqa: E402
from ijb200 import synth_vocab as sv  # noqa: E402


def golden_texts():
    rng = random.Random(11)
    texts = [sv.random_text(rng, rng.choice([5, 20, 60, 200])).encode() for _ in range(48)]
    texts += [
        b"", b"a", b" ", b"\n", b"\r\n", b"  \n\n  ", b"\t\t", "é".encode(), "😀".encode(), b"'s",
        b"don't WON'T I'm we'll you'd they've she's", b"12345678901234", b"3.14159 -2,000,000 1e10",
        b"hello world", b"  hello   world  ", b"line one\nline two\r\nline three\n\n\n",
        b"=" * 60, b"-" * 33 + b">", b" " * 100, b"a" * 100, b"ab" * 40,
        b"Supercalifragilisticexpialidociousinternationalization",
        "Ünïcödé wörds, Москва и 東京 😀🚀👍🏽 — «quotes» “curly” ½ ²".encode(),
        "naïve café nbsp　ideographic sep".encode(),
        b"<|begin_of_text|>user<|end_header_id|>", b"x = y + z * (a - b) / c; // comment",
        # not valid UTF-8: a stray continuation byte, 0xff, a truncated sequence,
        # an overlong form, a surrogate
        b"abc \x80 def", b"\xff\xfe text", b"trunc \xe2\x82", b"over \xc0\xaf long", b"sur \xed\xa0\x80 rogate",
        b"valid start " * 5 + b"\x80",
    ]
    return texts


def main():
    lib = ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref_harness.so"))
    lib.ref_last_error.restype = ctypes.c_char_p
    pairs = sv.train_merges(sv.training_corpus(), 700)
    tokens, merges = sv.synthetic_vocab(pairs)
    texts = golden_texts()
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "vocab.gguf").encode()
        write_vocab_gguf(path.decode(), tokens, merges)

        def enc(t: bytes):
            cap = 4 * len(t) + 16
            buf = (ctypes.c_int * cap)()
            n = ctypes.c_long()
            rc = lib.ref_tokenize(path, t, ctypes.c_long(len(t)), buf, ctypes.c_long(cap), ctypes.byref(n))
            if rc:
                raise RuntimeError(lib.ref_last_error().decode())
            return list(buf[:n.value])

        def dec(i: int):
            buf = ctypes.create_string_buffer(256)
            n = ctypes.c_int()
            rc = lib.ref_detokenize(path, i, buf, 256, ctypes.byref(n))
            return (buf.raw[:n.value], "") if rc == 0 else (b"", lib.ref_last_error().decode())

        ids = [enc(t) for t in texts]
        oracle = bpe.Tokenizer(tokens, merges)
        bad = [i for i, t in enumerate(texts) if oracle.encode(t) != ids[i]]
        print(f"{len(texts)} texts, {sum(map(len, ids))} ids; oracle disagrees on {bad}")
        dec_ids = list(range(0, 300)) + list(range(256, 256 + len(pairs), 7)) + list(range(127990, 128020)) + \
            [128255, -1, 128256]
        decoded = [dec(i) for i in dec_ids]
        chat_prompts = [b"", b"Hello", b"What is 2+2?\nAnswer briefly.", "Résumé: 東京 😀".encode(),
                        sv.random_text(random.Random(3), 150).encode()]

        def chat(t: bytes):
            cap = 4 * len(t) + 64
            buf = (ctypes.c_int * cap)()
            n = ctypes.c_long()
            if lib.ref_chat_prompt(path, t, ctypes.c_long(len(t)), buf, ctypes.c_long(cap), ctypes.byref(n)):
                raise RuntimeError(lib.ref_last_error().decode())
            return list(buf[:n.value])

        chats = [chat(t) for t in chat_prompts]
        specials = {}
        for name in sv.SPECIALS + ["<|nope|>"]:
            v = ctypes.c_int(-1)
            rc = lib.ref_special_token(path, name.encode(), ctypes.byref(v))
            specials[name] = v.value if rc == 0 else lib.ref_last_error().decode()
    out = os.path.join(ROOT, "tests", "golden", "tokenizer_golden.npz")
    np.savez_compressed(
        out,
        pairs=np.array(json.dumps(pairs)),
        text_bytes=np.frombuffer(b"".join(texts), np.uint8),
        text_off=np.cumsum([0] + [len(t) for t in texts]).astype(np.int64),
        ids=np.array([i for x in ids for i in x], np.int32),
        ids_off=np.cumsum([0] + [len(x) for x in ids]).astype(np.int64),
        dec_ids=np.array(dec_ids, np.int32),
        dec_bytes=np.array(json.dumps([[b.hex(), e] for b, e in decoded])),
        specials=np.array(json.dumps(specials)),
        chat=np.array(json.dumps([[t.hex(), c] for t, c in zip(chat_prompts, chats)])),
    )
    print("wrote", out, os.path.getsize(out), "bytes")


if __name__ == "__main__":
    main()
