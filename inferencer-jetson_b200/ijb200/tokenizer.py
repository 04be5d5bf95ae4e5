"""Python mirror of the reference's Tokenizer (inferencer.cu:361-451) over
the C ABI's ijb_tokenizer_* entry points (host code; no GPU involved).

    tok = Tokenizer(model_tokens, model_merges)   # tokenizer.ggml.tokens / .merges
    ids = tok.encode("Hello world")               # Tokenizer::encode
    tok.decode(ids[0])                            # Tokenizer::decode -> bytes
    tok.special("<|eot_id|>")                     # Tokenizer::special

Failures raise TokenizerError with the reference's messages ("Expected Llama 3
tokenizer", "Invalid token id", "Missing special token ...", ...).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import lib as _L


class TokenizerError(RuntimeError):
    pass


class Tokenizer:
    def __init__(self, tokens, merges):
        self.lib = _L.load()
        toks = [t.encode() if isinstance(t, str) else bytes(t) for t in tokens]
        mrgs = [m.encode() if isinstance(m, str) else bytes(m) for m in merges]
        ta = (ctypes.c_char_p * max(1, len(toks)))(*toks)
        ma = (ctypes.c_char_p * max(1, len(mrgs)))(*mrgs)
        h = ctypes.c_void_p()
        rc = self.lib.ijb_tokenizer_create(ta, len(toks), ma, len(mrgs), ctypes.byref(h))
        if rc != _L.OK:
            raise TokenizerError(self.lib.ijb_tokenizer_last_error(None).decode())
        self.h = h

    def _check(self, rc: int) -> None:
        if rc != _L.OK:
            raise TokenizerError(self.lib.ijb_tokenizer_last_error(self.h).decode())

    def _ids(self, fn, text) -> list[int]:
        data = text.encode() if isinstance(text, str) else bytes(text)
        cap = len(data) + 32
        n = ctypes.c_long()
        while True:
            buf = np.empty(cap, np.int32)
            self._check(fn(self.h, data, len(data), buf.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), cap,
                           ctypes.byref(n)))
            if n.value <= cap:
                return buf[:n.value].tolist()
            cap = n.value

    def encode(self, text) -> list[int]:
        return self._ids(self.lib.ijb_tokenizer_encode, text)

    def encode_batch(self, texts, threads: int = 0) -> list[list[int]]:
        """Many texts at once on `threads` host threads (0: all)."""
        data = [t.encode() if isinstance(t, str) else bytes(t) for t in texts]
        n = len(data)
        ptrs = (ctypes.c_char_p * max(1, n))(*data)
        lens = (ctypes.c_long * max(1, n))(*[len(d) for d in data])
        offs = (ctypes.c_long * (n + 1))()
        cap = sum(lens[:n]) + 16
        while True:
            buf = np.empty(max(1, cap), np.int32)
            rc = self.lib.ijb_tokenizer_encode_batch(self.h, ptrs, lens, n,
                                                     buf.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), cap, offs,
                                                     int(threads))
            if rc == _L.ERR_CAPACITY:
                cap = offs[n]
                continue
            self._check(rc)
            return [buf[offs[i]:offs[i + 1]].tolist() for i in range(n)]

    def chat_prompt(self, prompt) -> list[int]:
        """The reference's chat_prompt (inferencer.cu:1534-1551)."""
        return self._ids(self.lib.ijb_tokenizer_chat_prompt, prompt)

    def decode(self, token_id: int) -> bytes:
        buf = ctypes.create_string_buffer(256)
        n = ctypes.c_int()
        self._check(self.lib.ijb_tokenizer_decode(self.h, int(token_id), buf, 256, ctypes.byref(n)))
        if n.value > 256:
            buf = ctypes.create_string_buffer(n.value)
            self._check(self.lib.ijb_tokenizer_decode(self.h, int(token_id), buf, n.value, ctypes.byref(n)))
        return buf.raw[:n.value]

    def special(self, name: str) -> int:
        v = ctypes.c_int()
        self._check(self.lib.ijb_tokenizer_special(self.h, name.encode(), ctypes.byref(v)))
        return v.value

    def close(self) -> None:
        if self.h:
            self.lib.ijb_tokenizer_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
