"""CPU restatement of the reference's Llama-3 tokenizer.

TEST INFRASTRUCTURE ONLY: used by tests/ and tests/golden/make_tokenizer_golden.py
to check the product tokenizer (ijb_tokenizer_*, inferencer-jetson_b200/csrc/tokenizer.cpp);
never by the product.  It restates Tokenizer (inferencer.cu:361-451) step by
step, slowly and literally:
  * byte symbols (:374-378): bytes 33-126, 161-172 and 174-255 stand for
    themselves, every other byte for the next code point from 256 up;
  * pre-tokenizer (:379-383, :415-431): the same pattern (Python's `regex`
    module standing in for PCRE2 with UTF + UCP); text between matches and, on
    a failed match, the rest of the text are pieces too;
  * BPE (:391-413): merge the adjacent pair whose "left right" string has the
    lowest merge rank, leftmost among equals, until none has a rank;
  * decode (:432-445) and special (:446-450).
Parity: pinned against the reference's own Tokenizer run on the same vocabulary
(tests/golden/tokenizer_golden.npz, made by tests/golden/make_tokenizer_golden.py
through oracle/_ref/libref_harness.so).
"""
from __future__ import annotations

import regex

LLAMA3_VOCAB = 128256

PATTERN = (r"(?:'[sS]|'[tT]|'[rR][eE]|'[vV][eE]|'[mM]|'[lL][lL]|'[dD])|"
           r"[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}|"
           r" ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+")
_RE = regex.compile(PATTERN)


def byte_symbols() -> list[str]:
    """The 256 byte symbols in byte order (inferencer.cu:374-378)."""
    out, cp = [], 256
    for b in range(256):
        plain = 33 <= b <= 126 or 161 <= b <= 172 or b >= 174
        out.append(chr(b) if plain else chr(cp))
        if not plain:
            cp += 1
    return out


BYTE_SYMBOL = byte_symbols()
SYMBOL_BYTE = {s: b for b, s in enumerate(BYTE_SYMBOL)}


def pieces(text: bytes) -> list[bytes]:
    """The pre-tokenizer's pieces of `text` (inferencer.cu:415-431).  Text that
    is not valid UTF-8 makes the first match call fail, so it is one piece."""
    try:
        s = text.decode("utf-8")
    except UnicodeDecodeError:
        return [text] if text else []
    out, pos = [], 0
    while pos < len(s):
        m = _RE.search(s, pos)
        if m is None:
            out.append(s[pos:])
            break
        if m.start() > pos:
            out.append(s[pos:m.start()])
        if m.end() == m.start():
            raise RuntimeError("Tokenizer regex made no progress")
        out.append(m.group())
        pos = m.end()
    return [p.encode("utf-8") for p in out]


class Tokenizer:
    """The reference's Tokenizer over a token list and a merge list."""

    def __init__(self, tokens: list[str], merges: list[str]):
        if len(tokens) != LLAMA3_VOCAB:
            raise RuntimeError("Expected Llama 3 tokenizer")
        self.tokens = tokens
        self.ids: dict[str, int] = {}
        for i, t in enumerate(tokens):
            self.ids.setdefault(t, i)
        self.rank: dict[str, int] = {}
        for i, m in enumerate(merges):
            self.rank.setdefault(m, i)

    def bpe_piece(self, piece: bytes) -> list[int]:
        parts = [BYTE_SYMBOL[b] for b in piece]
        while len(parts) > 1:
            best, at = None, 0
            for i in range(len(parts) - 1):
                r = self.rank.get(parts[i] + " " + parts[i + 1])
                if r is not None and (best is None or r < best):
                    best, at = r, i
            if best is None:
                break
            parts[at:at + 2] = [parts[at] + parts[at + 1]]
        out = []
        for p in parts:
            if p not in self.ids:
                raise RuntimeError("Tokenizer produced an unknown token")
            out.append(self.ids[p])
        return out

    def encode(self, text: bytes) -> list[int]:
        out = []
        for p in pieces(text):
            out += self.bpe_piece(p)
        return out

    def decode(self, i: int) -> bytes:
        if i < 0 or i >= len(self.tokens):
            raise RuntimeError("Invalid token id")
        s = self.tokens[i].encode("utf-8")
        out, k = bytearray(), 0
        while k < len(s):
            first = s[k]
            n = 1 if first < 0x80 else 2 if first < 0xE0 else 3 if first < 0xF0 else 4
            if k + n > len(s):
                raise RuntimeError("Malformed token UTF-8")
            try:
                sym = s[k:k + n].decode("utf-8")
            except UnicodeDecodeError:
                sym = None
            if sym not in SYMBOL_BYTE:
                raise RuntimeError("Cannot decode token")
            out.append(SYMBOL_BYTE[sym])
            k += n
        return bytes(out)

    def special(self, name: str) -> int:
        if name not in self.ids:
            raise RuntimeError("Missing special token " + name)
        return self.ids[name]
