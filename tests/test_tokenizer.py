"""The host tokenizer (ijb_tokenizer_*, the reference's Tokenizer,
inferencer.cu:361-451) against the reference itself and the oracle.

The fixture holds the reference's own outputs (its unmodified Tokenizer run on
the host, tests/golden/make_tokenizer_golden.py) over a synthetic 128256-token
vocabulary: 80 texts (seeded mixed text, edge cases, long runs that take the
heap merge, and text that is not valid UTF-8), decodes of 333 ids (error
messages included) and the special-token lookups.  The oracle
(oracle/bpe.py) is pinned to the same fixture, then checks the product on
more seeded text (ijb200.synth_vocab).  No GPU involved."""
import json
import random
import threading

import numpy as np
import pytest

import bpe
from ijb200 import synth_vocab as sv
from ijb200.tokenizer import Tokenizer, TokenizerError


@pytest.fixture(scope="module")
def gold():
    g = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden",
                                           "tokenizer_golden.npz"))
    pairs = [tuple(p) for p in json.loads(str(g["pairs"]))]
    tokens, merges = sv.synthetic_vocab(pairs)
    tb, to = g["text_bytes"].tobytes(), g["text_off"]
    ids, io = g["ids"], g["ids_off"]
    texts = [tb[to[i]:to[i + 1]] for i in range(len(to) - 1)]
    want = [ids[io[i]:io[i + 1]].tolist() for i in range(len(to) - 1)]
    dec = [(int(i), bytes.fromhex(h), e) for i, (h, e) in zip(g["dec_ids"], json.loads(str(g["dec_bytes"])))]
    return {"tokens": tokens, "merges": merges, "texts": texts, "ids": want, "dec": dec,
            "specials": json.loads(str(g["specials"])),
            "chat": [(bytes.fromhex(h), c) for h, c in json.loads(str(g["chat"]))]}


@pytest.fixture(scope="module")
def tok(gold):
    t = Tokenizer(gold["tokens"], gold["merges"])
    yield t
    t.close()


@pytest.fixture(scope="module")
def ref(gold):
    return bpe.Tokenizer(gold["tokens"], gold["merges"])


def test_oracle_matches_reference_outputs(gold, ref):
    for text, want in zip(gold["texts"], gold["ids"]):
        assert ref.encode(text) == want, text[:80]
    for i, b, e in gold["dec"]:
        if e:
            with pytest.raises(RuntimeError, match=e):
                ref.decode(i)
        else:
            assert ref.decode(i) == b


def test_encode_matches_reference(gold, tok):
    for text, want in zip(gold["texts"], gold["ids"]):
        assert tok.encode(text) == want, text[:80]


def test_decode_and_special_match_reference(gold, tok):
    for i, b, e in gold["dec"]:
        if e:
            with pytest.raises(TokenizerError, match=e):
                tok.decode(i)
        else:
            assert tok.decode(i) == b
    for name, v in gold["specials"].items():
        if isinstance(v, str):
            with pytest.raises(TokenizerError, match=v):
                tok.special(name)
        else:
            assert tok.special(name) == v


def test_encode_matches_oracle_on_more_text(tok, ref):
    rng = random.Random(2024)
    for n in (1, 3, 10, 40, 150, 600):
        for _ in range(6):
            text = sv.random_text(rng, n).encode()
            assert tok.encode(text) == ref.encode(text), text[:80]
    # long pieces of one character class (the heap merge) and long mixed runs
    for text in (b"=" * 333, b" " * 257 + b"z", b"ab" * 150, b"abcdefghij" * 30, "ー".encode() * 90,
                 b"x" + b"\n" * 70, bytes(range(32, 127)) * 3):
        assert tok.encode(text) == ref.encode(text), text[:40]


def test_round_trip_and_chat_layout(tok, ref):
    rng = random.Random(5)
    for _ in range(20):
        text = sv.random_text(rng, 50).encode()
        assert b"".join(tok.decode(i) for i in tok.encode(text)) == text
    # the reference's chat prompt (inferencer.cu:1534-1551) built from these calls
    prompt = [tok.special("<|begin_of_text|>"), tok.special("<|start_header_id|>")] + tok.encode("user") + \
        [tok.special("<|end_header_id|>")] + tok.encode("\n\nHello there") + [tok.special("<|eot_id|>")]
    assert prompt[:2] == [128000, 128006] and prompt[-1] == 128009
    assert tok.encode("\n\nHello there") == ref.encode(b"\n\nHello there")


def test_chat_prompt_matches_reference(gold, tok):
    """chat_prompt (inferencer.cu:1534-1551) as the reference builds it."""
    for prompt, want in gold["chat"]:
        assert tok.chat_prompt(prompt) == want


def test_vocabulary_with_merges_that_make_no_token(gold):
    """A merge whose result is not a token: the reference keeps merging the
    string (and fails only if such a part survives); the product then uses its
    string path and gives the same ids or the same error."""
    tokens = list(gold["tokens"])
    merges = ["h e", "l l", "he ll", "hell o"] + list(gold["merges"])
    i_hell = tokens.index("hell") if "hell" in tokens else None
    if i_hell is not None:
        tokens[i_hell] = "<|no_hell|>"  # "he ll" now makes a string that is no token
    t = Tokenizer(tokens, merges)
    r = bpe.Tokenizer(tokens, merges)
    for text in (b"hello", b"hell", b"shell fish", b"hello hello world"):
        try:
            want = r.encode(text)
        except RuntimeError as e:
            with pytest.raises(TokenizerError, match=str(e)):
                t.encode(text)
        else:
            assert t.encode(text) == want
    t.close()


def test_errors_follow_the_reference(gold):
    with pytest.raises(TokenizerError, match="Expected Llama 3 tokenizer"):
        Tokenizer(gold["tokens"][:1000], gold["merges"])
    t = Tokenizer(gold["tokens"], gold["merges"])
    for bad in (-1, len(gold["tokens"])):
        with pytest.raises(TokenizerError, match="Invalid token id"):
            t.decode(bad)
    with pytest.raises(TokenizerError, match="Missing special token <|none|>"):
        t.special("<|none|>")
    assert t.encode(b"") == []
    t.close()


def test_concurrent_encodes_agree(tok, ref):
    rng = random.Random(9)
    texts = [sv.random_text(rng, 80).encode() for _ in range(16)]
    want = [ref.encode(x) for x in texts]
    got = [None] * len(texts)

    def run(k):
        for _ in range(5):
            got[k] = tok.encode(texts[k])

    threads = [threading.Thread(target=run, args=(k,)) for k in range(len(texts))]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    assert got == want


_SHIM_MAIN = r"""
#include "tokenizer.hpp"
#include <cstdio>
#include <fstream>
#include <iostream>
// the reference's GGUF members the tokenizer reads (inferencer.cu:207)
struct Model { std::vector<std::string> tokens, merges; };
static std::string unhex(const std::string &h) {
    std::string s;
    for (size_t i = 0; i + 1 < h.size(); i += 2) s.push_back(static_cast<char>(std::stoi(h.substr(i, 2), nullptr, 16)));
    return s;
}
int main(int argc, char **argv) {
    Model model;
    std::ifstream v(argv[1]);
    std::string line;
    bool merges = false;
    while (std::getline(v, line)) {
        if (line == "\x01---") { merges = true; continue; }
        (merges ? model.merges : model.tokens).push_back(unhex(line));
    }
    using ijb_host::Tokenizer;
    Tokenizer tok(model);
    std::ifstream t(argv[2]);
    while (std::getline(t, line)) {
        for (int id : tok.encode(unhex(line))) std::cout << id << ' ';
        std::cout << '\n';
    }
    std::cout << tok.special("<|eot_id|>") << ' ' << tok.decode(300).size() << '\n';
    try { tok.decode(-1); } catch (const std::runtime_error &e) { std::cout << e.what() << '\n'; }
    Model empty;
    try { Tokenizer bad(empty); } catch (const std::runtime_error &e) { std::cout << e.what() << '\n'; }
    return 0;
}
"""


def test_cpp_shim_matches_reference(gold, tmp_path):
    """The reference's call pattern through host/tokenizer.hpp (Tokenizer from
    a GGUF-like model; encode, special, decode; exceptions), compiled with g++
    and linked to libijb200.so, on the golden texts."""
    import os
    import shutil
    import subprocess
    from ijb200 import lib
    gxx = shutil.which("g++")
    if not gxx:
        pytest.skip("no g++")
    src = tmp_path / "main.cpp"
    src.write_text(_SHIM_MAIN)
    exe = tmp_path / "shim"
    libdir = os.path.join(lib.PKG_ROOT, "lib")
    r = subprocess.run([gxx, "-std=c++17", "-O1", "-I", os.path.join(lib.PKG_ROOT, "host"), str(src), "-L", libdir,
                        "-lijb200", f"-Wl,-rpath,{libdir}", "-Wl,--unresolved-symbols=ignore-in-shared-libs",
                        "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    vocab = tmp_path / "vocab.txt"
    vocab.write_text("\n".join(x.encode().hex() for x in gold["tokens"]) + "\n\x01---\n" +
                     "\n".join(x.encode().hex() for x in gold["merges"]) + "\n")
    texts = tmp_path / "texts.txt"
    texts.write_text("".join(t.hex() + "\n" for t in gold["texts"]))
    out = subprocess.run([str(exe), str(vocab), str(texts)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    lines = out.stdout.split("\n")
    for k, want in enumerate(gold["ids"]):
        assert [int(v) for v in lines[k].split()] == want, k
    n = len(gold["ids"])
    eot, n300 = lines[n].split()
    assert int(eot) == 128009 and int(n300) == len(bpe.Tokenizer(gold["tokens"], gold["merges"]).decode(300))
    assert lines[n + 1] == "Invalid token id"
    assert lines[n + 2] == "Expected Llama 3 tokenizer"


def test_batch_encode_matches_single_calls(gold, tok):
    """ijb_tokenizer_encode_batch on 1, 4 and all host threads (each worker
    with its own piece cache) gives every text the ids the reference gives it;
    a too-small buffer reports the count needed (IJB_ERR_CAPACITY) first."""
    import ctypes
    from ijb200 import lib
    texts = gold["texts"] * 3
    want = gold["ids"] * 3
    for threads in (1, 4, 0):
        assert tok.encode_batch(texts, threads) == want
    L = lib.load()
    ptrs = (ctypes.c_char_p * len(texts))(*texts)
    lens = (ctypes.c_long * len(texts))(*[len(t) for t in texts])
    offs = (ctypes.c_long * (len(texts) + 1))()
    buf = (ctypes.c_int * 4)()
    rc = L.ijb_tokenizer_encode_batch(tok.h, ptrs, lens, len(texts), buf, 4, offs, 2)
    assert rc == lib.ERR_CAPACITY and offs[len(texts)] == sum(map(len, want))
    assert tok.encode_batch([]) == []


_ALPHABET = (list("'sStTrReEvVmMlLdDxyzAQ019 \t\n\r\x0b\x0c.,;!?-_()[]{}\"#$%&*/\\@^`|~<>=+\x01\x1c\x1f\x7f") +
             ["'s", "'re", "'ll", "'VE", "  ", "\r\n", " \n", "\n\n", "é", "ß", "²", "٣", " ", "　",
              " ", "\u0085", "😀", "中", "Ⅻ", "½", "́", "\u2028", "Москва", "東京", "١٢٣٤", "\u00a0x", "x\u3000 "])


def test_scanner_matches_pcre(gold, tok):
    """The pre-tokenizer scanner (the pattern's alternatives over code point
    classes probed from PCRE2) against PCRE2 matching every piece
    (IJB_TOKENIZER_SCAN=0), on random strings built from the pattern's corner
    cases: contractions, letters, digits, every ASCII whitespace, CR/LF runs,
    punctuation, control bytes, and non-ASCII letters, numbers, spaces (NBSP,
    U+3000, NEL, U+2028), marks and symbols next to them.  Where the
    reference's own Tokenizer is built (oracle/_ref), it checks a share of the
    same strings too."""
    import ctypes
    import os
    import tempfile
    os.environ["IJB_TOKENIZER_SCAN"] = "0"
    try:
        pcre_only = Tokenizer(gold["tokens"], gold["merges"])
    finally:
        del os.environ["IJB_TOKENIZER_SCAN"]
    rng = random.Random(77)
    texts = ["".join(rng.choice(_ALPHABET) for _ in range(rng.randint(1, 40))).encode() for _ in range(8000)]
    for text in texts:
        assert tok.encode(text) == pcre_only.encode(text), text
    pcre_only.close()
    harness = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                           "libref_harness.so")
    if not os.path.exists(harness):
        return
    from gguf_writer import write_vocab_gguf
    lib = ctypes.CDLL(harness)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "vocab.gguf").encode()
        write_vocab_gguf(path.decode(), gold["tokens"], gold["merges"])
        buf = (ctypes.c_int * 512)()
        n = ctypes.c_long()
        for text in texts[:800]:
            assert lib.ref_tokenize(path, text, ctypes.c_long(len(text)), buf, ctypes.c_long(512), ctypes.byref(n)) == 0
            assert tok.encode(text) == list(buf[:n.value]), text
