"""Synthetic Llama-3-sized tokenizer data for tests and benchmarks: seeded
text, byte-level BPE merges trained on it, and a 128256-token vocabulary
around them (the real vocabulary and merges come from a GGUF file, which this
environment does not have).  Data generation only; the tokenizer itself is
ijb200.tokenizer (C ABI ijb_tokenizer_*)."""
from __future__ import annotations

import random

import regex

LLAMA3_VOCAB = 128256
# Llama 3's pre-tokenizer pattern (the one GGUF Llama-3 tokenizers use), to
# split the training text into pieces the way encoding will
PATTERN = (r"(?:'[sS]|'[tT]|'[rR][eE]|'[vV][eE]|'[mM]|'[lL][lL]|'[dD])|"
           r"[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}|"
           r" ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+")
_RE = regex.compile(PATTERN)

SPECIALS = ["<|begin_of_text|>", "<|end_of_text|>", "<|reserved_special_token_0|>",
            "<|reserved_special_token_1|>", "<|finetune_right_pad_id|>", "<|reserved_special_token_2|>",
            "<|start_header_id|>", "<|end_header_id|>", "<|eom_id|>", "<|eot_id|>", "<|python_tag|>"]


def byte_symbols() -> list[str]:
    """GGUF byte-level BPE symbols in byte order: bytes 33-126, 161-172 and
    174-255 stand for themselves, every other byte for the next code point
    from 256 up."""
    out, cp = [], 256
    for b in range(256):
        plain = 33 <= b <= 126 or 161 <= b <= 172 or b >= 174
        out.append(chr(b) if plain else chr(cp))
        if not plain:
            cp += 1
    return out


BYTE_SYMBOL = byte_symbols()


def _pieces(text: bytes) -> list[bytes]:
    try:
        s = text.decode("utf-8")
    except UnicodeDecodeError:
        return [text]
    return [m.group().encode("utf-8") for m in _RE.finditer(s)]


# ----------------------------------------------------------- synthetic data --

_WORDS = ("the of and to in is was for on that with as by at from his her they have this are be not "
          "were had which their an one all but been has more when there some would can who what will "
          "about if out so up said into time them only other new could also two first then after "
          "these may people any over such through where most state world year work between both under "
          "great during without water life government system program information development "
          "university international hello Hello THE And Über straße café naïve résumé jalapeño "
          "Москва данные 東京 数据 δεδομένα שלום مرحبا नमस्ते").split()
_PUNCT = list(".,;:!?-()[]{}\"'/\\@#$%^&*_+=<>|~`")
_UNI = ["é", "ß", "ø", "ñ", "ü", "ж", "ω", "λ", "中", "文", "日", "😀", "🚀", "👍🏽", "é", " ", " ",
        "　", "١٢٣", "Ⅻ", "½", "²", "𝔘"]


def random_text(rng: random.Random, n_items: int) -> str:
    """Seeded text mixing words, contractions, numbers, punctuation, Unicode
    letters and symbols, and runs of spaces, tabs and newlines."""
    out = []
    for _ in range(n_items):
        r = rng.random()
        if r < 0.55:
            w = rng.choice(_WORDS)
            if rng.random() < 0.1:
                w = w.upper() if rng.random() < 0.5 else w.capitalize()
            if rng.random() < 0.08:
                w += rng.choice(["'s", "'t", "'re", "'ve", "'m", "'ll", "'d", "'S", "'LL", "'x"])
            out.append(w)
        elif r < 0.65:
            out.append(str(rng.randrange(0, 10 ** rng.randint(1, 9))))
        elif r < 0.78:
            out.append("".join(rng.choice(_PUNCT) for _ in range(rng.randint(1, 3))))
        elif r < 0.86:
            out.append(rng.choice(_UNI) * rng.randint(1, 2))
        else:
            out.append(rng.choice([" ", "  ", "\t", "\n", "\n\n", "\r\n", " \n ", "   \n", "\n\t "]))
        out.append(" " if rng.random() < 0.8 else "")
    return "".join(out)


def train_merges(corpus: list[bytes], n_merges: int) -> list[tuple[str, str]]:
    """Plain byte-level BPE training over the corpus's pieces: repeatedly merge
    the most frequent adjacent symbol pair (ties: the smaller pair)."""
    words: dict[tuple[str, ...], int] = {}
    for text in corpus:
        for p in _pieces(text):
            key = tuple(BYTE_SYMBOL[b] for b in p)
            words[key] = words.get(key, 0) + 1
    merges = []
    for _ in range(n_merges):
        counts: dict[tuple[str, str], int] = {}
        for w, c in words.items():
            for a, b in zip(w, w[1:]):
                counts[(a, b)] = counts.get((a, b), 0) + c
        if not counts:
            break
        best = max(counts.items(), key=lambda kv: (kv[1], [-ord(ch) for ch in kv[0][0] + kv[0][1]]))[0]
        merges.append(best)
        new_words = {}
        for w, c in words.items():
            out, i = [], 0
            while i < len(w):
                if i + 1 < len(w) and (w[i], w[i + 1]) == best:
                    out.append(w[i] + w[i + 1])
                    i += 2
                else:
                    out.append(w[i])
                    i += 1
            new_words[tuple(out)] = new_words.get(tuple(out), 0) + c
        words = new_words
    return merges


def synthetic_vocab(pairs: list[tuple[str, str]]) -> tuple[list[str], list[str]]:
    """A Llama-3-sized vocabulary around trained merges: the 256 byte symbols,
    the merge results, fillers up to 128000, then the special tokens (ids
    128000-128010 as in Llama 3) and reserved ones up to 128256.  The merge
    list adds a repeated merge at a later rank (the first rank counts) and two
    merges whose halves are no tokens (they can never apply)."""
    tokens = list(BYTE_SYMBOL)
    seen = set(tokens)
    for a, b in pairs:
        if a + b not in seen:
            tokens.append(a + b)
            seen.add(a + b)
    i = 0
    while len(tokens) < 128000:
        t = f"<|filler_{i}|>"
        i += 1
        if t not in seen:
            tokens.append(t)
            seen.add(t)
    tokens += SPECIALS
    j = 3
    while len(tokens) < LLAMA3_VOCAB:
        tokens.append(f"<|reserved_special_token_{j}|>")
        j += 1
    merges = [a + " " + b for a, b in pairs]
    if merges:
        merges.append(merges[len(merges) // 2])
    merges += ["zzq xxq", "ĀĀĀ qqq"]
    return tokens, merges


def training_corpus() -> list[bytes]:
    """The seeded text the synthetic merges are trained on, with long runs and
    long words so that long pieces merge too."""
    rng = random.Random(7)
    texts = [random_text(rng, 120).encode() for _ in range(80)]
    texts += [b"=" * 48 + b"\n" + b"-" * 40, b" " * 64 + b"x", b"aaaaaaaaaaaaaaaaaaaaaaaaaaaaaaaaaaaa",
              b"internationalization internationalisation", b"Supercalifragilisticexpialidocious " * 3,
              "ーーーーーーーーーー".encode(), b"0123456789" * 4, b"!!!!!!!!!!!!!!!!!!!!!!!!!!!!!!"]
    return texts


def vocabulary(n_merges: int = 700) -> tuple[list[str], list[str]]:
    """The synthetic (tokens, merges) the tests and the bench use."""
    return synthetic_vocab(train_merges(training_corpus(), n_merges))
