"""Seeded synthetic GGUF-layout weights and workloads.

There are no real checkpoints or datasets on the build or GPU machines, so every
model here is random-init with the Llama-3.2 architecture and the Q4_K_M
quantisation mix the reference runs (Q4_K for attn_q/k/output and ffn_gate/up;
Q6_K for attn_v, ffn_down and the tied token_embd / lm_head).  Blocks are laid
out byte for byte as GGUF stores them (the reference reads them in place,
inferencer.cu:453-497):

* Q4_K, 144 B per 256 weights: fp16 d @0, fp16 dmin @2, 12 packed 6-bit
  scale/min bytes @4, 128 bytes of 4-bit quants @16.  Every bit of the 12
  scale bytes belongs to exactly one 6-bit scale or min, so uniform random
  bytes give scales and mins uniform on 0..63.
* Q6_K, 210 B per 256 weights: ql[128] @0, qh[64] @128, int8 scales[16] @192,
  fp16 d @208.
"""
from __future__ import annotations

import dataclasses

import numpy as np

Q4_K = 12
Q6_K = 14
F32 = 0

BLOCK_BYTES = {Q4_K: 144, Q6_K: 210}
TYPE_NAME = {Q4_K: "Q4_K", Q6_K: "Q6_K", F32: "F32"}


def _f16_bytes(values: np.ndarray) -> np.ndarray:
    return values.astype(np.float16).view(np.uint8).reshape(-1, 2)


def q4k_blocks(rng: np.random.Generator, nblocks: int, d_range=(1e-3, 1e-2),
               dmin_range=(1e-3, 1e-2)) -> np.ndarray:
    """[nblocks, 144] uint8 Q4_K super-blocks: d, dmin ~ U(range) as fp16,
    scale/min bytes and 4-bit quants uniform."""
    out = np.empty((nblocks, 144), dtype=np.uint8)
    out[:, 0:2] = _f16_bytes(rng.uniform(*d_range, nblocks).astype(np.float32))
    out[:, 2:4] = _f16_bytes(rng.uniform(*dmin_range, nblocks).astype(np.float32))
    out[:, 4:144] = rng.integers(0, 256, size=(nblocks, 140), dtype=np.uint8)
    return out


def q6k_blocks(rng: np.random.Generator, nblocks: int, d_range=(1e-4, 1e-3),
               scale_range=(-32, 31)) -> np.ndarray:
    """[nblocks, 210] uint8 Q6_K super-blocks: ql/qh bits uniform, int8 scales
    uniform on scale_range (inclusive), d ~ U(d_range) as fp16."""
    out = np.empty((nblocks, 210), dtype=np.uint8)
    out[:, 0:192] = rng.integers(0, 256, size=(nblocks, 192), dtype=np.uint8)
    sc = rng.integers(scale_range[0], scale_range[1] + 1, size=(nblocks, 16), dtype=np.int16)
    out[:, 192:208] = sc.astype(np.int8).view(np.uint8)
    out[:, 208:210] = _f16_bytes(rng.uniform(*d_range, nblocks).astype(np.float32))
    return out


def quant_matrix(rng, qtype: int, rows: int, cols: int, **kw) -> np.ndarray:
    """[rows, cols/256*block_bytes] uint8, rows of consecutive super-blocks
    (row_data = w + row*(cols/256)*bytes, inferencer.cu:563, :652)."""
    assert cols % 256 == 0
    nb = rows * (cols // 256)
    blocks = q4k_blocks(rng, nb, **kw) if qtype == Q4_K else q6k_blocks(rng, nb, **kw)
    return blocks.reshape(rows, (cols // 256) * BLOCK_BYTES[qtype])


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    name: str
    dim: int
    layers: int
    heads: int
    kv_heads: int
    hidden: int
    vocab: int
    rope_base: float = 500000.0
    eps: float = 1e-5
    attn_v_type: int = Q6_K
    ffn_down_type: int = Q6_K

    @property
    def head_dim(self) -> int:
        return self.dim // self.heads

    @property
    def kv_dim(self) -> int:
        return self.head_dim * self.kv_heads

    def type_of(self, short: str) -> int:
        if short == "attn_v":
            return self.attn_v_type
        if short == "ffn_down":
            return self.ffn_down_type
        if short in ("token_embd", "output"):
            return Q6_K
        return Q4_K

    def matrices(self):
        """(name, type, rows, cols) of every quantised matrix, in layer order."""
        out = []
        for l in range(self.layers):
            p = f"blk.{l}."
            out += [
                (p + "attn_q.weight", Q4_K, self.dim, self.dim),
                (p + "attn_k.weight", Q4_K, self.kv_dim, self.dim),
                (p + "attn_v.weight", self.attn_v_type, self.kv_dim, self.dim),
                (p + "attn_output.weight", Q4_K, self.dim, self.dim),
                (p + "ffn_gate.weight", Q4_K, self.hidden, self.dim),
                (p + "ffn_up.weight", Q4_K, self.hidden, self.dim),
                (p + "ffn_down.weight", self.ffn_down_type, self.dim, self.hidden),
            ]
        out.append(("token_embd.weight", Q6_K, self.vocab, self.dim))
        return out

    def weight_bytes(self) -> int:
        """Quantised + norm bytes one decode step reads (lm_head is the tied
        embedding, read once for the logits)."""
        total = 0
        for _, t, rows, cols in self.matrices():
            total += rows * (cols // 256) * BLOCK_BYTES[t]
        total += (2 * self.layers + 1) * self.dim * 4
        return total

    def kv_bytes_per_token(self, elem_bytes: int = 2) -> int:
        """K and V bytes one cached token occupies across all layers."""
        return 2 * self.layers * self.kv_dim * elem_bytes


# Llama-3.2 shapes and a small shape for fast tests.
LLAMA_1B = ModelConfig("llama-3.2-1b", dim=2048, layers=16, heads=32, kv_heads=8, hidden=8192, vocab=128256)
LLAMA_3B = ModelConfig("llama-3.2-3b", dim=3072, layers=28, heads=24, kv_heads=8, hidden=8192, vocab=128256)
TINY = ModelConfig("tiny", dim=512, layers=2, heads=8, kv_heads=2, hidden=1024, vocab=4096)
TINY_HD128 = ModelConfig("tiny-hd128", dim=512, layers=2, heads=4, kv_heads=2, hidden=768, vocab=2048)
# three query heads per KV head, as in the 3B shape (24 / 8)
TINY_G3 = ModelConfig("tiny-g3", dim=768, layers=2, heads=12, kv_heads=4, hidden=1024, vocab=4096)
TINY_HD128_G3 = ModelConfig("tiny-hd128-g3", dim=768, layers=2, heads=6, kv_heads=2, hidden=768, vocab=2048)

# Weight scale ranges for random-init models.  They are chosen so every
# projection of a unit-RMS input has roughly unit RMS output (sigma_w close to
# 1/sqrt(cols)): activations, K and V then stay far inside fp16 range at every
# layer (checked by tests/test_oracle.py::test_model_activation_range).
def _q4_model_kw(cols):
    a = 0.55 / (np.sqrt(cols) * 31.5 * 8.8)
    return dict(d_range=(a, 2 * a), dmin_range=(7.5 * a, 15 * a))


def _q6_model_kw(cols):
    a = 0.8 / (np.sqrt(cols) * 18.5 * 18.5)
    return dict(d_range=(a, 2 * a))


def make_model(cfg: ModelConfig, seed: int = 0):
    """Random-init weights for `cfg` as {GGUF tensor name: array}: quantised
    matrices as [rows, row_bytes] uint8, norm weights as float32 [dim]."""
    rng = np.random.default_rng(seed)
    w = {}
    for name, t, rows, cols in cfg.matrices():
        kw = _q4_model_kw(cols) if t == Q4_K else _q6_model_kw(cols)
        if name == "token_embd.weight":
            # the tied lm_head: larger entries give logits of unit-ish spread
            kw = dict(d_range=(kw["d_range"][0] * 4, kw["d_range"][1] * 4))
        w[name] = quant_matrix(rng, t, rows, cols, **kw)
    for l in range(cfg.layers):
        w[f"blk.{l}.attn_norm.weight"] = rng.uniform(0.8, 1.2, cfg.dim).astype(np.float32)
        w[f"blk.{l}.ffn_norm.weight"] = rng.uniform(0.8, 1.2, cfg.dim).astype(np.float32)
    w["output_norm.weight"] = rng.uniform(0.8, 1.2, cfg.dim).astype(np.float32)
    return w


def prompt_tokens(n: int, seed: int = 1, vocab_limit: int = 128000) -> np.ndarray:
    """Prompt token ids uniform in [0, vocab_limit) (BASELINE decode config)."""
    return np.random.default_rng(seed).integers(0, vocab_limit, size=n).astype(np.int32)


@dataclasses.dataclass
class RaggedRequest:
    prompt: np.ndarray
    max_new: int


def ragged_requests(count: int, prompt_range=(16, 1024), output_range=(32, 256), seed: int = 2,
                    vocab_limit: int = 128000):
    """Requests for the ragged continuous-batching workload: prompt lengths
    and target output lengths uniform on the inclusive ranges."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(count):
        plen = int(rng.integers(prompt_range[0], prompt_range[1] + 1))
        out.append(RaggedRequest(rng.integers(0, vocab_limit, size=plen).astype(np.int32),
                                 int(rng.integers(output_range[0], output_range[1] + 1))))
    return out
