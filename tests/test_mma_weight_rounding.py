"""The tensor-core path's weight conversion, emulated in numpy on the CPU and
checked against the oracle's exact dequantisation (q4_value / q6_value).

The GPU converts each weight with fp16 arithmetic under a per-matrix power of
two 2^e (e from the largest possible |w| of the matrix's blocks, so that every
scaled weight is below 2^15): Q4_K q * fp16(d*sc*2^e) + fp16(-dmin*m*2^e) with
one fp16 rounding of the fused multiply-add; Q6_K (q - 32) * fp16(d*2^e*sc)
with one fp16 rounding of the product.  Both scale products are rounded to
fp16 as well, so the worst error on random blocks is ~7.7e-4 of max|w| for
Q4_K and ~4.9e-4 for Q6_K; the tests hold both to 1e-3."""
import math

import numpy as np

import oracle as O
from ijb200 import synth

Q4_K, Q6_K = 12, 14


def _f16(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def _fma16(a, b, c):
    # one rounding of a*b + c (a, b, c fp16 values; the product is exact in float64)
    return (np.asarray(a, np.float64) * np.asarray(b, np.float64) + np.asarray(c, np.float64)).astype(np.float16).astype(np.float32)


def _scale_exp(bound: float) -> int:
    _, ex = math.frexp(bound)
    return max(-60, min(60, 15 - ex))


def _q4_tensor_core(blocks: np.ndarray):
    b = blocks.reshape(-1, 144)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(-1)
    dmin = b[:, 2:4].copy().view(np.float16).astype(np.float32).reshape(-1)
    s = b[:, 4:16].astype(np.int32)
    qs = b[:, 16:144].astype(np.int32)
    bound = float(np.max(np.abs(d) * 945.0 + np.abs(dmin) * 63.0))
    e = _scale_exp(bound)
    scale = np.float32(2.0 ** e)
    out = np.empty((b.shape[0], 256), np.float32)
    for j in range(8):
        if j < 4:
            sc, m = s[:, j] & 63, s[:, j + 4] & 63
        else:
            sc = (s[:, j + 4] & 15) | ((s[:, j - 4] >> 6) << 4)
            m = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
        s1 = _f16(d * sc.astype(np.float32) * scale)
        n2 = _f16(-(dmin * m.astype(np.float32) * scale))
        for i in range(32 * j, 32 * j + 32):
            byte = qs[:, (i // 64) * 32 + i % 32]
            q = byte & 15 if i % 64 < 32 else byte >> 4
            out[:, i] = _fma16(q.astype(np.float32), s1, n2)
    return out.reshape(-1), e


def _q6_tensor_core(blocks: np.ndarray):
    b = blocks.reshape(-1, 210)
    ql = b[:, 0:128].astype(np.int32)
    qh = b[:, 128:192].astype(np.int32)
    sc = b[:, 192:208].view(np.int8).astype(np.float32)
    d = b[:, 208:210].copy().view(np.float16).astype(np.float32).reshape(-1)
    e = _scale_exp(float(np.max(np.abs(d) * 128.0 * 32.0)))
    dd = d * np.float32(2.0 ** e)
    out = np.empty((b.shape[0], 256), np.float32)
    for i in range(256):
        g, p = divmod(i, 128)
        lane, part = p % 32, p // 32
        lowb = ql[:, g * 64 + (part % 2) * 32 + lane]
        low = lowb & 15 if part < 2 else lowb >> 4
        high = (qh[:, g * 32 + lane] >> (2 * part)) & 3
        q = (low | (high << 4)) - 32
        s = _f16(dd * sc[:, g * 8 + part * 2 + lane // 16])
        out[:, i] = (q.astype(np.float64) * s.astype(np.float64)).astype(np.float16).astype(np.float32)
    return out.reshape(-1), e


def _check(qtype, blocks, conv, bound):
    exact = O.dequant(qtype, blocks).astype(np.float64)
    w16, e = conv(blocks)
    assert np.all(np.abs(w16) < 2.0 ** 15)
    err = np.max(np.abs(w16.astype(np.float64) * 2.0 ** -e - exact)) / np.max(np.abs(exact))
    assert err <= bound, err
    return err


def test_q4k_tensor_core_weights_within_bound():
    rng = np.random.default_rng(1)
    blocks = synth.q4k_blocks(rng, 256)
    _check(Q4_K, blocks, _q4_tensor_core, 1e-3)


def test_q6k_tensor_core_weights_within_bound():
    rng = np.random.default_rng(2)
    blocks = synth.q6k_blocks(rng, 256)
    _check(Q6_K, blocks, _q6_tensor_core, 1e-3)
