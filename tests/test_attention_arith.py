"""The tensor-core decode attention's arithmetic, emulated in numpy on the CPU.

On the GPU the query and the softmax probabilities enter fp16 MMAs as a hi + lo
pair (hi = fp16(x), lo = fp16(x - hi), two MMAs each); products of fp16 values
are exact in the fp32 accumulator.  So, apart from fp32 accumulation order, the
only rounding left is the cache's own fp16 K/V.  This emulation checks that
claim against a float64 reference on the cached (fp16) K/V, and shows what a
single fp16 operand would cost instead."""
import numpy as np
import pytest


def _split(x):
    hi = x.astype(np.float16)
    lo = (x - hi.astype(np.float32)).astype(np.float16)
    return hi.astype(np.float32), lo.astype(np.float32)


def _attend(q, k16, v16, mode):
    """q [G, 64] fp32; k16, v16 [n, 64] fp16 (the cache).  mode: 'hilo' or 'single'."""
    k = k16.astype(np.float32)
    v = v16.astype(np.float32)
    if mode == "hilo":
        qh, ql = _split(q)
        s = (qh @ k.T).astype(np.float32) + (ql @ k.T).astype(np.float32)
    else:
        s = (q.astype(np.float16).astype(np.float32) @ k.T).astype(np.float32)
    s = s * np.float32(1.0 / 8.0)  # 1 / sqrt(64)
    m = s.max(axis=1, keepdims=True)
    p = np.exp(s - m).astype(np.float32)
    l = p.sum(axis=1, keepdims=True)
    if mode == "hilo":
        ph, pl = _split(p)
        o = ph @ v + pl @ v
    else:
        o = p.astype(np.float16).astype(np.float32) @ v
    return o / l


def _reference(q, k16, v16):
    k = k16.astype(np.float64)
    v = v16.astype(np.float64)
    s = (q.astype(np.float64) @ k.T) / 8.0
    p = np.exp(s - s.max(axis=1, keepdims=True))
    return (p @ v) / p.sum(axis=1, keepdims=True)


@pytest.mark.parametrize("n", [1, 37, 512, 1400])
def test_hi_lo_operands_leave_only_cache_rounding(n):
    rng = np.random.default_rng(n)
    q = (3.0 * rng.standard_normal((4, 64))).astype(np.float32)  # large scores stress the rounding
    k16 = rng.standard_normal((n, 64)).astype(np.float16)
    v16 = rng.standard_normal((n, 64)).astype(np.float16)
    ref = _reference(q, k16, v16)
    got = _attend(q, k16, v16, "hilo")
    err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert err < 2e-6, err


def test_single_fp16_operands_are_much_coarser():
    rng = np.random.default_rng(7)
    q = (3.0 * rng.standard_normal((4, 64))).astype(np.float32)
    k16 = rng.standard_normal((512, 64)).astype(np.float16)
    v16 = rng.standard_normal((512, 64)).astype(np.float16)
    ref = _reference(q, k16, v16)
    e_hilo = np.linalg.norm(_attend(q, k16, v16, "hilo") - ref) / np.linalg.norm(ref)
    e_single = np.linalg.norm(_attend(q, k16, v16, "single") - ref) / np.linalg.norm(ref)
    assert e_single > 50 * e_hilo, (e_single, e_hilo)
