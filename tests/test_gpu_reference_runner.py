"""The B200 engine against the reference's own full-model forward.

tests/golden/ref_runner_3b.npz holds what the reference's GGUF +
FastRunner::forward (inferencer.cu:204-340, :1424-1531), built unmodified for
sm_100a, returned on a B200 for a seeded random-init model of the only shape
it accepts (Llama-3.2-3B: 28 layers, dim 3072, 24 / 8 heads, head_dim 128,
FFN 8192, vocab 128256, :1215-1217), 20 tokens at positions 0..19 with logits
at every step (tests/golden/make_ref_runner_golden.py).  The engine runs the
same model and tokens two ways:
* token by token (ijb_forward, the CUDA-core GEMV path of batch-1 decode);
* as one 20-token packed prefill (the tensor-core path), all 20 rows of logits.
Bars: FP32 activation path, sampled logits rel-L2 <= 1e-2 and every argmax
equal; INT8 path (the reference default), twice the path's own floor (the
CPU oracle against itself with one multiply-add contraction changed,
measured here on the same tokens), and an argmax agreement within two of
the 20 steps of the oracle's own agreement with the reference on this path
(19 of 20: a flipped int8 code can move a near-tie)."""
import os

import numpy as np
import pytest

import oracle as O
from ijb200 import synth
from ijb200.engine import Engine

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_runner_3b.npz")


@pytest.fixture(scope="module")
def golden():
    if not os.path.exists(GOLDEN):
        pytest.skip("tests/golden/ref_runner_3b.npz not captured yet")
    g = dict(np.load(GOLDEN))
    return g, synth.make_model(synth.LLAMA_3B, seed=int(g["seed"]))


def _rel(lg, g, tag):
    rows = g["sample_rows"]
    a, b = lg[:, rows].astype(np.float64), g[f"{tag}_sample"].astype(np.float64)
    return np.linalg.norm(a - b, axis=1) / np.linalg.norm(b, axis=1)


def _int8_floor(weights, toks, rows, ref_next):
    """The INT8 path's own floor on these tokens: the oracle against itself
    with one contraction changed (logits), and the oracle's argmax agreement
    with the reference runner."""
    O.set_threads(16)
    out, nxt = [], None
    for c in (1, 0):
        m = O.OracleModel(synth.LLAMA_3B, weights, 64, True, True, contract=c)
        st = m.new_state()
        n, lg = m.forward_multi([st] * len(toks), toks, np.arange(len(toks)), True, want_logits=True)
        out.append(lg)
        nxt = n if nxt is None else nxt
    floor = np.linalg.norm((out[0] - out[1])[:, rows], axis=1) / np.linalg.norm(out[0][:, rows], axis=1)
    return floor, float(np.mean(nxt == ref_next))


@pytest.mark.parametrize("tag,dp4a", [("fp32", False), ("int8", True)])
@pytest.mark.parametrize("mode", ["token-by-token", "packed-prefill"])
def test_engine_matches_reference_runner_3b(cuda, golden, tag, dp4a, mode):
    g, weights = golden
    toks = [int(t) for t in g["tokens"]]
    n = len(toks)
    if mode == "token-by-token":
        eng = Engine(synth.LLAMA_3B, weights, context=64, max_batch=1, max_seqs=2, use_dp4a=dp4a, use_q6_dp4a=dp4a)
        nxt, lg = [], []
        for i, t in enumerate(toks):
            nxt.append(eng.forward(t, i, True))
            lg.append(eng.logits(1)[0])
        lg = np.stack(lg)
    else:
        eng = Engine(synth.LLAMA_3B, weights, context=64, max_batch=64, max_seqs=2, use_dp4a=dp4a, use_q6_dp4a=dp4a)
        eng.prefill(toks)
        lg = eng.logits(n)
        nxt = [int(np.argmax(r)) for r in lg]  # the step's argmax keys follow the same tie rule
    eng.close()
    rel = _rel(lg, g, tag)
    agree = float(np.mean(np.array(nxt) == g[f"{tag}_next"]))
    print(f"\n3B {mode} {tag}: sampled logits rel-L2 max {rel.max():.3e} mean {rel.mean():.3e}; argmax {agree:.3f}")
    if not dp4a:
        assert rel.max() <= 1e-2, rel
        assert agree == 1.0
    else:
        floor, oracle_agree = _int8_floor(weights, g["tokens"], g["sample_rows"], g[f"{tag}_next"])
        print(f"int8 floor max {floor.max():.3e} mean {floor.mean():.3e}; oracle argmax agreement {oracle_agree:.3f}")
        assert rel.max() <= 2 * floor.max(), (rel.max(), floor.max())
        # within two of the 20 steps of what the oracle itself reaches on this path
        assert agree >= oracle_agree - 0.1, (agree, oracle_agree)
