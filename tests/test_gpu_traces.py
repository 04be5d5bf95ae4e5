"""Debug traces of FastRunner::forward / prefill (inferencer.cu:1279-1283,
:1424-1426) through ijb_forward_traced / ijb_prefill_traced: per-layer
residuals and the int8 activations the INT8 path quantises in each layer,
checked against the CPU oracle, and the reference's --compare-prefill use
(inferencer.cu:1707-1833): token-by-token and packed prefill traces of the
same prompt agree.  Traced steps give the same tokens and logits as untraced
ones."""
import numpy as np
import pytest

import oracle as O
from ijb200 import synth
from ijb200.engine import Engine

pytestmark = pytest.mark.gpu


def test_forward_traces_match_the_oracle(cuda):
    cfg = synth.TINY
    w = synth.make_model(cfg, seed=11)
    prompt = synth.prompt_tokens(6, seed=1, vocab_limit=cfg.vocab)
    eng = Engine(cfg, w, context=32, max_batch=1, max_seqs=2, kv_f32=True)
    plain = Engine(cfg, w, context=32, max_batch=1, max_seqs=2, kv_f32=True)
    om = O.OracleModel(cfg, w, 32, True, True)
    st = om.new_state()
    for i, t in enumerate(prompt):
        nxt, lt, qt = eng.forward_traced(int(t), i, True)
        assert plain.forward(int(t), i, True) == nxt
        assert np.array_equal(eng.logits(1), plain.logits(1))
        want, trace = st.forward(int(t), i, True, trace=True)
        assert nxt == want
        rel = np.linalg.norm(lt - trace, axis=1) / np.linalg.norm(trace, axis=1)
        assert rel.max() < 1e-4, rel
        # the attention input of layer 0 is rmsnorm(embedding) quantised: the
        # oracle's codes from the same residual (the embedding is exact)
        x0 = O.dequant(14, w["token_embd.weight"][int(t)]).astype(np.float32)
        xq, _ = O.quantize_x32(O.rmsnorm(x0, w["blk.0.attn_norm.weight"], cfg.eps))
        assert np.mean(qt[0, :cfg.dim] == xq) > 0.99
        assert np.abs(qt).max() <= 127
    eng.close()
    plain.close()


@pytest.mark.parametrize("max_batch", [8, 64])
def test_prefill_traces_agree_with_token_by_token(cuda, max_batch):
    cfg = synth.TINY
    w = synth.make_model(cfg, seed=12)
    prompt = synth.prompt_tokens(21, seed=2, vocab_limit=cfg.vocab)
    # FP32 activation path: the INT8 path's requantisation would turn the
    # tensor-core path's fp16 rounding into ~1% differences (its own floor)
    eng = Engine(cfg, w, context=64, max_batch=max_batch, max_seqs=2, use_dp4a=False, use_q6_dp4a=False)
    nxt, allt, fq, lq = eng.prefill_traced(prompt)
    seq = Engine(cfg, w, context=64, max_batch=1, max_seqs=2, use_dp4a=False, use_q6_dp4a=False)
    for i, t in enumerate(prompt):
        n1, lt, qt = seq.forward_traced(int(t), i, i + 1 == len(prompt))
        tol = 5e-3 if max_batch >= 16 else 1e-5  # the tensor-core path rounds to fp16
        rel = np.linalg.norm(allt[i] - lt, axis=1) / np.linalg.norm(lt, axis=1)
        assert rel.max() < tol, (i, rel)
        if i == 0:
            assert np.mean(fq == qt) > 0.95
    assert np.mean(lq == qt) > 0.95
    assert nxt == n1
    eng.close()
    seq.close()
