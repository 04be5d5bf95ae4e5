"""ijb_generate (device-side greedy loop) against the same loop run from the
host with ijb_decode_step, following the reference's decode loop
(inferencer.cu:1870-1883): a stop id ends it unemitted, max_tokens emitted
tokens or the context end it after emitting."""
import numpy as np
import pytest

from ijb200 import synth
from ijb200.engine import Engine

pytestmark = pytest.mark.gpu


def host_loop(eng, seq, first, max_tokens, stops, context):
    """The reference loop on the host: returns the emitted tokens."""
    pos0 = eng.seq_length(seq)
    out, nxt = [], first
    for i in range(max_tokens):
        if nxt in stops:
            break
        out.append(int(nxt))
        if i + 1 == max_tokens or pos0 + i >= context:
            break
        nxt = int(eng.decode_step([seq], [nxt])[0])
    return out


def _pair(cfg, weights, prompt, context, max_batch):
    a = Engine(cfg, weights, context=context, max_batch=max_batch, max_seqs=3)
    b = Engine(cfg, weights, context=context, max_batch=max_batch, max_seqs=3)
    sa, sb = a.seq_open(), b.seq_open()
    fa, fb = a.seq_prefill(sa, prompt), b.seq_prefill(sb, prompt)
    assert fa == fb
    return a, b, sa, sb, fa


@pytest.mark.parametrize("max_batch", [1, 64])
def test_generate_matches_host_loop(cuda, max_batch):
    cfg = synth.TINY
    weights = synth.make_model(cfg, seed=17)
    prompt = synth.prompt_tokens(24, seed=3, vocab_limit=cfg.vocab)
    context = 128
    a, b, sa, sb, first = _pair(cfg, weights, prompt, context, max_batch)
    want = host_loop(b, sb, first, 40, set(), context)
    got = a.generate(sa, first, 40)
    assert got == want and len(got) == 40
    assert a.seq_length(sa) == b.seq_length(sb) == len(prompt) + 39
    # the caches agree: one more step on both gives the same token and logits
    ta = a.decode_step([sa], [got[-1]])[0]
    tb = b.decode_step([sb], [want[-1]])[0]
    assert ta == tb
    np.testing.assert_array_equal(a.logits(1).view(np.uint32), b.logits(1).view(np.uint32))
    a.close()
    b.close()


def test_generate_stop_ids_context_and_empty(cuda):
    cfg = synth.TINY
    weights = synth.make_model(cfg, seed=18)
    prompt = synth.prompt_tokens(20, seed=4, vocab_limit=cfg.vocab)
    # a stop id taken from the free-running sequence: the loop ends before it
    a, b, sa, sb, first = _pair(cfg, weights, prompt, 96, 1)
    free = a.generate(sa, first, 30)
    stop = free[7]
    a.close()
    b.close()
    a, b, sa, sb, first = _pair(cfg, weights, prompt, 96, 1)
    got = a.generate(sa, first, 30, stop_ids=[stop, cfg.vocab - 1])
    want = host_loop(b, sb, first, 30, {stop, cfg.vocab - 1}, 96)
    assert got == want and stop not in got and len(got) <= 7
    assert a.seq_length(sa) == b.seq_length(sb)
    # the sequence keeps decoding normally afterwards
    assert a.decode_step([sa], [5])[0] == b.decode_step([sb], [5])[0]
    a.close()
    b.close()
    # the context ends the loop: 20-token prompt, context 32
    a, b, sa, sb, first = _pair(cfg, weights, prompt, 32, 1)
    got = a.generate(sa, first, 100)
    want = host_loop(b, sb, first, 100, set(), 32)
    assert got == want and a.seq_length(sa) == b.seq_length(sb) == 32
    # the first token itself is a stop id: nothing is emitted or fed
    n0 = a.seq_length(sa)
    assert a.generate(sa, 3, 10, stop_ids=[3]) == []
    assert a.seq_length(sa) == n0
    a.close()
    b.close()
