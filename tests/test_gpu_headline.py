"""Parity of the benchmarked path at its own shape: the tensor-core ragged
decode step of the Llama-3.2-1B-width model with 64 live sequences, against
the CPU oracle's restatement of FastRunner::forward (inferencer.cu:1424-1531)
run on the same tokens, teacher-forced.

Shape: dim 2048, FFN 8192, 32 query / 8 KV heads (head_dim 64), vocab 128256,
2 of the model's 16 layers (the CPU oracle stays within minutes); 64
sequences with prompts U[16, 1024] (the bench workload's distribution), 32
decode steps, plus 128 steps on 16 of the sequences.  The oracle runs its
packed forward (orc_forward_multi: the per-token arithmetic of orc_forward,
layer by layer over all entries) with the engine's fp16 KV format.

Bars (the project's stated tolerances):
* every projection at the 1B shapes (Q4_K q/k/o/gate/up, Q6_K v/down and the
  128256-row lm_head), 64 tokens: rel-L2 <= 1e-3 against the oracle;
* FP32 activation path: logits rel-L2 <= 1e-2 at every step, >= 99% greedy
  top-1 agreement;
* INT8 activation path (the reference's default: per-32 int8 activations and
  __dp4a dots, inferencer.cu:520-556, :613-643): every ulp-level difference
  can flip int8 codes at the next projection, so two CPU restatements of the
  reference that differ only in one multiply-add contraction already disagree
  by ~1% here.  The test measures that floor on the same model and sequences
  (oracle contract=1 against contract=0) and holds the GPU to twice it (max and
  mean over steps), with >= 99% greedy agreement.
The top-2 logit margins of the steps are printed with the results."""
import numpy as np
import pytest

import oracle as O
from ijb200 import synth
from ijb200.engine import Engine

pytestmark = pytest.mark.gpu

CFG = synth.ModelConfig("llama-1b-width-2layer", dim=2048, layers=2, heads=32, kv_heads=8, hidden=8192,
                        vocab=128256)
NSEQ, STEPS, LONG_SEQS, LONG_STEPS = 64, 32, 16, 128
PROJ_BAR = 1e-3
FP32_BAR = 1e-2
GREEDY_BAR = 0.99


def rel_l2(a, b):
    a = np.asarray(a, np.float64); b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def model():
    return synth.make_model(CFG, seed=3)


@pytest.fixture(scope="module")
def requests():
    return synth.ragged_requests(NSEQ, prompt_range=(16, 1024), output_range=(32, 256), seed=11)


def _top2_margin(logits):
    top = np.partition(logits, -2)[-2:]
    return float(abs(top[1] - top[0]) / np.std(logits))


def _run(model, reqs, dp, steps, contract=1, with_engine=True):
    """Prefill every request, then `steps` packed decode steps over all of
    them; the oracle's argmax feeds both sides.  Returns per-(step, seq)
    logits errors, greedy agreement, margins and the oracle's logits."""
    ctx = max(len(r.prompt) for r in reqs) + steps + 8
    O.set_threads(16)
    om = O.OracleModel(CFG, model, ctx, dp, dp, contract=contract, kv_fp16=True)
    states = [om.new_state() for _ in reqs]
    cur = [om.prefill(st, r.prompt) for st, r in zip(states, reqs)]
    eng = None
    if with_engine:
        eng = Engine(CFG, model, context=ctx, max_batch=64, max_seqs=len(reqs) + 1, use_dp4a=dp, use_q6_dp4a=dp)
        seqs = [eng.seq_open() for _ in reqs]
        got0 = [eng.seq_prefill(s, r.prompt) for s, r in zip(seqs, reqs)]
    errs, agree, margins, ref_logits = [], [], [], []
    for step in range(steps):
        pos = [len(r.prompt) + step for r in reqs]
        want, lg_ref = om.forward_multi(states, cur, pos, True, want_logits=True)
        ref_logits.append(lg_ref)
        margins += [_top2_margin(row) for row in lg_ref]
        if eng is not None:
            got = eng.decode_step(seqs, cur)
            lg = eng.logits(len(reqs))
            errs.append([rel_l2(lg[i], lg_ref[i]) for i in range(len(reqs))])
            agree += [int(g == w) for g, w in zip(got, want)]
        cur = [int(t) for t in want]
    if eng is not None:
        eng.close()
    return np.array(errs), np.array(agree), np.array(margins), ref_logits


def _report(tag, errs, agree, margins):
    bad = np.flatnonzero(agree == 0)
    print(f"\n{tag}: logits rel-L2 max {errs.max():.3e} mean {errs.mean():.3e}; greedy {agree.mean():.4f} "
          f"({agree.sum()}/{agree.size}); top-2 margin (sigma units) p1 {np.percentile(margins, 1):.3f} "
          f"p5 {np.percentile(margins, 5):.3f} median {np.median(margins):.3f}; margins where greedy differs: "
          f"{[round(float(margins[i]), 4) for i in bad[:10]]}")


@pytest.mark.parametrize("dp4a", [False, True], ids=["fp32-path", "int8-path"])
def test_projections_at_1b_shapes(cuda, model, dp4a):
    import torch
    eng = Engine(CFG, model, context=32, max_batch=64, use_dp4a=dp4a, use_q6_dp4a=dp4a)
    rng = np.random.default_rng(5)
    worst = {}
    for name, t, rows, cols in CFG.matrices():
        if not name.startswith("blk.0.") and name != "token_embd.weight":
            continue
        x = rng.standard_normal((64, cols)).astype(np.float32)
        y = eng.matvec(name, torch.from_numpy(x).to(cuda), 64).cpu().numpy()
        ref = O.matvec_multi(t, model[name], x, cols, rows, dp4a, dp4a)
        worst[name] = max(rel_l2(y[b], ref[b]) for b in range(64))
    eng.close()
    print("\nper-projection worst rel-L2 over 64 tokens:", {k: f"{v:.2e}" for k, v in worst.items()})
    assert max(worst.values()) <= PROJ_BAR, worst


def test_ragged64_fp32_path_vs_oracle(cuda, model, requests):
    errs, agree, margins, _ = _run(model, requests, False, STEPS)
    _report("fp32 path, 64 seqs x 32 steps", errs, agree, margins)
    assert errs.max() <= FP32_BAR, errs.max()
    assert agree.mean() >= GREEDY_BAR, agree.mean()


def test_ragged64_int8_path_vs_oracle_and_its_floor(cuda, model, requests):
    errs, agree, margins, ref_logits = _run(model, requests, True, STEPS)
    _report("int8 path, 64 seqs x 32 steps", errs, agree, margins)
    # the path's own floor: the same algorithm with one contraction changed,
    # on the first 16 sequences, same tokens
    sub = requests[:16]
    _, _, _, alt_logits = _run(model, sub, True, STEPS, contract=0, with_engine=False)
    floor = np.array([[rel_l2(alt_logits[s][i], ref_logits[s][i]) for i in range(len(sub))] for s in range(STEPS)])
    print(f"int8 floor (oracle contract 0 vs 1): max {floor.max():.3e} mean {floor.mean():.3e}")
    assert errs.max() <= 2 * floor.max(), (errs.max(), floor.max())
    assert errs.mean() <= 2 * floor.mean(), (errs.mean(), floor.mean())
    assert agree.mean() >= GREEDY_BAR, agree.mean()


def test_ragged16_fp32_path_128_steps(cuda, model, requests):
    errs, agree, margins, _ = _run(model, requests[:LONG_SEQS], False, LONG_STEPS)
    _report("fp32 path, 16 seqs x 128 steps", errs, agree, margins)
    assert errs.max() <= FP32_BAR, errs.max()
    assert agree.mean() >= GREEDY_BAR, agree.mean()
