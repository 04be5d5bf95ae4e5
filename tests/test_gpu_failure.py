"""Failure paths on a B200 that fault nothing: a bounded device wait that
expires, and NaN inputs to the greedy argmax.

* Every device-side wait in the library is bounded; on expiry the kernel
  records an error code in the engine's status word and returns, and the call
  fails with IJB_ERR_DEVICE (the reference has no device waits; its errors
  surface through cuda_check, inferencer.cu:126-128).  ijb_probe_wait_timeout
  runs one kernel whose wait on a barrier that nothing signals expires after
  1 ms; the engine must report the error, clear it, and decode correctly
  afterwards.
* NaN in the argmax: a NaN never wins against a number, and an all-NaN input
  gives index 0 (what the reference's trees, argmax_blocks_cuda +
  argmax_final_cuda, inferencer.cu:1063-1099, return for it).  Checked for
  ijb_argmax, ijb_argmax_noalloc and the logits epilogues of both projection
  paths (CUDA-core GEMV and tensor-core GEMM)."""
import numpy as np
import pytest

from ijb200 import lib, synth
from ijb200.engine import Engine

pytestmark = pytest.mark.gpu


def _decode(eng, prompt, steps):
    toks, logits = [], []
    t = eng.prefill(prompt)
    for s in range(steps):
        t = eng.forward(int(t), len(prompt) + s, True)
        toks.append(t)
        logits.append(eng.logits(1)[0].copy())
    return toks, np.stack(logits)


def test_expired_wait_reports_device_error_and_engine_recovers(cuda):
    cfg = synth.TINY
    weights = synth.make_model(cfg, seed=11)
    prompt = synth.prompt_tokens(20, seed=1, vocab_limit=cfg.vocab)
    ref = Engine(cfg, weights, context=64, max_batch=1, max_seqs=2)
    want_toks, want_logits = _decode(ref, prompt, 6)
    ref.close()

    eng = Engine(cfg, weights, context=64, max_batch=1, max_seqs=2)
    eng.prefill(prompt[:5])
    rc = eng.probe_wait_timeout(1_000_000)  # 1 ms
    assert rc == lib.ERR_DEVICE, rc
    assert "bounded wait expired" in eng.last_error()
    assert eng.probe_wait_timeout(1_000_000) == lib.ERR_DEVICE  # reported again, not stuck
    got_toks, got_logits = _decode(eng, prompt, 6)  # the next steps run normally
    eng.close()
    assert got_toks == want_toks
    assert np.array_equal(got_logits, want_logits)


def test_probe_rejects_limits_outside_its_range(cuda):
    cfg = synth.TINY
    eng = Engine(cfg, synth.make_model(cfg, seed=1), context=32, max_batch=1, max_seqs=2)
    assert eng.probe_wait_timeout(10) == lib.ERR_INVALID
    assert eng.probe_wait_timeout(10 ** 10) == lib.ERR_INVALID
    eng.close()


def _argmax_both(v):
    import torch
    L = lib.load()
    t = torch.from_numpy(np.ascontiguousarray(v, np.float32)).cuda()
    out = torch.full((2,), -7, dtype=torch.int32, device="cuda")
    lib.check(L.ijb_argmax(t.data_ptr(), t.numel(), out[0:].data_ptr(), None))
    lib.check(L.ijb_argmax_noalloc(t.data_ptr(), t.numel(), out[1:].data_ptr(), None))
    torch.cuda.synchronize()
    return [int(i) for i in out.tolist()]


@pytest.mark.parametrize("n", [1, 300, 128256])
def test_argmax_all_nan_gives_index_zero(cuda, n):
    assert _argmax_both(np.full(n, np.nan, np.float32)) == [0, 0]


@pytest.mark.parametrize("nan_at", [[0], [5], [0, 1, 2, 700], list(range(0, 5000, 3))])
def test_argmax_nan_never_beats_a_number(cuda, nan_at):
    v = np.random.default_rng(len(nan_at)).standard_normal(5000).astype(np.float32)
    v[nan_at] = np.nan
    want = int(np.nanargmax(v))
    assert _argmax_both(v) == [want, want]
    v[[17, 4000]] = np.float32(-np.inf)
    assert _argmax_both(v) == [want, want]


@pytest.mark.parametrize("max_batch,n", [(1, 1), (64, 20)], ids=["gemv-epilogue", "tensor-core-epilogue"])
def test_logits_epilogue_skips_nan_rows(cuda, max_batch, n):
    """An untied lm_head whose Q6_K scale d is NaN in some rows gives NaN
    logits there; the step's argmax is the largest non-NaN logit."""
    cfg = synth.TINY
    weights = synth.make_model(cfg, seed=7)
    out = weights["token_embd.weight"].copy()
    rng = np.random.default_rng(3)
    nan_rows = rng.choice(cfg.vocab, size=300, replace=False)
    nb = cfg.dim // 256
    for r in nan_rows:
        for b in range(nb):
            out[r, b * 210 + 208:b * 210 + 210] = [0x00, 0x7E]  # fp16 NaN
    weights["output.weight"] = out
    eng = Engine(cfg, weights, context=64, max_batch=max_batch, max_seqs=n + 1)
    seqs = [eng.seq_open() for _ in range(n)]
    prompts = [synth.prompt_tokens(4 + i, seed=i, vocab_limit=cfg.vocab) for i in range(n)]
    cur = [eng.seq_prefill(s, p) for s, p in zip(seqs, prompts)]
    for _ in range(3):
        cur = eng.decode_step(seqs, cur)
        lg = eng.logits(n)
        assert np.isnan(lg[:, nan_rows]).all()
        assert [int(np.nanargmax(row)) for row in lg] == [int(c) for c in cur]
    eng.close()
