"""The row-split lm_head (ijb200.tp over libijb200's ijb_weight_*) on one GPU:
the slices of 4 ranks computed in one process and put together as the NCCL
all-gather would, against the whole matrix as one slice and against the
oracle's FastGPU::matvec restatement (inferencer.cu:1156-1171); the next
tokens from the ranks' packed keys (max over ranks) against the argmax of the
whole row with the reference's tie rule."""
import numpy as np
import pytest

import oracle as O
from ijb200 import synth, tp

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dp4a", [True, False], ids=["int8-path", "fp32-path"])
def test_row_split_slices_match_the_whole_lm_head(cuda, dp4a):
    import torch
    vocab, cols, n, world = 128256, 3072, 80, 4
    rng = np.random.default_rng(3)
    blocks = synth.quant_matrix(rng, 14, vocab, cols, d_range=(2e-5, 4e-5))
    x = torch.from_numpy(rng.standard_normal((n, cols)).astype(np.float32)).to(cuda)
    full = tp.RowSplitLmHead(blocks, 14, vocab, cols, 0, 1)
    yf, kf = full.local(x, dp4a=dp4a)
    parts, keys = [], []
    for r in range(world):
        h = tp.RowSplitLmHead(blocks, 14, vocab, cols, r, world)
        y, k = h.local(x, dp4a=dp4a)
        parts.append(y[:, :h.rows])
        keys.append(tp.flip(k))
        h.close()
    torch.cuda.synchronize()
    logits = torch.cat(parts, dim=1)
    rel = float(torch.linalg.norm(logits - yf[:, :vocab]) / torch.linalg.norm(yf))
    assert rel < 1e-6, rel
    best = tp.flip(torch.stack(keys).max(dim=0).values)
    tokens = full.tokens_from_keys(best).cpu().numpy()
    assert np.array_equal(tokens, full.tokens_from_keys(kf).cpu().numpy())
    lg = logits.cpu().numpy()
    assert [O.argmax(row) for row in lg[:8]] == list(tokens[:8])
    O.set_threads(8)
    xs = x.cpu().numpy()
    for t in (0, 41, 79):
        ref = O.matvec(14, blocks, xs[t], cols, vocab, dp4a, dp4a)
        assert np.linalg.norm(lg[t] - ref) / np.linalg.norm(ref) < 1e-3
    full.close()


def test_layer_projection_timing_entry(cuda):
    """ijb_time_layer_projections runs the step's four projection launches of
    layer 0 and leaves the engine usable (sequence 0 empty again)."""
    import ctypes
    from ijb200 import lib
    from ijb200.engine import Engine
    cfg = synth.TINY
    w = synth.make_model(cfg, seed=2)
    eng = Engine(cfg, w, context=128, max_batch=64, max_seqs=2)
    ms = ctypes.c_float()
    lib.check(eng.lib.ijb_time_layer_projections(eng.h, 64, 3, ctypes.byref(ms)), eng.h)
    assert ms.value > 0
    prompt = synth.prompt_tokens(10, seed=1, vocab_limit=cfg.vocab)
    ref = Engine(cfg, w, context=128, max_batch=64, max_seqs=2)
    assert eng.prefill(prompt) == ref.prefill(prompt)
    assert np.array_equal(eng.logits(10), ref.logits(10))
    eng.close()
    ref.close()
