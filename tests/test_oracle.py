"""The CPU oracle pinned against the reference: golden vectors captured from
the reference's own kernels on a B200 (tests/golden/ref_kernels.npz) and the
independent gguf package dequantiser."""
import os

import numpy as np
import pytest

import oracle as O
from ijb200 import synth


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("name,qtype", [("q4_edge", 12), ("q6_edge", 14), ("q4_rand", 12), ("q6_rand", 14)])
def test_dequant_bit_exact_vs_reference(golden, golden_inputs, name, qtype):
    for contract in (0, 1):
        got = O.dequant(qtype, golden_inputs[name], contract)
        np.testing.assert_array_equal(bits(got), bits(golden["ref_dequant_" + name]))


def test_dequant_bit_exact_vs_gguf():
    gguf = pytest.importorskip("gguf")
    from gguf import quants, GGMLQuantizationType as T
    rng = np.random.default_rng(5)
    for qtype, gt, blocks in ((12, T.Q4_K, synth.q4k_blocks(rng, 128)), (14, T.Q6_K, synth.q6k_blocks(rng, 128))):
        ref = quants.dequantize(blocks.reshape(-1), gt).reshape(-1).astype(np.float32)
        np.testing.assert_array_equal(bits(O.dequant(qtype, blocks)), bits(ref))


@pytest.mark.parametrize("xname", ["x2048", "x8192"])
def test_quantize_bit_exact_vs_reference(golden, golden_inputs, xname):
    xq, xs = O.quantize_x32(golden_inputs[xname])
    np.testing.assert_array_equal(xq, golden["ref_xq_" + xname])
    np.testing.assert_array_equal(bits(xs), bits(golden["ref_xscale_" + xname]))
    assert xs[0] == 1.0 if xname == "x8192" else True  # an all-zero group keeps scale 1


@pytest.mark.parametrize("wname,qtype,cols,rows,xname", [
    ("w4", 12, 2048, 64, "x2048"), ("w6", 14, 2048, 64, "x2048"), ("w6k8192", 14, 8192, 16, "x8192")])
def test_gemv_bit_exact_vs_reference(golden, golden_inputs, wname, qtype, cols, rows, xname):
    """With the reference build's multiply-add contractions (contract=1) the
    oracle reproduces FastGPU::matvec bit for bit in both activation paths."""
    w, x = golden_inputs[wname], golden_inputs[xname]
    xq, xs = O.quantize_x32(x)
    np.testing.assert_array_equal(bits(O.gemv_dp4a(qtype, w, xq, xs, cols, rows, 1)),
                                  bits(golden[f"ref_matvec_{wname}_dp4a"]))
    np.testing.assert_array_equal(bits(O.gemv_f32(qtype, w, x, cols, rows, 1)),
                                  bits(golden[f"ref_matvec_{wname}_f32"]))
    # the un-contracted restatement stays within float rounding of it
    ref = golden[f"ref_matvec_{wname}_f32"]
    got = O.gemv_f32(qtype, w, x, cols, rows, 0)
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-6


@pytest.mark.parametrize("n", [2048, 3072])
def test_rmsnorm_vs_reference(golden, golden_inputs, n):
    """rsqrtf is not reproduced on the CPU (1/sqrtf is used): outputs agree to
    a couple of ulp of the shared scale."""
    got = O.rmsnorm(golden_inputs["norm_x"][:n], golden_inputs["norm_w"][:n], 1e-5)
    ref = golden[f"ref_rmsnorm_{n}"]
    np.testing.assert_allclose(got, ref, rtol=3e-7, atol=0)


@pytest.mark.parametrize("pos", [0, 37, 63])
def test_attention_vs_reference(golden, golden_inputs, pos):
    d = golden_inputs
    got = O.attention(d["att_q"], d["att_k"].reshape(64, 1024), d["att_v"].reshape(64, 1024), pos, 24, 8, 128)
    ref = golden[f"ref_attention_pos{pos}"]
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-6


@pytest.mark.parametrize("name", ["argmax_rand", "argmax_tie", "argmax_flat"])
def test_argmax_vs_reference(golden, golden_inputs, name):
    assert O.argmax(golden_inputs[name]) == int(golden["ref_" + name][0])


def _tournament(v):
    """Python statement of argmax_blocks_cuda + argmax_final_cuda's trees."""
    n = len(v)
    nb = (n + 255) // 256
    bv, bi = [], []
    for b in range(nb):
        vals = [v[b * 256 + l] if b * 256 + l < n else -np.inf for l in range(256)]
        idx = [b * 256 + l for l in range(256)]
        s = 128
        while s:
            for l in range(s):
                if vals[l + s] > vals[l]:
                    vals[l], idx[l] = vals[l + s], idx[l + s]
            s //= 2
        bv.append(vals[0]); bi.append(idx[0])
    bv += [-np.inf] * (512 - nb); bi += [2**31 - 1] * (512 - nb)
    s = 256
    while s:
        for i in range(s):
            if bv[i + s] > bv[i]:
                bv[i], bi[i] = bv[i + s], bi[i + s]
        s //= 2
    return bi[0]


def _bitrev_rule(v):
    m = np.max(v)
    cand = np.nonzero(v == m)[0]
    key = lambda j: (int(f"{j >> 8:09b}"[::-1], 2), int(f"{j & 255:08b}"[::-1], 2))
    return int(min(cand, key=key))


@pytest.mark.parametrize("ties", [[3, 5], [256 + 7, 512 + 7], [3, 5, 256, 512], [1000, 2000, 3000, 4000],
                                  [255, 254, 128], list(range(0, 4096, 17))])
def test_argmax_tie_rule(ties):
    v = np.random.default_rng(len(ties)).standard_normal(4096).astype(np.float32)
    v[ties] = 9.0
    assert O.argmax(v) == _tournament(list(v)) == _bitrev_rule(v)


def test_rope_tables_match_float_formula():
    c, s = O.rope_tables(64, 64, 500000.0)
    freq = np.power(np.float32(500000.0), (np.float32(-2.0) * np.arange(32, dtype=np.float32)) / np.float32(64))
    ang = (np.arange(64, dtype=np.float32)[:, None] * freq[None, :]).astype(np.float32)
    # numpy's float32 pow/cos differ from libm's powf/cosf by a few ulp of
    # angles up to ~64 rad
    np.testing.assert_allclose(c, np.cos(ang), atol=2e-5)
    np.testing.assert_allclose(s, np.sin(ang), atol=2e-5)


def test_model_activation_range():
    """Random-init weights keep activations, K and V well inside fp16 range."""
    cfg = synth.TINY
    m = O.OracleModel(cfg, synth.make_model(cfg, 0), 64)
    st = m.new_state()
    for i, t in enumerate(synth.prompt_tokens(24, 1, cfg.vocab)):
        _, tr = st.forward(int(t), i, True, trace=True)
        assert np.abs(tr).max() < 1e3
    lg = st.logits()
    assert np.isfinite(lg).all() and 0.5 < lg.std() < 50


def test_oracle_threads_deterministic():
    rng = np.random.default_rng(3)
    w = synth.quant_matrix(rng, 12, 512, 2048)
    x = rng.standard_normal(2048).astype(np.float32)
    O.set_threads(1)
    a = O.matvec(12, w, x, 2048, 512)
    O.set_threads(4)
    b = O.matvec(12, w, x, 2048, 512)
    O.set_threads(1)
    np.testing.assert_array_equal(a, b)


def test_forward_rejects_bad_position():
    cfg = synth.TINY
    m = O.OracleModel(cfg, synth.make_model(cfg, 0), 16)
    st = m.new_state()
    with pytest.raises(ValueError):
        st.forward(0, 16)
    with pytest.raises(ValueError):
        st.forward(cfg.vocab, 0)


def test_dp4a_path_noise_floor():
    """The reference's INT8 path is sensitive to ulp-level changes: two oracle
    variants that differ only in multiply-add contraction give logits ~1%
    apart (same greedy tokens), while the FP32 path stays within 1e-4.  This
    floor sets the DP4A-mode full-model bar of the GPU tests."""
    cfg = synth.TINY_HD128
    w = synth.make_model(cfg, 11)
    prompt = synth.prompt_tokens(40, 1, cfg.vocab)
    for dp4a, lo, hi in ((True, 3e-3, 2e-2), (False, 0.0, 1e-4)):
        a = O.OracleModel(cfg, w, 64, dp4a, dp4a, contract=1).new_state()
        b = O.OracleModel(cfg, w, 64, dp4a, dp4a, contract=0).new_state()
        for i, t in enumerate(prompt):
            ta = a.forward(int(t), i, True)
            tb = b.forward(int(t), i, True)
        la, lb = a.logits(), b.logits()
        err = np.linalg.norm(la - lb) / np.linalg.norm(la)
        assert lo <= err < hi, (dp4a, err)
        assert ta == tb


def _reference_trees(values):
    """argmax_blocks_cuda + argmax_final_cuda (inferencer.cu:1063-1099) in Python:
    256-wide blocks, then one 512-wide pass, each a halving tree where a slot
    takes its partner only if the partner is strictly greater."""
    v = np.asarray(values, np.float32)
    n = v.size
    blocks = (n + 255) // 256
    bv, bi = [], []
    for b in range(blocks):
        vals = [float(v[b * 256 + l]) if b * 256 + l < n else -np.inf for l in range(256)]
        idx = [b * 256 + l for l in range(256)]
        stride = 128
        while stride:
            for l in range(stride):
                if vals[l + stride] > vals[l]:
                    vals[l], idx[l] = vals[l + stride], idx[l + stride]
            stride //= 2
        bv.append(vals[0]); bi.append(idx[0])
    bv += [-np.inf] * (512 - blocks); bi += [2 ** 31 - 1] * (512 - blocks)
    stride = 256
    while stride:
        for i in range(stride):
            if bv[i + stride] > bv[i]:
                bv[i], bi[i] = bv[i + stride], bi[i + stride]
        stride //= 2
    return bi[0]


@pytest.mark.parametrize("nan_at", [[0], [3], [700], [0, 2500], [256, 300], [131]])
def test_oracle_argmax_nan_semantics_follow_the_reference_trees(nan_at):
    """With NaN inputs the reference's trees neither skip NaN nor let it win
    everywhere: a NaN in a left slot stays there and hides the partner subtree.
    The oracle reproduces that exactly (the GPU argmax does not: there NaN never
    wins)."""
    v = np.random.default_rng(len(nan_at)).standard_normal(3000).astype(np.float32)
    v[nan_at] = np.nan
    assert O.argmax(v) == _reference_trees(v)


@pytest.mark.parametrize("dp4a", [True, False], ids=["int8", "fp32"])
@pytest.mark.parametrize("contract", [1, 0])
def test_packed_forward_is_bit_identical_to_token_by_token(dp4a, contract):
    """orc_forward_multi (layer by layer over many entries, weights decoded once
    per block for all of them) gives exactly orc_forward's results: chunked
    prefills of several sequences, then packed decode steps over all of them."""
    cfg = synth.TINY
    w = synth.make_model(cfg, seed=4)
    O.set_threads(4)
    m = O.OracleModel(cfg, w, 128, dp4a, dp4a, contract=contract, kv_fp16=True)
    reqs = synth.ragged_requests(5, prompt_range=(3, 40), output_range=(4, 8), seed=2, vocab_limit=cfg.vocab)
    a = [m.new_state() for _ in reqs]
    b = [m.new_state() for _ in reqs]
    na, nb = [], []
    for sa, sb, r in zip(a, b, reqs):
        for i, t in enumerate(r.prompt):
            x = sa.forward(int(t), i, i + 1 == len(r.prompt))
        na.append(x)
        nb.append(m.prefill(sb, r.prompt, chunk=7))
    assert na == nb
    cur = na
    for step in range(4):
        want = [sa.forward(int(t), len(r.prompt) + step, True) for sa, t, r in zip(a, cur, reqs)]
        la = np.stack([s.logits() for s in a])
        got, lb = m.forward_multi(b, cur, [len(r.prompt) + step for r in reqs], True, want_logits=True)
        assert list(got) == want
        assert np.array_equal(la, lb)
        cur = want


@pytest.mark.parametrize("qt,rows,cols", [(12, 300, 512), (14, 200, 1024)])
def test_multi_vector_matvec_equals_matvec(qt, rows, cols):
    rng = np.random.default_rng(0)
    W = synth.quant_matrix(rng, qt, rows, cols)
    xs = rng.standard_normal((9, cols)).astype(np.float32)
    for dp in (True, False):
        for c in (0, 1):
            y = O.matvec_multi(qt, W, xs, cols, rows, dp, dp, c)
            for i in range(9):
                assert np.array_equal(y[i], O.matvec(qt, W, xs[i], cols, rows, dp, dp, c))


RUNNER_GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_runner_3b.npz")


@pytest.fixture(scope="module")
def runner_golden():
    if not os.path.exists(RUNNER_GOLDEN):
        pytest.skip("tests/golden/ref_runner_3b.npz not captured yet (make_ref_runner_golden.py)")
    import make_ref_runner_golden as G
    g = dict(np.load(RUNNER_GOLDEN))
    return g, G, synth.make_model(synth.LLAMA_3B, seed=int(g["seed"]))


def _sample_rel(logits, g, tag):
    rows = g["sample_rows"]
    a = logits[:, rows].astype(np.float64)
    b = g[f"{tag}_sample"].astype(np.float64)
    return np.linalg.norm(a - b, axis=1) / np.linalg.norm(b, axis=1)


@pytest.mark.parametrize("tag,dp4a", [("fp32", False), ("int8", True)])
def test_oracle_full_model_matches_the_reference_runner(runner_golden, tag, dp4a):
    """The oracle's whole layer sequence (embedding, 28 layers of norm / QKV /
    RoPE / cache / attention / O / residual / norm / gate-up / SiLU / down /
    residual, output norm, tied Q6_K lm_head, argmax) against the reference's
    own GGUF + FastRunner::forward (inferencer.cu:1424-1531) run on a B200 on
    the same seeded 3B-shape model and tokens (tests/golden/ref_runner_3b.npz).
    FP32 path: the GEMVs are bit-exact and only rsqrtf / __expf differ from
    the oracle's 1/sqrtf / expf, so the logits agree to ~1e-5.  INT8 path:
    those ulp differences flip int8 codes, so the bar is twice the path's own
    floor (the oracle against itself with one contraction changed)."""
    g, G, weights = runner_golden
    toks = g["tokens"]
    O.set_threads(8)

    def run(contract):
        m = O.OracleModel(synth.LLAMA_3B, weights, G.CONTEXT, dp4a, dp4a, contract=contract)
        st = m.new_state()
        nxt, lg = m.forward_multi([st] * len(toks), toks, np.arange(len(toks)), True, want_logits=True)
        return nxt, lg

    nxt, lg = run(1)
    rel = _sample_rel(lg, g, tag)
    agree = float(np.mean(nxt == g[f"{tag}_next"]))
    top_match = float(np.mean(np.take_along_axis(lg, g[f"{tag}_top_idx"], axis=1)[:, 0] == g[f"{tag}_top_val"][:, 0]))
    print(f"\n{tag}: sampled logits rel-L2 max {rel.max():.3e} mean {rel.mean():.3e}; argmax agreement {agree:.3f}; "
          f"top-1 value equal {top_match:.3f}")
    if not dp4a:
        assert rel.max() < 1e-4, rel
        assert agree == 1.0
    else:
        _, lg_alt = run(0)
        floor = np.linalg.norm((lg_alt - lg)[:, g["sample_rows"]], axis=1) / np.linalg.norm(lg[:, g["sample_rows"]],
                                                                                              axis=1)
        print(f"int8 floor max {floor.max():.3e} mean {floor.mean():.3e}")
        assert rel.max() <= 2 * max(floor.max(), 1e-6), (rel.max(), floor.max())
        assert agree >= 0.95
