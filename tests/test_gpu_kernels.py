"""Kernel parity on a B200: the CUDA library against the CPU oracle and the
golden outputs of the reference's own kernels.

Tolerances: dequantisation, int8 activations, argmax and the Q6_K repack are
bit-exact.  GEMVs compute the same integer DP4A dot products as the reference
(or the same fp32 products) in a different summation order, so they are
checked at rel-L2 <= 1e-5; the project bar (per-projection rel-L2 <= 1e-3) is
far looser."""
import ctypes

import numpy as np
import pytest

import oracle as O
from ijb200 import lib, synth

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = np.asarray(a, np.float64); b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _gemv(dev, qtype, w_raw, x, cols, rows, batch, dp4a):
    import torch
    L = lib.load()
    w = _t(w_raw, dev)
    if qtype == 14:
        rb = L.ijb_q6k_planar_row_bytes(cols)
        wp = torch.empty(rows * rb, dtype=torch.uint8, device=dev)
        lib.check(L.ijb_repack_q6k(w.data_ptr(), wp.data_ptr(), rows, cols, None))
        w = wp
    xt = _t(x.reshape(batch, cols), dev)
    y = torch.empty((batch, rows), dtype=torch.float32, device=dev)
    lib.check(L.ijb_gemv(qtype, w.data_ptr(), xt.data_ptr(), y.data_ptr(), cols, rows, batch, int(dp4a), None))
    torch.cuda.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("name,qtype", [("q4_edge", 12), ("q6_edge", 14), ("q4_rand", 12), ("q6_rand", 14)])
def test_dequant_bit_exact(cuda, golden, golden_inputs, name, qtype):
    import torch
    blocks = golden_inputs[name]
    b = _t(blocks, cuda)
    out = torch.empty(blocks.shape[0] * 256, dtype=torch.float32, device=cuda)
    lib.check(lib.load().ijb_dequant(qtype, b.data_ptr(), blocks.shape[0], out.data_ptr(), None))
    got = out.cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), golden["ref_dequant_" + name].view(np.uint32))


@pytest.mark.parametrize("wname,qtype,cols,rows,xname", [
    ("w4", 12, 2048, 64, "x2048"), ("w6", 14, 2048, 64, "x2048"), ("w6k8192", 14, 8192, 16, "x8192")])
@pytest.mark.parametrize("dp4a", [1, 0])
def test_gemv_vs_reference_golden(cuda, golden, golden_inputs, wname, qtype, cols, rows, xname, dp4a):
    y = _gemv(cuda, qtype, golden_inputs[wname], golden_inputs[xname], cols, rows, 1, dp4a)[0]
    ref = golden[f"ref_matvec_{wname}_{'dp4a' if dp4a else 'f32'}"]
    assert rel_l2(y, ref) < 1e-5


@pytest.mark.parametrize("qtype,cols,rows", [(12, 2048, 8192), (14, 2048, 4096), (14, 8192, 512),
                                             (12, 3072, 256), (14, 3072, 256), (12, 8192, 64),
                                             (12, 256, 100), (14, 256, 37), (14, 4352, 33), (12, 1280, 7)])
@pytest.mark.parametrize("batch", [1, 2, 3, 8])
@pytest.mark.parametrize("dp4a", [1, 0])
def test_gemv_vs_oracle(cuda, qtype, cols, rows, batch, dp4a):
    rng = np.random.default_rng(cols + rows + batch)
    w = synth.quant_matrix(rng, qtype, rows, cols)
    x = rng.standard_normal((batch, cols)).astype(np.float32)
    got = _gemv(cuda, qtype, w, x, cols, rows, batch, dp4a)
    for b in range(batch):
        ref = O.matvec(qtype, w, x[b], cols, rows, bool(dp4a), bool(dp4a))
        assert rel_l2(got[b], ref) < 1e-5, (b, rel_l2(got[b], ref))


def test_gemv_baseline_config0_full_size(cuda):
    """ffn_gate 8192 x 2048 Q4_K, d/dmin ~ U[1e-3, 1e-2],
    x ~ N(0,1), seed 0, batch 1, against the reference's math on the CPU."""
    rng = np.random.default_rng(0)
    w = synth.quant_matrix(rng, 12, 8192, 2048)
    x = rng.standard_normal(2048).astype(np.float32)
    for dp4a in (1, 0):
        got = _gemv(cuda, 12, w, x, 2048, 8192, 1, dp4a)[0]
        ref = O.matvec(12, w, x, 2048, 8192, bool(dp4a), bool(dp4a))
        assert rel_l2(got, ref) < 1e-5
        if not dp4a:  # the FP32 path also meets the project bar against fp64 truth
            W = O.dequant(12, w).reshape(8192, 2048).astype(np.float64)
            assert rel_l2(got, W @ x.astype(np.float64)) < 1e-3


def q6_unit_layout(row_blocks: np.ndarray) -> np.ndarray:
    """numpy statement of the Q6_K unit layout (gemv.cuh): per unit of up to
    8 blocks, 208-byte block bodies (lane-major), then the blocks' d."""
    nb = row_blocks.shape[0]
    out = []
    for u0 in range(0, nb, 8):
        ub = row_blocks[u0:u0 + 8]
        n = ub.shape[0]
        unit = np.zeros(((n * 210 + 15) // 16) * 16, dtype=np.uint8)
        for blk in range(n):
            b = ub[blk]
            body = unit[blk * 208:(blk + 1) * 208]
            for g in range(2):
                for h in range(2):
                    j = 2 * g + h
                    body[j * 16:(j + 1) * 16] = b[g * 64 + 16 * h:g * 64 + 16 * h + 16]
                    body[64 + j * 16:64 + (j + 1) * 16] = b[g * 64 + 32 + 16 * h:g * 64 + 48 + 16 * h]
                    body[128 + j * 16:128 + (j + 1) * 16] = b[128 + g * 32 + 16 * h:128 + g * 32 + 16 * h + 16]
                    for part in range(4):
                        body[192 + j * 4 + part] = b[192 + g * 8 + 2 * part + h]
            unit[n * 208 + blk * 2:n * 208 + blk * 2 + 2] = b[208:210]
        out.append(unit)
    return np.concatenate(out)


def test_repack_round_trip(cuda):
    """The Q6_K repack moves bytes into the unit layout exactly."""
    import torch
    rng = np.random.default_rng(9)
    for cols in (2048, 3072, 8192, 4352):
        w = synth.quant_matrix(rng, 14, 8, cols)
        L = lib.load()
        rb = L.ijb_q6k_planar_row_bytes(cols)
        wp = torch.empty(8 * rb, dtype=torch.uint8, device=cuda)
        lib.check(L.ijb_repack_q6k(_t(w, cuda).data_ptr(), wp.data_ptr(), 8, cols, None))
        got = wp.cpu().numpy().reshape(8, rb)
        for r in range(8):
            np.testing.assert_array_equal(got[r], q6_unit_layout(w[r].reshape(cols // 256, 210)))


@pytest.mark.parametrize("name", ["argmax_rand", "argmax_tie", "argmax_flat"])
def test_argmax_vs_reference(cuda, golden, golden_inputs, name):
    import torch
    v = _t(golden_inputs[name], cuda)
    idx = torch.zeros(1, dtype=torch.int32, device=cuda)
    lib.check(lib.load().ijb_argmax(v.data_ptr(), v.numel(), idx.data_ptr(), None))
    assert int(idx.item()) == int(golden["ref_" + name][0])


@pytest.mark.parametrize("ties", [[3, 5], [256 + 7, 512 + 7], [3, 5, 256, 512], [255, 254, 128],
                                  list(range(0, 128256, 997))])
def test_argmax_tie_rule(cuda, ties):
    import torch
    v = np.random.default_rng(len(ties)).standard_normal(128256).astype(np.float32)
    v[ties] = 9.0
    vt = _t(v, cuda)
    idx = torch.zeros(1, dtype=torch.int32, device=cuda)
    lib.check(lib.load().ijb_argmax(vt.data_ptr(), v.size, idx.data_ptr(), None))
    assert int(idx.item()) == O.argmax(v)


@pytest.mark.parametrize("dp4a", [1, 0])
def test_gemv_pdl_chain_reads_previous_output(cuda, dp4a):
    """IJB_GEMV_PDL: a chain y1 = W1 x, y2 = W2 y1, y3 = W1 y2 ... launched with
    programmatic dependent launch on one stream, each GEMV reading the output
    of the one before, matches the same chain launched without PDL (bit for
    bit) and the oracle."""
    import torch
    L = lib.load()
    rng = np.random.default_rng(21)
    n = 2048
    w1 = synth.quant_matrix(rng, 12, n, n)
    w2 = synth.quant_matrix(rng, 12, n, n)
    d1, d2 = _t(w1, cuda), _t(w2, cuda)
    x = rng.standard_normal(n).astype(np.float32)
    outs = {}
    for flags in (dp4a, dp4a | lib.GEMV_PDL):
        bufs = [_t(x[None, :], cuda)] + [torch.empty((1, n), dtype=torch.float32, device=cuda) for _ in range(6)]
        s = torch.cuda.current_stream().cuda_stream
        for i in range(6):
            w = d1 if i % 2 == 0 else d2
            lib.check(L.ijb_gemv(12, w.data_ptr(), bufs[i].data_ptr(), bufs[i + 1].data_ptr(), n, n, 1, flags,
                                 ctypes.c_void_p(s)))
        torch.cuda.synchronize()
        outs[flags] = [b.cpu().numpy()[0] for b in bufs[1:]]
    for a, b in zip(outs[dp4a], outs[dp4a | lib.GEMV_PDL]):
        np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
    prev = x
    for i in range(6):  # each link against the oracle on the GPU's own input to it
        ref = O.matvec(12, w1 if i % 2 == 0 else w2, prev, n, n, bool(dp4a), bool(dp4a))
        assert rel_l2(outs[dp4a][i], ref) < 1e-5, i
        prev = outs[dp4a][i]
