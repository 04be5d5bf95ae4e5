"""ctypes front-end of the CPU oracle (oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference leg, always as the checker or the timed
CPU baseline, never as part of the product path.  Every function mirrors the
reference routine named in oracle.c (inferencer.cu file:line citations there).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

Q4_K = 12
Q6_K = 14
F32 = 0

_lib = None


def build() -> str:
    """Compile liboracle.so with the committed Makefile (gcc only)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or (
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "oracle.c"))
        ):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        i32, i64, f32 = ctypes.c_int, ctypes.c_long, ctypes.c_float
        L.orc_dequant.argtypes = [i32, P, i64, P, i32]
        L.orc_quantize_x32.argtypes = [P, i32, P, P]
        L.orc_gemv_f32.argtypes = [i32, P, P, P, i32, i64, i32]
        L.orc_gemv_dp4a.argtypes = [i32, P, P, P, P, i32, i64, i32]
        L.orc_matvec.argtypes = [i32, P, P, P, i32, i64, i32, i32, i32]
        L.orc_rmsnorm.argtypes = [P, P, P, i32, f32, i32]
        L.orc_rope_tables.argtypes = [i32, i32, f32, P, P]
        L.orc_rope.argtypes = [P, i32, i32, i32, P, P]
        L.orc_attention.argtypes = [P, P, P, P, i32, i32, i32, i32, f32]
        L.orc_silu.argtypes = [P, P, i32]
        L.orc_argmax.argtypes = [P, i32]
        L.orc_argmax.restype = i32
        L.orc_set_threads.argtypes = [i32]
        L.orc_get_threads.restype = i32
        L.orc_half_to_float.argtypes = [ctypes.c_uint16]
        L.orc_half_to_float.restype = f32
        L.orc_model_create.argtypes = [i32, i32, i32, i32, i32, i32, i32, f32, f32, i32, i32, i32]
        L.orc_model_create.restype = P
        L.orc_model_set_global.argtypes = [P, P, P, i32, P]
        L.orc_model_set_layer.argtypes = [P, i32, P, P, P, P, P, i32, P, P, P, P, i32]
        L.orc_model_destroy.argtypes = [P]
        L.orc_model_set_kv_fp16.argtypes = [P, i32]
        L.orc_state_create.argtypes = [P]
        L.orc_state_create.restype = P
        L.orc_state_destroy.argtypes = [P]
        L.orc_state_logits.argtypes = [P]
        L.orc_state_logits.restype = ctypes.POINTER(ctypes.c_float)
        L.orc_state_residual.argtypes = [P]
        L.orc_state_residual.restype = ctypes.POINTER(ctypes.c_float)
        L.orc_state_fill_kv.argtypes = [P, i32]
        L.orc_forward.argtypes = [P, i32, i32, i32, P]
        L.orc_forward.restype = i32
        L.orc_matvec_multi.argtypes = [i32, P, P, P, i32, i64, i32, i32, i32, i32]
        L.orc_matvec_multi.restype = i32
        L.orc_forward_multi.argtypes = [P, P, P, i32, i32, P, P]
        L.orc_forward_multi.restype = i32
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def dequant(qtype: int, blocks: np.ndarray, contract: int = 0) -> np.ndarray:
    """q4_value / q6_value over every weight of the given super-blocks."""
    bpb = 144 if qtype == Q4_K else 210
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
    n = blocks.size // bpb
    out = np.empty(n * 256, dtype=np.float32)
    rc = lib().orc_dequant(qtype, _p(blocks), n, _p(out), contract)
    assert rc == 0
    return out


def quantize_x32(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    n = x.size
    xq = np.zeros(n, dtype=np.int8)
    xs = np.zeros((n + 31) // 32, dtype=np.float32)
    lib().orc_quantize_x32(_p(x), n, _p(xq), _p(xs))
    return xq, xs


def gemv_f32(qtype, w, x, cols, rows, contract=1):
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(rows, dtype=np.float32)
    assert lib().orc_gemv_f32(qtype, _p(w), _p(x), _p(y), cols, rows, contract) == 0
    return y


def gemv_dp4a(qtype, w, xq, xs, cols, rows, contract=1):
    w = np.ascontiguousarray(w, dtype=np.uint8)
    xq = np.ascontiguousarray(xq, dtype=np.int8)
    xs = np.ascontiguousarray(xs, dtype=np.float32)
    y = np.empty(rows, dtype=np.float32)
    assert lib().orc_gemv_dp4a(qtype, _p(w), _p(xq), _p(xs), _p(y), cols, rows, contract) == 0
    return y


def matvec(qtype, w, x, cols, rows, use_dp4a=True, use_q6_dp4a=True, contract=1):
    """FastGPU::matvec (inferencer.cu:1156-1171) on the CPU."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(rows, dtype=np.float32)
    rc = lib().orc_matvec(qtype, _p(w), _p(x), _p(y), cols, rows, int(use_dp4a), int(use_q6_dp4a), contract)
    assert rc == 0
    return y


def matvec_multi(qtype, w, xs, cols, rows, use_dp4a=True, use_q6_dp4a=True, contract=1):
    """matvec over each row of xs [n][cols] -> [n][rows], decoding each weight
    block once for all vectors (every output equals matvec's for its vector)."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    xs = np.ascontiguousarray(xs, dtype=np.float32).reshape(-1, cols)
    y = np.empty((xs.shape[0], rows), dtype=np.float32)
    rc = lib().orc_matvec_multi(qtype, _p(w), _p(xs), _p(y), cols, rows, xs.shape[0], int(use_dp4a),
                                int(use_q6_dp4a), contract)
    assert rc == 0
    return y


def rmsnorm(x, w, eps, contract=1):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x)
    lib().orc_rmsnorm(_p(x), _p(w), _p(out), x.size, eps, contract)
    return out


def rope_tables(ctx, head_dim, base):
    half = head_dim // 2
    c = np.empty(ctx * half, dtype=np.float32)
    s = np.empty(ctx * half, dtype=np.float32)
    lib().orc_rope_tables(ctx, head_dim, base, _p(c), _p(s))
    return c.reshape(ctx, half), s.reshape(ctx, half)


def rope(v, pos, head_dim, cos_t, sin_t):
    v = np.array(v, dtype=np.float32, copy=True)
    cos_t = np.ascontiguousarray(cos_t, dtype=np.float32)
    sin_t = np.ascontiguousarray(sin_t, dtype=np.float32)
    lib().orc_rope(_p(v), v.size // 2, pos, head_dim // 2, _p(cos_t), _p(sin_t))
    return v


def attention(q, kcache, vcache, pos, heads, kv_heads, head_dim, scale=None):
    if scale is None:
        scale = float(np.float32(1.0) / np.sqrt(np.float32(head_dim)))
    q = np.ascontiguousarray(q, dtype=np.float32)
    kcache = np.ascontiguousarray(kcache, dtype=np.float32)
    vcache = np.ascontiguousarray(vcache, dtype=np.float32)
    out = np.empty(heads * head_dim, dtype=np.float32)
    lib().orc_attention(_p(q), _p(kcache), _p(vcache), _p(out), pos, heads, kv_heads, head_dim, scale)
    return out


def silu(g, u):
    g = np.array(g, dtype=np.float32, copy=True)
    u = np.ascontiguousarray(u, dtype=np.float32)
    lib().orc_silu(_p(g), _p(u), g.size)
    return g


def argmax(values) -> int:
    v = np.ascontiguousarray(values, dtype=np.float32)
    return int(lib().orc_argmax(_p(v), v.size))


class OracleModel:
    """A Llama-shaped model over GGUF-layout host weights, run one token at a
    time exactly as FastRunner::forward (inferencer.cu:1424-1531) does, with a
    fp32 [layer][ctx][kv_dim] KV cache per sequence (inferencer.cu:1132).
    ``kv_fp16`` rounds cached K/V to binary16, the B200 build's cache format.

    ``weights`` is the dict produced by ``ijb200.synth.make_model`` (raw GGUF
    bytes per tensor name)."""

    def __init__(self, cfg, weights, context, use_dp4a=True, use_q6_dp4a=True, contract=1, kv_fp16=False):
        self.cfg = cfg
        self.w = weights  # keeps the arrays alive
        L = lib()
        self._m = L.orc_model_create(cfg.dim, cfg.layers, cfg.heads, cfg.kv_heads, cfg.hidden,
                                     cfg.vocab, context, cfg.eps, cfg.rope_base, int(use_dp4a),
                                     int(use_q6_dp4a), contract)
        L.orc_model_set_kv_fp16(self._m, int(kv_fp16))
        self._keep = []

        def P(name):
            a = np.ascontiguousarray(weights[name])
            self._keep.append(a)
            return _p(a)

        out = weights.get("output.weight")
        L.orc_model_set_global(self._m, P("token_embd.weight"),
                               P("output.weight") if out is not None else None,
                               Q6_K, P("output_norm.weight"))
        for l in range(cfg.layers):
            pre = f"blk.{l}."
            L.orc_model_set_layer(self._m, l, P(pre + "attn_norm.weight"), P(pre + "ffn_norm.weight"),
                                  P(pre + "attn_q.weight"), P(pre + "attn_k.weight"),
                                  P(pre + "attn_v.weight"), cfg.type_of("attn_v"),
                                  P(pre + "attn_output.weight"), P(pre + "ffn_gate.weight"),
                                  P(pre + "ffn_up.weight"), P(pre + "ffn_down.weight"),
                                  cfg.type_of("ffn_down"))
        self.context = context

    def new_state(self):
        return OracleState(self)

    def forward_multi(self, states, tokens, positions, need_logits=True, want_logits=False):
        """One packed step: entry i feeds tokens[i] at positions[i] to states[i]
        (entries may repeat a state at consecutive positions, in order).  Same
        per-token arithmetic as OracleState.forward, layer by layer over all
        entries.  Returns the argmax per entry (-1 without logits) and, with
        want_logits, the [n][vocab] logits."""
        n = len(states)
        arr = (ctypes.c_void_p * n)(*[s._s for s in states])
        tok = np.ascontiguousarray(tokens, dtype=np.int32)
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        nxt = np.empty(n, dtype=np.int32)
        lg = np.empty((n, self.cfg.vocab), dtype=np.float32) if (need_logits and want_logits) else None
        r = lib().orc_forward_multi(arr, _p(tok), _p(pos), n, int(need_logits),
                                    _p(lg) if lg is not None else None, _p(nxt))
        if r == -2:
            raise ValueError("Token or position outside model context")
        return (nxt, lg) if want_logits else nxt

    def prefill(self, state, tokens, start=0, chunk=64):
        """Feeds tokens at positions start.. through forward_multi in chunks;
        returns the argmax after the last token."""
        nxt = -1
        for c in range(0, len(tokens), chunk):
            part = tokens[c:c + chunk]
            last = c + len(part) == len(tokens)
            out = self.forward_multi([state] * len(part), part, np.arange(start + c, start + c + len(part)), last)
            nxt = int(out[-1])
        return nxt

    def __del__(self):
        try:
            lib().orc_model_destroy(self._m)
        except Exception:
            pass


class OracleState:
    def __init__(self, model: OracleModel):
        self.model = model
        self._s = lib().orc_state_create(model._m)

    def forward(self, token, pos, need_logits=True, trace=False):
        cfg = self.model.cfg
        tr = np.zeros((cfg.layers, cfg.dim), dtype=np.float32) if trace else None
        r = lib().orc_forward(self._s, token, pos, int(need_logits), _p(tr) if trace else None)
        if r == -2:
            raise ValueError("Token or position outside model context")
        return (r, tr) if trace else r

    def fill_kv(self, length: int) -> None:
        """Timing helper: stands in for a prefilled context of `length`."""
        lib().orc_state_fill_kv(self._s, int(length))

    def logits(self):
        v = self.model.cfg.vocab
        return np.ctypeslib.as_array(lib().orc_state_logits(self._s), shape=(v,)).copy()

    def residual(self):
        d = self.model.cfg.dim
        return np.ctypeslib.as_array(lib().orc_state_residual(self._s), shape=(d,)).copy()

    def __del__(self):
        try:
            lib().orc_state_destroy(self._s)
        except Exception:
            pass
