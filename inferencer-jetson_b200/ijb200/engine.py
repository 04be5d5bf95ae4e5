"""Python mirror of the reference's runner interface over the C ABI.

``Engine`` offers the methods FastRunner exposes (forward, prefill, reset and
the logits / residual buffers, inferencer.cu:1182-1532) plus the ragged
continuous-batching calls (seq_open, decode_step, ...).  Weights are uploaded
with torch (device memory only) and handed to ``ijb_create`` as GGUF tensor
views; everything after that runs in libijb200.so.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import lib as _L
from .synth import F32, ModelConfig


def _cudart():
    import torch  # noqa: F401  (loads the CUDA runtime the process uses)
    return ctypes.CDLL("libcudart.so.12")


def copy_d2h(dst: np.ndarray, src_ptr: int) -> np.ndarray:
    rt = _cudart()
    rc = rt.cudaMemcpy(ctypes.c_void_p(dst.ctypes.data), ctypes.c_void_p(src_ptr), ctypes.c_size_t(dst.nbytes),
                       ctypes.c_int(2))
    if rc != 0:
        raise RuntimeError(f"cudaMemcpy D2H failed ({rc})")
    return dst


class Engine:
    def __init__(self, cfg: ModelConfig, weights: dict, context: int = 1024, max_batch: int = 1,
                 max_seqs: int = 2, use_dp4a: bool = True, use_q6_dp4a: bool = True, device: int = 0,
                 num_pages: int = 0, page_size: int = 16, kv_f32: bool = False):
        import torch
        self.lib = _L.load()
        self.cfg = cfg
        self.device = device
        self._keep = []
        shapes = {name: (t, rows, cols) for name, t, rows, cols in cfg.matrices()}
        views = (_L.TensorView * len(weights))()
        for i, (name, arr) in enumerate(weights.items()):
            t = torch.from_numpy(np.ascontiguousarray(arr)).to(f"cuda:{device}")
            self._keep.append(t)
            v = views[i]
            v.name = name.encode()
            v.data_dev = t.data_ptr()
            if name == "output.weight" and name not in shapes:
                # an untied lm_head: [vocab][row_bytes] Q4_K or Q6_K blocks
                per_block = arr.shape[1] // (cfg.dim // 256)
                v.type, v.n_dims = {144: 12, 210: 14}[per_block], 2
                v.dims[0], v.dims[1] = cfg.dim, cfg.vocab
            elif name in shapes:
                qt, rows, cols = shapes[name]
                v.type, v.n_dims = qt, 2
                v.dims[0], v.dims[1] = cols, rows
            else:
                v.type, v.n_dims = F32, 1
                v.dims[0] = arr.size
        d = _L.ModelDesc(dim=cfg.dim, layers=cfg.layers, heads=cfg.heads, kv_heads=cfg.kv_heads,
                         hidden=cfg.hidden, vocab=cfg.vocab, eps=cfg.eps, rope_base=cfg.rope_base,
                         context=context, max_batch=max_batch, max_seqs=max_seqs, page_size=page_size,
                         num_pages=num_pages, use_dp4a=int(use_dp4a), use_q6_dp4a=int(use_q6_dp4a),
                         kv_f32=int(kv_f32), device=device)
        h = ctypes.c_void_p()
        rc = self.lib.ijb_create(ctypes.byref(d), views, len(weights), ctypes.byref(h))
        _L.check(rc, None)
        self.h = h
        self.context = context
        self.max_batch = max_batch

    # ---- FastRunner surface
    def forward(self, token: int, pos: int, need_logits: bool = True) -> int:
        nxt = ctypes.c_int(-1)
        _L.check(self.lib.ijb_forward(self.h, int(token), int(pos), int(need_logits), ctypes.byref(nxt)), self.h)
        return nxt.value

    def prefill(self, tokens) -> int:
        arr = (ctypes.c_int * len(tokens))(*[int(t) for t in tokens])
        nxt = ctypes.c_int(-1)
        _L.check(self.lib.ijb_prefill(self.h, arr, len(tokens), ctypes.byref(nxt)), self.h)
        return nxt.value

    def forward_traced(self, token: int, pos: int, need_logits: bool = True):
        """FastRunner::forward with its traces: (next, layer_trace [layers][dim],
        quant_trace [layers][3*dim + hidden] int8)."""
        c = self.cfg
        lt = np.zeros((c.layers, c.dim), np.float32)
        qt = np.zeros((c.layers, 3 * c.dim + c.hidden), np.int8)
        nxt = ctypes.c_int(-1)
        _L.check(self.lib.ijb_forward_traced(self.h, int(token), int(pos), int(need_logits), ctypes.byref(nxt),
                                             lt.ctypes.data, qt.ctypes.data), self.h)
        return nxt.value, lt, qt

    def prefill_traced(self, tokens):
        """FastRunner::prefill with its traces: (next, all_layer_trace
        [n][layers][dim], first_quant_trace, last_quant_trace)."""
        c = self.cfg
        n = len(tokens)
        arr = (ctypes.c_int * n)(*[int(t) for t in tokens])
        allt = np.zeros((n, c.layers, c.dim), np.float32)
        fq = np.zeros((c.layers, 3 * c.dim + c.hidden), np.int8)
        lq = np.zeros_like(fq)
        nxt = ctypes.c_int(-1)
        _L.check(self.lib.ijb_prefill_traced(self.h, arr, n, ctypes.byref(nxt), allt.ctypes.data, fq.ctypes.data,
                                             lq.ctypes.data), self.h)
        return nxt.value, allt, fq, lq

    def reset(self) -> None:
        _L.check(self.lib.ijb_reset(self.h), self.h)

    def logits(self, n: int = 1) -> np.ndarray:
        out = np.empty((n, self.cfg.vocab), dtype=np.float32)
        return copy_d2h(out, self.lib.ijb_logits_dev(self.h))

    def residual(self, n: int = 1) -> np.ndarray:
        out = np.empty((n, self.cfg.dim), dtype=np.float32)
        return copy_d2h(out, self.lib.ijb_residual_dev(self.h))

    def tensor_index(self, name: str) -> int:
        return self.lib.ijb_tensor_index(self.h, name.encode())

    def matvec(self, name: str, x, batch: int = 1):
        """FastGPU::matvec through the engine: x is a torch cuda float32
        tensor [batch, cols]; returns [batch, rows]."""
        import torch
        qt_rows_cols = {n: (t, r, c) for n, t, r, c in self.cfg.matrices()}[name]
        _, rows, cols = qt_rows_cols
        y = torch.empty((batch, rows), dtype=torch.float32, device=x.device)
        _L.check(self.lib.ijb_matvec(self.h, self.tensor_index(name), x.data_ptr(), y.data_ptr(), cols, rows, batch,
                                     None), self.h)
        torch.cuda.synchronize(x.device)
        return y

    # ---- ragged batching
    def seq_open(self) -> int:
        s = ctypes.c_int(-1)
        _L.check(self.lib.ijb_seq_open(self.h, ctypes.byref(s)), self.h)
        return s.value

    def seq_close(self, seq: int) -> None:
        _L.check(self.lib.ijb_seq_close(self.h, int(seq)), self.h)

    def seq_length(self, seq: int) -> int:
        return self.lib.ijb_seq_length(self.h, int(seq))

    def seq_prefill(self, seq: int, tokens) -> int:
        arr = (ctypes.c_int * len(tokens))(*[int(t) for t in tokens])
        nxt = ctypes.c_int(-1)
        _L.check(self.lib.ijb_seq_prefill(self.h, int(seq), arr, len(tokens), ctypes.byref(nxt)), self.h)
        return nxt.value

    def decode_step(self, seq_ids, tokens) -> np.ndarray:
        s = np.ascontiguousarray(seq_ids, dtype=np.int32)
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        n = len(s)
        if len(t) != n:
            raise ValueError("seq_ids and tokens differ in length")
        out = np.empty(n, dtype=np.int32)
        ip = ctypes.POINTER(ctypes.c_int)
        _L.check(self.lib.ijb_decode_step(self.h, n, s.ctypes.data_as(ip), t.ctypes.data_as(ip),
                                          out.ctypes.data_as(ip)), self.h)
        return out

    def generate(self, seq_id: int, first_token: int, max_tokens: int, stop_ids=()) -> list:
        """ijb_generate: greedy tokens from first_token on, fed back on the device
        (the reference's decode loop: stop ids end it unemitted)."""
        out = (ctypes.c_int * max(1, max_tokens))()
        stops = (ctypes.c_int * max(1, len(stop_ids)))(*[int(v) for v in stop_ids])
        n = ctypes.c_int()
        _L.check(self.lib.ijb_generate(self.h, int(seq_id), int(first_token), int(max_tokens), stops, len(stop_ids),
                                       out, ctypes.byref(n)), self.h)
        return [int(v) for v in out[:n.value]]

    def time_layer_attention(self, seq_ids, reps: int = 20):
        """ijb_time_layer_attention: (ms per layer, K/V bytes per launch) of layer 0's
        attention for one token of each listed sequence at its newest position."""
        n = len(seq_ids)
        s = (ctypes.c_int * n)(*[int(v) for v in seq_ids])
        ms = ctypes.c_float()
        kvb = ctypes.c_longlong()
        _L.check(self.lib.ijb_time_layer_attention(self.h, n, s, int(reps), ctypes.byref(ms), ctypes.byref(kvb)),
                 self.h)
        return float(ms.value), int(kvb.value)

    def probe_wait_timeout(self, limit_ns: int) -> int:
        """ijb_probe_wait_timeout: the status code of a step whose bounded wait expired."""
        return int(self.lib.ijb_probe_wait_timeout(self.h, int(limit_ns)))

    def last_error(self) -> str:
        return self.lib.ijb_last_error(self.h).decode()

    def last_step_ms(self) -> float:
        """Device time of the last step (CUDA events on the engine's stream)."""
        return float(self.lib.ijb_last_step_ms(self.h))

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.ijb_destroy(self.h)
            self.h = None
        self._keep = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
