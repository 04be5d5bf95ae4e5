"""Row-split lm_head over the ranks of a process group (tensor parallel).

The reference computes the lm_head as one GEMV over all 128256 rows of the
tied Q6_K embedding, then a two-pass argmax (inferencer.cu:1519-1526,
:1063-1099).  Here rank r of `world` holds rows [r0, r1) of that matrix
(balanced: sizes differ by at most one row) as an ijb_weight and computes
their logits on the tensor cores for a batch of tokens, with the packed
argmax key of each token over its rows carrying the global row index.  Two
ways to finish the step:

* "logits": NCCL all-gather of every rank's logits slice (padded to the
  largest slice), reassembled into [n][vocab] on every rank; the next tokens
  come from the keys as below;
* "keys": one NCCL all-reduce (MAX) of the n packed keys (8 bytes a token);
  the maximum key over the ranks is the reference's argmax of the whole row
  (the key orders (value, tie rank) as an unsigned integer; its top bit is
  flipped on the wire so that signed 64-bit MAX keeps that order).

The default replicas need no data-path collective; this is the optional
measured variant.  torch.distributed provides the process group and the NCCL
calls; the projection and the key decoding are libijb200.so."""
from __future__ import annotations

import ctypes

import numpy as np

from . import lib as _L

SIGN = -(1 << 63)  # int64 with only the top bit set


def row_range(vocab: int, world: int, rank: int):
    """Rows [r0, r1) of rank `rank`: balanced, sizes differ by at most one."""
    return vocab * rank // world, vocab * (rank + 1) // world


def flip(keys_i64):
    """Unsigned key order <-> signed int64 order (top bit flipped)."""
    return keys_i64 ^ SIGN


class RowSplitLmHead:
    def __init__(self, blocks: np.ndarray, qtype: int, vocab: int, cols: int, rank: int = 0, world: int = 1,
                 device: int = 0):
        import torch
        self.lib = _L.load()
        self.vocab, self.cols, self.rank, self.world = vocab, cols, rank, world
        self.r0, self.r1 = row_range(vocab, world, rank)
        self.rows = self.r1 - self.r0
        self.rows_max = -(-vocab // world)
        self.device = torch.device(f"cuda:{device}")
        part = torch.from_numpy(np.ascontiguousarray(blocks[self.r0:self.r1])).to(self.device)
        h = ctypes.c_void_p()
        _L.check(self.lib.ijb_weight_create(qtype, part.data_ptr(), self.rows, cols, device, ctypes.byref(h)))
        self.h = h
        del part

    def local(self, x, norm_w=None, eps: float = 1e-5, dp4a: bool = True, stream=None):
        """This rank's logits [n][rows_max] (rows past self.rows are zero) and
        the packed argmax keys [n] (as int64) of its rows."""
        import torch
        n = x.shape[0]
        y = torch.zeros((n, self.rows_max), dtype=torch.float32, device=self.device)
        keys = torch.empty(n, dtype=torch.int64, device=self.device)
        s = stream if stream is not None else torch.cuda.current_stream(self.device).cuda_stream
        _L.check(self.lib.ijb_weight_matmul(self.h, x.data_ptr(), n, norm_w.data_ptr() if norm_w is not None else None,
                                            float(eps), int(dp4a), y.data_ptr(), self.rows_max, self.r0,
                                            keys.data_ptr(), ctypes.c_void_p(s)))
        return y, keys

    def tokens_from_keys(self, keys):
        """Packed keys (int64 tensor, unsigned order) -> token ids."""
        import torch
        out = torch.empty(keys.shape[0], dtype=torch.int32, device=self.device)
        s = torch.cuda.current_stream(self.device).cuda_stream
        _L.check(self.lib.ijb_keys_to_tokens(keys.data_ptr(), keys.shape[0], out.data_ptr(), ctypes.c_void_p(s)))
        return out

    def forward(self, x, norm_w=None, eps: float = 1e-5, dp4a: bool = True, gather: str = "logits", group=None):
        """Next tokens [n] (and, with gather="logits", the full logits
        [n][vocab] on every rank)."""
        import torch
        import torch.distributed as dist
        y, keys = self.local(x, norm_w, eps, dp4a)
        wk = flip(keys)
        if self.world > 1:
            dist.all_reduce(wk, op=dist.ReduceOp.MAX, group=group)
        tokens = self.tokens_from_keys(flip(wk))
        if gather != "logits":
            return tokens, None
        if self.world > 1:
            allg = torch.empty((self.world,) + tuple(y.shape), dtype=y.dtype, device=y.device)
            dist.all_gather_into_tensor(allg, y, group=group)
        else:
            allg = y.unsqueeze(0)
        counts = [row_range(self.vocab, self.world, r)[1] - row_range(self.vocab, self.world, r)[0]
                  for r in range(self.world)]
        return tokens, torch.cat([allg[r, :, :counts[r]] for r in range(self.world)], dim=1)

    def close(self):
        if getattr(self, "h", None):
            self.lib.ijb_weight_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
