"""Host logic of the row-split lm_head (ijb200.tp) on the CPU: balanced row
ranges, the key order kept through signed 64-bit MAX, and that MAX run as a
two-rank gloo all-reduce (the NCCL all-reduce of the GPU run)."""
import multiprocessing as mp
import os
import socket
import sys

import numpy as np
import pytest

from ijb200 import tp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_row_ranges_cover_the_vocab_once(world):
    v = 128256
    rs = [tp.row_range(v, world, r) for r in range(world)]
    assert rs[0][0] == 0 and rs[-1][1] == v
    assert all(rs[i][1] == rs[i + 1][0] for i in range(world - 1))
    sizes = [b - a for a, b in rs]
    assert max(sizes) - min(sizes) <= 1 and max(sizes) == -(-v // world)


def _key(value, index):
    """The packed key of the GPU argmax (argmax_key): ordered value bits, then
    0xFFFFFFFF - the bit-reversed rank of the index (the reference's tie rule)."""
    b = int(np.float32(value).view(np.uint32))
    ord_ = (~b & 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)
    blk, pos = index >> 8, index & 255
    rank = (int(f"{blk:09b}"[::-1], 2) << 8) | int(f"{pos:08b}"[::-1], 2)
    return (ord_ << 32) | (0xFFFFFFFF - rank)


def _signed(k):
    return k - (1 << 64) if k >= (1 << 63) else k


def test_signed_max_of_flipped_keys_is_the_unsigned_max():
    import torch
    rng = np.random.default_rng(0)
    vals = rng.standard_normal(500).astype(np.float32)
    vals[[3, 77]] = vals.max()  # a tie
    keys = [_key(v, i) for i, v in enumerate(vals)]
    signed = torch.tensor([_signed(k) for k in keys], dtype=torch.int64)
    best = int(tp.flip(torch.max(tp.flip(signed))).item()) & ((1 << 64) - 1)
    assert best == max(keys)
    assert (0 ^ tp.SIGN) < 0  # an empty key (0) sorts below every real key after the flip


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world)})
    sys.path.insert(0, os.path.join(REPO, "inferencer-jetson_b200"))
    try:
        import torch
        import torch.distributed as dist
        from ijb200 import tp as T
        dist.init_process_group("gloo", rank=rank, world_size=world)
        # rank r holds rows [r0, r1) of a 1000-row vocabulary; its best key per token
        vals = np.random.default_rng(5).standard_normal((4, 1000)).astype(np.float32)
        r0, r1 = T.row_range(1000, world, rank)
        local = [max(_key(v, r0 + i) for i, v in enumerate(row[r0:r1])) for row in vals]
        t = T.flip(torch.tensor([_signed(k) for k in local], dtype=torch.int64))
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        got = [int(v) & ((1 << 64) - 1) for v in T.flip(t).tolist()]
        want = [max(_key(v, i) for i, v in enumerate(row)) for row in vals]
        dist.destroy_process_group()
        q.put((rank, got == want))
    except Exception as ex:
        q.put((rank, repr(ex)))


def test_two_gloo_ranks_reduce_keys_to_the_global_argmax():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(o[1] is True for o in out), out
