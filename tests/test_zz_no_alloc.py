"""ijb_argmax_noalloc: the argmax for callers that cannot allocate device
memory (inside a CUDA graph capture, in host loops that cannot take the
synchronisation an allocation may cause, under a framework that owns all
device memory).  Checked through the C ABI against ijb_argmax, the entry
point that allocates its scratch on first use, over two calls in a row.

This file sorts last so that a run stopping at the first failure has already
run every other test; it also passes alone in a fresh process (the first
call looks up the scratch array's device address)."""
import numpy as np
import pytest

from ijb200 import lib

pytestmark = pytest.mark.gpu


def test_noalloc_argmax_matches_ijb_argmax(cuda):
    import torch
    L = lib.load()
    rng = np.random.default_rng(123)
    v1 = rng.standard_normal(128256).astype(np.float32)          # the vocab size
    v2 = rng.standard_normal(5000).astype(np.float32)
    v2[[3, 5, 300, 4000]] = 7.0                                   # equal maxima: the tie rule decides
    inputs = [torch.from_numpy(v).to(cuda) for v in (v1, v2)]
    ref = torch.full((2,), -7, dtype=torch.int32, device=cuda)
    got = torch.full((2,), -7, dtype=torch.int32, device=cuda)
    for i, vt in enumerate(inputs):
        lib.check(L.ijb_argmax(vt.data_ptr(), vt.numel(), ref[i:].data_ptr(), None))
    torch.cuda.synchronize()
    # two calls in a row on the same stream, sharing the static scratch
    for i, vt in enumerate(inputs):
        lib.check(L.ijb_argmax_noalloc(vt.data_ptr(), vt.numel(), got[i:].data_ptr(), None))
    torch.cuda.synchronize()
    assert got.tolist() == ref.tolist()
    assert int(got[0]) == int(np.argmax(v1))


def test_noalloc_argmax_allocates_nothing(cuda):
    import torch
    L = lib.load()
    v = torch.randn(100000, device=cuda)
    out = torch.zeros(1, dtype=torch.int32, device=cuda)
    lib.check(L.ijb_argmax_noalloc(v.data_ptr(), v.numel(), out.data_ptr(), None))  # first call: address lookup
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for _ in range(2):
        lib.check(L.ijb_argmax_noalloc(v.data_ptr(), v.numel(), out.data_ptr(), None))
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before
    assert int(out.item()) == int(torch.argmax(v).item())


def test_noalloc_argmax_rejects_sizes_beyond_its_scratch(cuda):
    import torch
    L = lib.load()
    v = torch.zeros(131073, device=cuda)
    out = torch.zeros(1, dtype=torch.int32, device=cuda)
    assert L.ijb_argmax_noalloc(v.data_ptr(), 131073, out.data_ptr(), None) == lib.ERR_INVALID
    assert "131072" in L.ijb_last_error(None).decode()
    assert L.ijb_argmax_noalloc(v.data_ptr(), 0, out.data_ptr(), None) == lib.ERR_INVALID
    lib.check(L.ijb_argmax_noalloc(v.data_ptr(), 131072, out.data_ptr(), None))
    torch.cuda.synchronize()
    assert int(out.item()) == 0  # all zeros: block 0, position 0 wins the ties
