"""Capture the reference's own full-model forward on a B200 as a golden fixture.

Run on a GPU box (needs oracle/_ref/libref_harness.so, built from the
reference's inferencer.cu by oracle/Makefile.ref):

    python tests/golden/make_ref_runner_golden.py <out_dir> [<scratch_dir>]

The reference's runner accepts only the Llama-3.2-3B shape
(inferencer.cu:1215-1217), so the model is synth.LLAMA_3B with seeded
random-init weights (synth.make_model(LLAMA_3B, seed=SEED)), written as a GGUF
file (oracle/gguf_writer.py) into <scratch_dir> (default /tmp) and loaded by
the reference's GGUF + FastRunner (inferencer.cu:204-340, :1182-1531) through
ref_run_gguf.  TOKENS are fed at positions 0..N-1 with need_logits on every
step, once on the FP32 activation path (--float-gemv --float-q6) and once on
the default INT8 path, both with the default (unfused) kernels.

``ref_runner_3b.npz`` holds, per path: the argmax of every step, the logits
at SAMPLE (a fixed seeded set of vocabulary rows) and at each step's 16
largest logits, and each step's full-vector L2 norm.  The tests run the CPU
oracle (tests/test_oracle.py) and the B200 engine (tests/test_gpu_reference_runner.py)
on the same model and tokens and compare.
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "inferencer-jetson_b200"))
sys.path.insert(0, os.path.join(REPO, "oracle"))
from ijb200 import synth  # noqa: E402

SEED = 7
N_TOKENS = 20
CONTEXT = 64


def tokens() -> np.ndarray:
    return synth.prompt_tokens(N_TOKENS, seed=5)


def sample_rows(vocab: int = 128256, n: int = 2048) -> np.ndarray:
    return np.sort(np.random.default_rng(99).choice(vocab, size=n, replace=False)).astype(np.int64)


def compact(logits: np.ndarray) -> dict:
    """What the fixture keeps of [steps][vocab] logits."""
    top = np.argsort(-logits, axis=1, kind="stable")[:, :16]
    return {"sample": logits[:, sample_rows()], "top_idx": top,
            "top_val": np.take_along_axis(logits, top, axis=1), "norm": np.linalg.norm(logits.astype(np.float64), axis=1)}


def run_reference(gguf_path: str, toks: np.ndarray, dp4a: bool, vocab: int = 128256):
    lib = ctypes.CDLL(os.path.join(REPO, "oracle", "_ref", "libref_harness.so"))
    lib.ref_last_error.restype = ctypes.c_char_p
    lib.ref_run_gguf.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                 ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    toks = np.ascontiguousarray(toks, dtype=np.int32)
    nxt = np.zeros(len(toks), dtype=np.int32)
    logits = np.zeros((len(toks), vocab), dtype=np.float32)
    rc = lib.ref_run_gguf(gguf_path.encode(), CONTEXT, toks.ctypes.data, len(toks), int(dp4a), int(dp4a), 0,
                          nxt.ctypes.data, logits.ctypes.data, vocab)
    if rc:
        raise RuntimeError(lib.ref_last_error().decode())
    return nxt, logits


def write_model(scratch: str) -> str:
    import gguf_writer
    path = os.path.join(scratch, f"synthetic_llama3b_seed{SEED}.gguf")
    if not os.path.exists(path):
        gguf_writer.write_gguf(path, synth.LLAMA_3B, synth.make_model(synth.LLAMA_3B, seed=SEED))
    return path


def main(out_dir: str, scratch: str = "/tmp") -> None:
    path = write_model(scratch)
    toks = tokens()
    out = {"tokens": toks, "sample_rows": sample_rows(), "seed": np.int64(SEED)}
    for tag, dp in (("fp32", False), ("int8", True)):
        nxt, logits = run_reference(path, toks, dp)
        out[f"{tag}_next"] = nxt
        for k, v in compact(logits).items():
            out[f"{tag}_{k}"] = v
    os.makedirs(out_dir, exist_ok=True)
    np.savez_compressed(os.path.join(out_dir, "ref_runner_3b.npz"), **out)
    print("wrote", os.path.join(out_dir, "ref_runner_3b.npz"), {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main(*sys.argv[1:])
