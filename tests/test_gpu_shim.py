"""The C++ shim (host/fast_runner.hpp) as a drop-in for the reference's
runner: oracle/_ref/shim_check (built from oracle/shim_check.cu with the
reference's inferencer.cu #included unmodified, linked against libijb200.so)
loads one GGUF with the reference's own reader, builds the reference's
FastRunner and the shim's FastRunner from the same GGUF object with the
reference's constructor arguments (inferencer.cu:1196-1198), and drives both
through the calls the reference's main makes: forward with the timer and
gpu.x / gpu.logits, prefill, the --compare-prefill traces, FastGPU::matvec.
The model is the only shape the reference's runner accepts (3B), random-init."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from ijb200 import synth

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CHECK = os.path.join(REPO, "oracle", "_ref", "shim_check")


@pytest.fixture(scope="module")
def gguf_3b(tmp_path_factory):
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import gguf_writer
    path = str(tmp_path_factory.mktemp("gguf") / "synthetic_3b.gguf")
    gguf_writer.write_gguf(path, synth.LLAMA_3B, synth.make_model(synth.LLAMA_3B, seed=7))
    yield path
    os.remove(path)


@pytest.mark.parametrize("dp4a", [0, 1], ids=["fp32-path", "int8-path"])
def test_shim_is_a_drop_in_for_the_reference_runner(cuda, gguf_3b, dp4a):
    if not os.path.exists(CHECK):
        pytest.skip("oracle/_ref/shim_check not built (no reference checkout at build time)")
    toks = [str(int(t)) for t in synth.prompt_tokens(20, seed=5)]
    out = subprocess.run([CHECK, gguf_3b, str(dp4a)] + toks, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr
    r = json.loads(out.stdout.strip().splitlines()[-1])
    print("\n", r)
    n = r["tokens"]
    assert r["trace_layers"] == 28 and r["all_layer_trace"] == 28 * n
    assert r["quant_trace_vectors"] == 4 * 28 and r["first_quant_vectors"] == 4 * 28
    assert r["gpu_seconds"][1] > 0 and r["calls"][1] > 0
    # the reference's batched prefill always runs its INT8 kernels
    # (rmsnorm_quantize_batch_cuda + qkv_batch_cuda / gemv_batch_dp4a,
    # inferencer.cu:1265-1320), even on the FP32 path, so its prefill logits sit
    # at the INT8 path's floor (~2%) against any FP32 computation
    assert r["prefill_logits_rel"] < 5e-2
    assert r["matvec_rel"] < 1e-5
    if dp4a:
        # INT8 path: ulp-level differences flip int8 codes (the path's own floor,
        # ~2% in logits, see test_gpu_reference_runner.py)
        assert r["forward_agree"] >= 0.85 * n
        assert r["forward_logits_rel"] < 5e-2
        assert r["quant_trace_same"] > 0.3
    else:
        assert r["forward_agree"] == n
        assert r["forward_logits_rel"] < 1e-4 and r["forward_x_rel"] < 1e-4
        assert r["trace_rel"] < 1e-2 and r["quant_trace_same"] > 0.9
