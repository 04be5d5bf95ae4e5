#!/usr/bin/env python3
"""Decode-throughput benchmark of the B200 hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload ragged64|decode1|ragged256_3b|gemv_q4k|gemv_q6k|gemm_q6k_b64|gemm_layer|
                                tp_lm_head|tokenize]

Workloads (seeded synthetic inputs; random-init weights, no checkpoint):
  ragged64  (default) Llama-3.2-1B-architecture Q4_K_M, 64 concurrent
            sequences, prompts U[16,1024], targets U[32,256]; finished
            sequences are replaced from the same distributions; paged fp16 KV,
            16-token pages.  The population starts pre-aged (each sequence at
            a uniform point of its output, its generated part prefilled), so
            replacements happen inside the timed window and contexts sit at
            the steady-state mix.  A step is one packed decode step over the
            64 live sequences.  The line also carries a `decode1` record
            (the batch-1 configuration on the same GPU) and a `tokenizer`
            record (the tokenize workload below, host only).
  decode1   same model, one sequence: 512-token prompt (ids U[0,128000),
            seed 1), then greedy decode steps.
  ragged256_3b  Llama-3.2-3B-architecture Q4_K_M (head_dim 128, 24 / 8
            heads), 256 ragged sequences per GPU, prompts U[64,4096], outputs
            U[64,512], pre-aged and replaced as in ragged64.
  gemv_q4k / gemv_q6k  BASELINE configs 0 / 1 (batch 1) in GB/s.
  gemm_q6k_b64  the vocab projection alone (tensor-core GEMM, 64 tokens).
  gemm_layer    one layer's four projection launches alone (tensor-core GEMM,
            64 tokens): the kernel the ragged64 roofline reports.
  tp_lm_head  the 3B lm_head (Q6_K 128256x3072) row-split over the N ranks,
            256 tokens per step: each rank's slice on the tensor cores, then
            an NCCL all-gather of the logits (the line's value) or one
            all-reduce of the packed argmax keys (`keys_only`); total work is
            fixed (strong scaling), checked against one GPU's full lm_head.
  tokenize  host tokenizer throughput (no GPU): ijb_tokenizer_encode over a
            seeded ~1 MB text corpus on one core, a fresh tokenizer (empty
            piece cache) per step, against the reference's own Tokenizer
            (oracle/_ref, same vocabulary) on the same corpus.
`value` is whole-job decode tokens/s: tokens generated in the K timed steps
on all ranks / max over ranks of the device time of those steps (CUDA events
around each step's graph).  Replacement prefills run between timed steps and
are not counted (the reference's "steady decode" excludes prefill too,
inferencer.cu:1877-1882, :1907-1908).  `e2e` is the same metric through the
C ABI call with host buffers (token ids in, next tokens out), wall-clocked.
Each rank runs an independent replica (no collective on the data path).

`--impl reference` times the reference's arithmetic on the host cores: the
CPU restatement of FastRunner::forward in oracle/ (the reference has no CPU
implementation of the path; its kernels are CUDA only), all host threads,
one sequence token per step at the workload's context lengths.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import random
import re
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "inferencer-jetson_b200"))
sys.path.insert(0, os.path.join(REPO, "oracle"))  # CPU baseline / reference arm only

from ijb200 import lib as ijblib, synth  # noqa: E402

MEASURED_PEAKS = os.path.join(REPO, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS = 6650.0
PROFILES = os.path.join(REPO, "profiles")
REF_HARNESS = os.path.join(REPO, "oracle", "_ref", "libref_harness.so")

# arithmetic of each path (what the step computes in, not a precision claim)
DTYPE_TC = ("fp16 x fp16 tcgen05 MMA, fp32 accumulate (weights: exact Q4_K/Q6_K dequant rounded to fp16; "
            "activations: the reference's int8 per-32 quantise-dequantise rounded to fp16); fp16 KV")
DTYPE_DP4A = "int8 x q4/q6 dp4a dot products, fp32 accumulate; fp16 KV"


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=48)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["ragged64", "decode1", "ragged256_3b", "gemv_q4k", "gemv_q6k",
                                           "gemm_q6k_b64", "gemm_layer", "tp_lm_head", "tokenize"],
                    default="ragged64")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="ragged64: skip the decode1 record, kernel timings and reference CUDA timings")
    ap.add_argument("--prompt", type=int, default=512, help="decode1 prompt length")
    ap.add_argument("--batch", type=int, default=0,
                    help="ragged workloads: live sequences (0 = the BASELINE config's 64 / 256; smaller for "
                         "profiling captures)")
    ap.add_argument("--prompt-max", type=int, default=1024,
                    help="ragged64 longest prompt (1024 in the BASELINE config; smaller for profiling captures)")
    ap.add_argument("--nvtx-step", action="store_true",
                    help="wrap the last timed step in an NVTX range 'step' (ncu --nvtx-include step/)")
    return ap.parse_args(argv)


# --------------------------------------------------------------- helpers --

def hbm_peak():
    try:
        with open(MEASURED_PEAKS) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profile_figure(name: str, key: str):
    """A figure recorded in a profiles/ summary as a `key: value` line (an
    ncu measurement of the same kernel, e.g. its DRAM bytes per launch)."""
    try:
        with open(os.path.join(PROFILES, name)) as f:
            for line in f:
                m = re.match(rf"\s*[-*]?\s*`?{re.escape(key)}`?\s*:\s*([0-9.eE+]+)", line)
                if m:
                    return float(m.group(1))
    except OSError:
        pass
    return None


REASON_NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


def _clock_record(rows, interval_ms, source):
    sm = [r[0] for r in rows if r[0] is not None]
    mx = [r[1] for r in rows if r[1] is not None]
    reasons = sorted({n for r in rows for n in r[2]})
    return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
            "reasons": reasons, "samples": len(rows), "interval_ms": interval_ms, "source": source}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every `interval_ms` from
    before the warm-up; only the samples that arrive inside the timed region
    (mark_start / mark_end) are reported.  Fallback of NvmlClockSampler."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int, interval_ms: int = 50, cmd=None):
        self.index = index
        self.interval_ms = interval_ms
        self.cmd = cmd
        self.rows = []  # (arrival time, (sm, max, reasons))
        self.proc = None
        self.t0 = None
        self.t1 = None

    def start(self):
        cmd = self.cmd or ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                           "--format=csv,noheader,nounits", "-lms", str(self.interval_ms)]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 6:
                num = lambda s: float(s) if s.replace(".", "").isdigit() else None  # noqa: E731
                reasons = [REASON_NAMES[i] for i in range(4) if parts[2 + i].lower() == "active"]
                self.rows.append((time.perf_counter(), (num(parts[0]), num(parts[1]), reasons)))

    def wait_first(self, timeout_s: float = 3.0):
        """Blocks until the sampler has produced a line (or timeout_s passed)."""
        end = time.perf_counter() + timeout_s
        while self.proc and not self.rows and time.perf_counter() < end and self.proc.poll() is None:
            time.sleep(0.01)

    def mark_start(self):
        self.t0 = time.perf_counter()

    def mark_end(self):
        self.t1 = time.perf_counter()

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        t0 = self.t0 if self.t0 is not None else float("-inf")
        t1 = self.t1 if self.t1 is not None else float("inf")
        return _clock_record([r for t, r in self.rows if t0 <= t <= t1], self.interval_ms, "nvidia-smi")


class NvmlClockSampler:
    """Read-only NVML queries of the SM clock and the active clock-event
    reasons every `interval_ms` (default 5 ms, so a timed region of a few tens
    of milliseconds still holds several samples).  The GPU is found by its PCI
    bus id, so the record belongs to the device this rank runs on whatever
    CUDA_VISIBLE_DEVICES says.  Nothing is set."""

    # nvmlClocksEventReason* bits
    BITS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, cuda_index: int, interval_ms: float = 5.0):
        import pynvml
        import torch
        self.nv = pynvml
        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(cuda_index)
        bus = "%08x:%02x:%02x.0" % (getattr(props, "pci_domain_id", 0), props.pci_bus_id, props.pci_device_id)
        self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
        self.interval_ms = interval_ms
        self.rows = []
        self.t0 = self.t1 = None
        self._stop = threading.Event()

    def _sample(self):
        nv = self.nv
        sm = float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
        get = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or nv.nvmlDeviceGetCurrentClocksThrottleReasons
        bits = int(get(self.h))
        return sm, self.max_mhz, [n for n, b in self.BITS.items() if bits & b]

    def _loop(self):
        while not self._stop.is_set():
            try:
                self.rows.append((time.perf_counter(), self._sample()))
            except Exception:
                pass
            time.sleep(self.interval_ms / 1e3)

    def start(self):
        self._sample()  # fails here (not in the thread) when NVML cannot be read
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()

    def wait_first(self, timeout_s: float = 3.0):
        end = time.perf_counter() + timeout_s
        while not self.rows and time.perf_counter() < end:
            time.sleep(0.001)

    def mark_start(self):
        self.t0 = time.perf_counter()

    def mark_end(self):
        self.t1 = time.perf_counter()

    def stop(self):
        self._stop.set()
        self.thread.join(timeout=2)
        t0 = self.t0 if self.t0 is not None else float("-inf")
        t1 = self.t1 if self.t1 is not None else float("inf")
        return _clock_record([r for t, r in self.rows if t0 <= t <= t1], self.interval_ms, "nvml")


def make_clock_sampler(cuda_index: int):
    try:
        s = NvmlClockSampler(cuda_index)
        s.start()
        return s
    except Exception:
        s = ClockSampler(cuda_index)
        s.start()
        return s


def dist_setup(n_gpus):
    """One process per GPU under torchrun: NCCL when CUDA is present (the bench),
    gloo otherwise (the CPU tests of the multi-rank bookkeeping)."""
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                    device_id=torch.device(f"cuda:{local}"))
        else:
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def reduce_max_sum(world, values_max, values_sum):
    """(max over ranks of values_max, sum over ranks of values_sum)."""
    if world == 1:
        return values_max, values_sum
    import torch
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    a = torch.tensor(values_max, dtype=torch.float64, device=dev)
    b = torch.tensor(values_sum, dtype=torch.float64, device=dev)
    dist.all_reduce(a, op=dist.ReduceOp.MAX)
    dist.all_reduce(b, op=dist.ReduceOp.SUM)
    return a.tolist(), b.tolist()


def barrier(world):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    if torch.cuda.is_available():
        torch.cuda.synchronize()


def job_throughput(world, tokens, dev_ms, wall_s):
    """Whole-job tokens/s: all ranks' tokens over the slowest rank's device time
    (`value`) and over the slowest rank's wall time (`e2e`)."""
    (max_dev_ms, max_wall), (sum_tokens,) = reduce_max_sum(world, [dev_ms, wall_s], [float(tokens)])
    return sum_tokens / (max_dev_ms / 1e3), sum_tokens / max_wall, max_dev_ms


# ------------------------------------------------------------ workloads --

class RaggedServer:
    """`batch` live sequences; replaces finished ones from the request stream.

    aged: each initial sequence starts at a uniform point g0 in [0, target) of
    its output, its prompt and the g0 tokens it would have generated prefilled
    (seeded synthetic ids stand in for them), so the population is already in
    its steady state when timing starts: sequences finish and are replaced
    throughout the timed window, and contexts follow the steady-state mix."""

    def __init__(self, eng, batch, seed, vocab_limit=128000, prompt_max=1024, aged=True, prompt_min=16,
                 out_range=(32, 256)):
        self.eng = eng
        self.prompt_min = prompt_min
        self.prompt_max = prompt_max
        self.out_range = out_range
        self.batch = batch
        self.rng = np.random.default_rng(seed)
        self.vocab_limit = vocab_limit
        self.live = []  # [seq_id, next_token, generated, target]
        self.prefill_tokens = 0
        self.prefill_s = 0.0
        self.replaced = 0
        for _ in range(batch):
            self.live.append(self._admit(aged))

    def _admit(self, aged=False):
        plen = int(self.rng.integers(self.prompt_min, self.prompt_max + 1))
        target = int(self.rng.integers(self.out_range[0], self.out_range[1] + 1))
        g0 = int(self.rng.integers(0, target)) if aged else 0
        prompt = self.rng.integers(0, self.vocab_limit, size=plen + g0).astype(np.int32)
        s = self.eng.seq_open()
        t0 = time.perf_counter()
        nxt = self.eng.seq_prefill(s, prompt)
        self.prefill_s += time.perf_counter() - t0
        self.prefill_tokens += len(prompt)
        return [s, nxt, g0, target]

    def contexts(self):
        return [self.eng.seq_length(e[0]) for e in self.live]

    def step(self):
        """One timed packed decode step; returns (tokens, device_ms, wall_s, kv_read_tokens)."""
        seqs = [e[0] for e in self.live]
        toks = [e[1] for e in self.live]
        ctx = sum(self.eng.seq_length(s) + 1 for s in seqs)
        t0 = time.perf_counter()
        out = self.eng.decode_step(seqs, toks)
        wall = time.perf_counter() - t0
        ms = self.eng.last_step_ms()
        for e, t in zip(self.live, out):
            e[1] = int(t)
            e[2] += 1
        return len(seqs), ms, wall, ctx

    def replace_finished(self):
        for i, e in enumerate(self.live):
            if e[2] >= e[3]:
                self.eng.seq_close(e[0])
                self.live[i] = self._admit()
                self.replaced += 1


GEMV_CASES = (("q4k_ffn_gate_8192x2048", 12, 8192, 2048), ("q6k_lm_head_128256x2048", 14, 128256, 2048))
# BASELINE config 1 at batch 8 (the CUDA-core GEMV's largest batch; batch 64 is the vocab projection)
GEMV_B8_CASE = ("q6k_lm_head_128256x2048_b8", 14, 128256, 2048, 8)


def gemv_roofline(cuda, peak, cases=GEMV_CASES, iters_min=20):
    """The CUDA-core GEMV (ijb_gemv_kernel, the batch-1 projection) timed
    alone: the 1B ffn_gate Q4_K shape and the Q6_K lm_head
    (config 1; a case may give a batch, up to 8), weights rotated over > 4x L2.
    The launches are captured into one CUDA graph, chained with programmatic
    dependent launch (IJB_GEMV_PDL: each GEMV's weight prefetch overlaps the
    previous one's tail), and the graph's replay is timed with CUDA events (a
    9.5 MB GEMV takes ~1.5 us at peak bandwidth, less than a host launch, so a
    host loop would time the host); the graph without PDL and the host loop are
    reported beside it."""
    import torch
    L = ijblib.load()
    out = {}
    rng = np.random.default_rng(0)
    for case in cases:
        name, qtype, rows, cols = case[:4]
        batch = case[4] if len(case) > 4 else 1
        w = synth.quant_matrix(rng, qtype, rows, cols)
        wd = torch.from_numpy(w).to(cuda)
        if qtype == 14:
            rb = L.ijb_q6k_planar_row_bytes(cols)
            wp = torch.empty(rows * rb, dtype=torch.uint8, device=cuda)
            ijblib.check(L.ijb_repack_q6k(wd.data_ptr(), wp.data_ptr(), rows, cols, None))
            wd = wp
        nbytes = wd.numel()
        copies = max(1, int(np.ceil(4 * 126e6 / nbytes)))
        ws = [wd] + [wd.clone() for _ in range(copies - 1)]
        x = torch.randn(batch, cols, device=cuda)
        y = torch.empty(batch, rows, device=cuda)
        stream = torch.cuda.current_stream().cuda_stream
        for i in range(3 * copies):
            ijblib.check(L.ijb_gemv(qtype, ws[i % copies].data_ptr(), x.data_ptr(), y.data_ptr(), cols, rows, batch, 1,
                                    ctypes.c_void_p(stream)))
        iters = max(iters_min, 4 * copies)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        for i in range(iters):
            ijblib.check(L.ijb_gemv(qtype, ws[i % copies].data_ptr(), x.data_ptr(), y.data_ptr(), cols, rows, batch, 1,
                                    ctypes.c_void_p(stream)))
        b.record()
        torch.cuda.synchronize()
        ms_loop = a.elapsed_time(b) / iters
        def graph_ms(flags):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                gs = torch.cuda.current_stream().cuda_stream
                for i in range(iters):
                    ijblib.check(L.ijb_gemv(qtype, ws[i % copies].data_ptr(), x.data_ptr(), y.data_ptr(), cols, rows,
                                            batch, flags, ctypes.c_void_p(gs)))
            graph.replay()
            torch.cuda.synchronize()
            a.record()
            graph.replay()
            b.record()
            torch.cuda.synchronize()
            del graph
            return a.elapsed_time(b) / iters
        ms_plain = graph_ms(1)
        ms = graph_ms(1 | ijblib.GEMV_PDL)
        algo = nbytes + batch * (cols * 4 + rows * 4)
        out[name] = {"us_per_launch": ms * 1e3, "algorithmic_bytes": algo, "gbs": algo / (ms * 1e-3) / 1e9,
                     "frac": algo / (ms * 1e-3) / 1e9 / peak, "rotated_copies": copies, "batch": batch,
                     "method": f"CUDA graph of {iters} launches chained with programmatic dependent launch",
                     "us_per_launch_graph_no_pdl": ms_plain * 1e3, "us_per_launch_host_loop": ms_loop * 1e3}
        del ws, wd
        torch.cuda.empty_cache()
    return out


def _timed_launches(fn, iters, stream_obj):
    """Mean milliseconds per fn() over `iters` calls, CUDA events on stream_obj."""
    import torch
    torch.cuda.synchronize()
    with torch.cuda.stream(stream_obj):
        for _ in range(3):
            fn()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream_obj)
        for _ in range(iters):
            fn()
        b.record(stream_obj)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def layer_roofline(cuda, peak, local, iters=20, batch=64):
    """The step's dominant kernel, timed as the step issues it: one layer's
    four tensor-core projection launches (QKV with RoPE and the K/V cache
    write, O + residual, gate/up + SiLU, down + residual; ijb_mma_gemm_kernel,
    each preceded by its activation prep ijb_mma_prep_kernel) for `batch`
    tokens, replayed `iters` times in one CUDA graph by
    ijb_time_layer_projections on a one-layer engine of the 1B widths (CUDA
    events on the engine's stream).  Algorithmic bytes per layer: the weights as
    stored + each projection's fp32 input read and output written (a residual
    add counts its read and its write) + the fp16 K/V written.  Each matrix
    alone through ijb_matvec (prep + GEMM per matrix) is reported beside it."""
    import torch
    L = ijblib.load()
    eng = _layer_engine(local, context=max(128, batch))
    cfg = eng.cfg
    ms = ctypes.c_float()
    ijblib.check(L.ijb_time_layer_projections(eng.h, batch, iters, ctypes.byref(ms)), eng.h)
    shapes = {n: (t, r, c) for n, t, r, c in cfg.matrices()}
    w_bytes = sum(r * (c // 256) * synth.BLOCK_BYTES[t] for n, (t, r, c) in shapes.items() if n.startswith("blk.0."))
    D, F, KV = cfg.dim, cfg.hidden, cfg.kv_dim
    act = batch * 4 * (D + D          # QKV: x read, q written
                       + D + 2 * D    # O: attention output read, residual read + written
                       + D + F        # gate/up: x read, h written
                       + F + 2 * D)   # down: h read, residual read + written
    act += batch * 2 * KV * 2 + 2 * D * 4  # K and V written (fp16), the two norm weight vectors
    algo = w_bytes + act
    gbs = algo / (ms.value * 1e-3) / 1e9
    side = torch.cuda.Stream(device=cuda)
    stream = side.cuda_stream
    per = {}
    for m in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"):
        name = f"blk.0.{m}.weight"
        t, rows, cols = shapes[name]
        x = torch.randn(batch, cols, device=cuda)
        y = torch.empty(batch, rows, device=cuda)
        idx = eng.tensor_index(name)

        def launch():
            ijblib.check(L.ijb_matvec(eng.h, idx, x.data_ptr(), y.data_ptr(), cols, rows, batch,
                                      ctypes.c_void_p(stream)), eng.h)
        us = _timed_launches(launch, iters, side) * 1e3
        b = rows * (cols // 256) * synth.BLOCK_BYTES[t] + batch * (cols + rows) * 4
        per[m] = {"us": us, "gbs": b / (us * 1e-6) / 1e9}
    eng.close()
    traffic = profile_figure("mma_gemm_layer_ragged64.md", "dram_bytes_per_layer")
    return {"kernel": f"ijb_mma_gemm_kernel + ijb_mma_prep_kernel: one layer's 4 projection launches as the step "
                      f"issues them, {batch} tokens (1B widths)", "us_per_layer": ms.value * 1e3,
            "algorithmic_bytes": algo, "weight_bytes": w_bytes, "gbs": gbs, "frac": gbs / peak,
            "traffic": traffic,
            "traffic_source": "profiles/mma_gemm_layer_ragged64.md (ncu dram__bytes_read.sum + "
                              "dram__bytes_write.sum over the layer's 8 launches)" if traffic else None,
            "per_matrix_alone": per}


def attention_roofline(eng, server, peak, head_dim, iters=20):
    """Decode attention as a step issues it: layer 0's launch (the streaming
    kernel ijb_attention_stream_kernel and its merge) for one token of every
    live sequence at its newest position, replayed `iters` times in one CUDA
    graph by ijb_time_layer_attention (CUDA events on the engine's stream).
    Algorithmic bytes per launch: every cached K and V row of those sequences
    (fp16), read once."""
    ids = [int(s[0]) for s in server.live]
    ms, kv_bytes = eng.time_layer_attention(ids, iters)
    gbs = kv_bytes / (ms * 1e-3) / 1e9
    prof = f"attention_stream_hd{head_dim}_traffic.md"
    ratio = profile_figure(prof, "traffic_per_algorithmic_byte")
    return {"kernel": f"ijb_attention_stream_kernel<{head_dim}, G> + ijb_attention_finish_kernel: one layer's decode "
                      f"attention for {len(ids)} sequences at their current contexts",
            "us_per_layer": ms * 1e3, "algorithmic_bytes": kv_bytes, "gbs": gbs, "frac": gbs / peak,
            "traffic": kv_bytes * ratio if ratio else None,
            "traffic_source": (f"profiles/{prof}: ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch "
                               f"of a smaller population divided by its K/V bytes ({ratio:.4f}), times this "
                               f"launch's K/V bytes")
            if ratio else None}


def mma_vocab_roofline(eng, cuda, peak, iters=20, batch=64):
    """The vocab projection (Q6_K 128256x2048, the largest single launch of a
    step) through ijb_matvec for `batch` tokens: activation prep +
    ijb_mma_gemm_kernel, CUDA events on its own stream."""
    import torch
    L = ijblib.load()
    cfg = eng.cfg
    idx = eng.tensor_index("token_embd.weight")
    cols, rows = cfg.dim, cfg.vocab
    x = torch.randn(batch, cols, device=cuda)
    y = torch.empty(batch, rows, device=cuda)
    side = torch.cuda.Stream(device=cuda)
    stream = side.cuda_stream

    def launch():
        ijblib.check(L.ijb_matvec(eng.h, idx, x.data_ptr(), y.data_ptr(), cols, rows, batch, ctypes.c_void_p(stream)),
                     eng.h)
    ms = _timed_launches(launch, iters, side)
    w_bytes = rows * (cols // 256) * 210
    algo = w_bytes + batch * cols * 4 + batch * rows * 4
    gbs = algo / (ms * 1e-3) / 1e9
    traffic = profile_figure("mma_gemm_q6k_vocab_b64.md", "dram_bytes_per_launch")
    return {"us_per_launch": ms * 1e3, "algorithmic_bytes": algo, "gbs": gbs, "frac": gbs / peak,
            "kernel": f"ijb_mma_gemm_kernel + ijb_mma_prep_kernel (Q6_K {rows}x{cols} vocab projection, {batch} tokens)",
            "traffic": traffic}


def reference_cuda_gemv(cases=GEMV_CASES):
    """The reference's own CUDA GEMVs (FastGPU::matvec: quantize_x32_cuda +
    gemv_q4_dp4a / gemv_q6_dp4a, inferencer.cu:544-674, :1156-1171, built
    unmodified for sm_100a into oracle/_ref/) timed on this GPU with CUDA
    events over weights rotated across > 4x L2, same inputs as gemv_roofline."""
    if not os.path.exists(REF_HARNESS):
        return {"unavailable": "oracle/_ref/libref_harness.so not built (the reference tree was absent at build)"}
    L = ctypes.CDLL(REF_HARNESS)
    L.ref_time_matvec.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                  ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                  ctypes.POINTER(ctypes.c_float)]
    L.ref_last_error.restype = ctypes.c_char_p
    rng = np.random.default_rng(0)
    out = {}
    for name, qt, rows, cols in cases:
        w = synth.quant_matrix(rng, qt, rows, cols)
        x = np.random.default_rng(1).standard_normal(cols).astype(np.float32)
        copies = max(1, int(np.ceil(4 * 126e6 / w.nbytes)))
        ms = ctypes.c_float()
        rc = L.ref_time_matvec(qt, w.ctypes.data, cols, rows, x.ctypes.data, 1, 1, 4, copies, max(20, 4 * copies),
                               ctypes.byref(ms))
        if rc:
            out[name] = {"error": L.ref_last_error().decode()}
            continue
        algo = w.nbytes + cols * 4 + rows * 4
        out[name] = {"us_per_launch": ms.value * 1e3, "gbs": algo / (ms.value * 1e-3) / 1e9,
                     "path": "INT8 DP4A (reference default), 4 warps per Q6_K CTA"}
    return out


def decode_3b_b1(local, prompt_len=128, steps=64, scratch="/tmp"):
    """The only full-model configuration the reference's runner accepts
    (Llama-3.2-3B shape, inferencer.cu:1215-1217), batch 1, on this GPU: the
    reference's own GGUF + FastRunner (unmodified, built into oracle/_ref/;
    steady decode as in its main loop, inferencer.cu:1870-1883: each
    forward() ends in its blocking token download) and this build's engine on
    the same seeded weights, prompt and step count.  Tokens/s over the decode
    steps; the reference's number is wall time (its own measure), the
    engine's is given both ways."""
    out = {"config": f"llama-3.2-3b-shape Q4_K_M random-init, batch 1, {prompt_len}-token prompt, {steps} steps"}
    cfg = synth.LLAMA_3B
    weights = synth.make_model(cfg, seed=7)
    prompt = synth.prompt_tokens(prompt_len, seed=5)
    if os.path.exists(REF_HARNESS):
        try:
            import gguf_writer
            path = os.path.join(scratch, "bench_llama3b_seed7.gguf")
            gguf_writer.write_gguf(path, cfg, weights)
            L = ctypes.CDLL(REF_HARNESS)
            L.ref_last_error.restype = ctypes.c_char_p
            L.ref_time_decode.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_int, ctypes.POINTER(ctypes.c_double)]
            secs = ctypes.c_double()
            p32 = np.ascontiguousarray(prompt, dtype=np.int32)
            rc = L.ref_time_decode(path.encode(), prompt_len + steps + 8, p32.ctypes.data, prompt_len, steps, 0,
                                   ctypes.byref(secs))
            os.remove(path)
            out["reference"] = ({"tokens_per_s": steps / secs.value, "ms_per_token": secs.value / steps * 1e3,
                                 "timing": "wall, blocking token download per step"} if rc == 0
                                else {"error": L.ref_last_error().decode()})
        except Exception as ex:  # reported, not fatal
            out["reference"] = {"error": repr(ex)}
    else:
        out["reference"] = {"unavailable": "oracle/_ref/libref_harness.so not built"}
    from ijb200.engine import Engine
    eng = Engine(cfg, weights, context=prompt_len + steps + 8, max_batch=1, max_seqs=2, device=local)
    nxt = eng.prefill(prompt)
    dev_ms, wall = 0.0, 0.0
    for i in range(steps):
        t0 = time.perf_counter()
        nxt = eng.forward(nxt, prompt_len + i, True)
        wall += time.perf_counter() - t0
        dev_ms += eng.last_step_ms()
    eng.close()
    out["ours"] = {"tokens_per_s_device": steps / (dev_ms / 1e3), "tokens_per_s_wall": steps / wall,
                   "ms_per_token_device": dev_ms / steps}
    return out


def cpu_forward(cfg, weights, contexts, threads, budget_s=20.0):
    """The oracle's FastRunner::forward on the host cores: decode one token at
    each sampled context length; returns tokens/s and the sample used."""
    import oracle as O
    O.set_threads(threads)
    m = O.OracleModel(cfg, weights, max(contexts) + 2, True, True)
    done, t_total, used = 0, 0.0, []
    for ctx in contexts:
        st = m.new_state()
        st.fill_kv(ctx)
        t0 = time.perf_counter()
        st.forward(1, ctx, True)
        t_total += time.perf_counter() - t0
        done += 1
        used.append(ctx)
        del st
        if t_total > budget_s:
            break
    return done / t_total, used


def cpu_gemv(threads, budget_s=6.0):
    """The oracle's FastGPU::matvec (INT8 path) on the host cores over the two
    GEMV configs, GB/s of quantised weights + activation + output."""
    import oracle as O
    O.set_threads(threads)
    rng = np.random.default_rng(0)
    out = {}
    for name, qt, rows, cols in GEMV_CASES:
        w = synth.quant_matrix(rng, qt, rows, cols)
        x = rng.standard_normal(cols).astype(np.float32)
        n, t = 0, 0.0
        while t < budget_s / 2 and n < 50:
            t0 = time.perf_counter()
            O.matvec(qt, w, x, cols, rows)
            t += time.perf_counter() - t0
            n += 1
        algo = w.nbytes + cols * 4 + rows * 4
        out[name] = {"ms_per_call": t / n * 1e3, "gbs": algo * n / t / 1e9, "calls": n}
    return out


# ------------------------------------------------------------------ arms --

def run_gemv(args):
    """BASELINE configs 0 / 1: one GEMV per step, weights rotated over > 4x L2."""
    import torch
    world, rank, local = dist_setup(args.gpus)
    cuda = torch.device(f"cuda:{local}")
    peak, src = hbm_peak()
    case = GEMV_CASES[0] if args.workload == "gemv_q4k" else GEMV_CASES[1]
    r = gemv_roofline(cuda, peak, (case,), iters_min=args.steps)[case[0]]
    if rank != 0:
        return None
    return {"metric": "GEMV HBM GB/s (" + case[0] + ", batch 1)", "value": r["gbs"], "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["us_per_launch"] / 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": DTYPE_DP4A,
            "data": "synthetic (seeded)", "config": {"workload": case[0], "rotated_copies": r["rotated_copies"]},
            "roofline": {"bound": "hbm", "achieved": r["gbs"], "peak": peak, "unit": "GB/s", "frac": r["frac"],
                         "traffic": None, "peak_source": src},
            "reference_cuda": reference_cuda_gemv((case,)).get(case[0])}


def _layer_engine(local, layers=1, context=32):
    full = synth.LLAMA_1B
    cfg = synth.ModelConfig(f"llama-3.2-1b-{layers}layer", dim=full.dim, layers=layers, heads=full.heads,
                            kv_heads=full.kv_heads, hidden=full.hidden, vocab=full.vocab)
    from ijb200.engine import Engine
    return Engine(cfg, synth.make_model(cfg, seed=0), context=context, max_batch=64, max_seqs=2, device=local)


def run_gemm(args):
    """The tensor-core GEMM alone: the vocab projection (gemm_q6k_b64) or one
    layer's seven projections (gemm_layer)."""
    import torch
    world, rank, local = dist_setup(args.gpus)
    cuda = torch.device(f"cuda:{local}")
    peak, src = hbm_peak()
    if args.workload == "gemm_layer":
        r = layer_roofline(cuda, peak, local, iters=max(args.steps, 5))
        metric, value, ms = ("GEMM HBM GB/s (one 1B layer's 4 projection launches, 64 tokens)", r["gbs"],
                             r["us_per_layer"] / 1e3)
    else:
        eng = _layer_engine(local)
        r = mma_vocab_roofline(eng, cuda, peak, iters=max(args.steps, 5))
        metric, value, ms = "GEMM HBM GB/s (Q6_K 128256x2048 vocab projection, 64 tokens)", r["gbs"], r["us_per_launch"] / 1e3
        eng.close()
    if rank != 0:
        return None
    return {"metric": metric, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": 3,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": DTYPE_TC,
            "data": "synthetic (seeded)", "config": {"workload": args.workload, "l2": "weights > L2 per pass"},
            "roofline": {"bound": "hbm", "achieved": value, "peak": peak, "unit": "GB/s", "frac": value / peak,
                         "traffic": r["traffic"], "kernel": r["kernel"], "peak_source": src}}


def decode1_record(cuda, local, cfg, weights, peak, steps, warmup, prompt_len=512):
    """BASELINE config 2 on this GPU: batch 1 after a 512-token prompt,
    `steps` greedy steps (device time per step from CUDA events around the
    step graph; e2e wall time of the ijb_forward calls)."""
    from ijb200.engine import Engine
    eng = Engine(cfg, weights, context=prompt_len + steps + warmup + 8, max_batch=1, max_seqs=2, device=local)
    prompt = synth.prompt_tokens(prompt_len, seed=1)
    nxt = eng.prefill(prompt)
    pos = len(prompt)
    for _ in range(warmup):
        nxt = eng.forward(nxt, pos, True)
        pos += 1
    dev_ms, wall, ctx = 0.0, 0.0, 0
    for _ in range(steps):
        t0 = time.perf_counter()
        nxt = eng.forward(nxt, pos, True)
        wall += time.perf_counter() - t0
        dev_ms += eng.last_step_ms()
        pos += 1
        ctx += pos
    eng.close()
    # the same decode with the token fed back on the device (ijb_generate, the
    # reference's decode loop): one call for `steps` tokens after the prompt
    eng = Engine(cfg, weights, context=prompt_len + 2 * steps + 8, max_batch=1, max_seqs=2, device=local)
    seq = eng.seq_open()
    first = eng.seq_prefill(seq, prompt)
    eng.generate(seq, first, 4)  # the generate step graph is captured here
    t0 = time.perf_counter()
    toks = eng.generate(seq, first, steps + 1)
    gen_wall = time.perf_counter() - t0
    gen_ms = eng.last_step_ms()
    eng.close()
    step_bytes = cfg.weight_bytes() + cfg.kv_bytes_per_token(2) * ctx / steps
    ms = dev_ms / steps
    return {"metric": "decode tokens/s (1B Q4_K_M, batch 1)", "value": steps / (dev_ms / 1e3), "unit": "tokens/s",
            "ms_per_step": ms, "steps": steps, "warmup": warmup, "dtype": DTYPE_DP4A,
            "e2e": {"value": steps / wall, "unit": "tokens/s", "h2d_bytes_per_step": 16,
                    "d2h_bytes_per_step": 8},  # the next token and the device status word
            "generate": {"value": (len(toks) - 1) / gen_wall, "unit": "tokens/s",
                         "device_ms_per_step": gen_ms,
                         "method": f"one ijb_generate call for {steps} decode steps after the {prompt_len}-token "
                                   "prompt, token feedback on the device, wall time of the call"},
            "config": {"workload": f"llama-3.2-1b Q4_K_M decode, batch 1, {prompt_len}-token prompt"},
            "step_roofline": {"bytes_per_step": step_bytes, "achieved_gbs": step_bytes / (ms * 1e-3) / 1e9,
                              "frac": step_bytes / (ms * 1e-3) / 1e9 / peak}}


def run_tp_lm_head(args):
    """BASELINE config 4's optional variant: the lm_head row-split over the
    ranks with an NCCL all-gather of the logits (ijb200.tp)."""
    import torch
    import torch.distributed as dist
    world, rank, local = dist_setup(args.gpus)
    cuda = torch.device(f"cuda:{local}")
    peak, src = hbm_peak()
    from ijb200 import tp
    cfg = synth.LLAMA_3B
    rng = np.random.default_rng(7)
    blocks = synth.quant_matrix(rng, 14, cfg.vocab, cfg.dim, d_range=(2e-5, 4e-5))
    norm_w = torch.from_numpy(rng.uniform(0.8, 1.2, cfg.dim).astype(np.float32)).to(cuda)
    n = 256
    x = torch.from_numpy(np.random.default_rng(8).standard_normal((n, cfg.dim)).astype(np.float32)).to(cuda)
    head = tp.RowSplitLmHead(blocks, 14, cfg.vocab, cfg.dim, rank, world, local)
    timings = {}
    tokens = logits = None
    for mode in ("keys", "logits"):
        for _ in range(max(3, args.warmup)):
            head.forward(x, norm_w, cfg.eps, True, gather=mode)
        barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            tokens, logits = head.forward(x, norm_w, cfg.eps, True, gather=mode)
        b.record()
        barrier(world)
        (ms_max,), _ = reduce_max_sum(world, [a.elapsed_time(b) / args.steps], [0.0])
        timings[mode] = ms_max
    check = None
    if rank == 0:
        full = tp.RowSplitLmHead(blocks, 14, cfg.vocab, cfg.dim, 0, 1, local)
        ft, fl = full.forward(x, norm_w, cfg.eps, True, gather="logits")
        rel = float(torch.linalg.norm(logits - fl) / torch.linalg.norm(fl))
        check = {"logits_rel_l2_vs_one_gpu": rel, "tokens_equal": float((tokens == ft).float().mean())}
        full.close()
    head.close()
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None
    step_bytes = cfg.vocab * (cfg.dim // 256) * 210 + n * cfg.dim * 4 + n * cfg.vocab * 4
    ms = timings["logits"]
    achieved = step_bytes / world / (ms * 1e-3) / 1e9
    return {"metric": "lm_head tokens/s (3B Q6_K 128256x3072, row-split, all-gather of logits)",
            "value": n / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": DTYPE_TC, "data": "synthetic (seeded)",
            "config": {"workload": "tp_lm_head", "tokens": n, "rows_per_rank": -(-cfg.vocab // world),
                       "parallelism": f"tp{world} (lm_head rows)"},
            "keys_only": {"ms_per_step": timings["keys"], "value": n / (timings["keys"] * 1e-3),
                          "bytes_per_rank": n * 8},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": None,
                         "kernel": "ijb_mma_gemm_kernel (each rank's lm_head slice) + NCCL all-gather",
                         "peak_source": src},
            "check": check}


TOKENIZE_ITEMS = 240_000  # random_text items of the corpus (~1.1 MB)


def tokenize_setup():
    """The synthetic vocabulary and the seeded corpus of the tokenize workload."""
    from ijb200 import synth_vocab as sv
    tokens, merges = sv.vocabulary()
    rng = random.Random(31)
    corpus = [sv.random_text(rng, 400).encode() for _ in range(TOKENIZE_ITEMS // 400)]
    return tokens, merges, corpus


def reference_tokenize(tokens, merges, corpus, budget_s=15.0):
    """The reference's Tokenizer (inferencer.cu:361-451, oracle/_ref) over the
    corpus's texts in order until budget_s: (tokens/s, bytes/s, sample)."""
    if not os.path.exists(REF_HARNESS):
        return None
    import tempfile
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    from gguf_writer import write_vocab_gguf
    lib = ctypes.CDLL(REF_HARNESS)
    lib.ref_last_error.restype = ctypes.c_char_p
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "vocab.gguf").encode()
        write_vocab_gguf(path.decode(), tokens, merges)
        n = ctypes.c_long()
        buf = (ctypes.c_int * 1)()
        lib.ref_tokenize(path, b"warm", 4, buf, 0, ctypes.byref(n))  # builds the GGUF and Tokenizer
        toks = nbytes = done = 0
        t0 = time.perf_counter()
        for text in corpus:
            if lib.ref_tokenize(path, text, len(text), buf, 0, ctypes.byref(n)):
                raise RuntimeError(lib.ref_last_error().decode())
            toks += n.value
            nbytes += len(text)
            done += 1
            if time.perf_counter() - t0 > budget_s:
                break
        dt = time.perf_counter() - t0
    return toks / dt, nbytes / dt, f"{done} of {len(corpus)} corpus texts ({nbytes} bytes) in {dt:.1f} s"


def run_tokenize(args):
    """Host tokenizer throughput; `value` is encode tokens/s on one core."""
    from ijb200.tokenizer import Tokenizer
    tokens, merges, corpus = tokenize_setup()
    nbytes = sum(map(len, corpus))
    ref = reference_tokenize(tokens, merges, corpus)
    ref_rec = ({"value": ref[0], "unit": "tokens/s", "bytes_per_s": ref[1], "cores": 1, "kind": "reference",
                "sample": ref[2]} if ref else
               {"unavailable": "oracle/_ref/libref_harness.so not built (the reference tree was absent at build)"})
    if args.impl == "reference":
        if not ref:
            return {"impl": "reference", **ref_rec}
        return {"impl": "reference", "metric": "tokenizer encode tokens/s (host, 1 core)", "value": ref[0],
                "unit": "tokens/s", "higher_is_better": True, "cpu_baseline": ref_rec,
                "e2e": {"value": ref[0], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                "config": {"workload": "tokenize"}}
    times = []
    count = 0
    for k in range(args.warmup + args.steps):
        tok = Tokenizer(tokens, merges)  # empty piece cache every step
        t0 = time.perf_counter()
        count = sum(len(tok.encode(text)) for text in corpus)
        dt = time.perf_counter() - t0
        tok.close()
        if k >= args.warmup:
            times.append(dt)
    dt = float(np.median(times))
    # the same corpus through the batch entry point on every host core
    cores = os.cpu_count() or 1
    mt = []
    for k in range(args.warmup + args.steps):
        tok = Tokenizer(tokens, merges)
        t0 = time.perf_counter()
        n_mt = sum(map(len, tok.encode_batch(corpus, cores)))
        mt.append(time.perf_counter() - t0)
        tok.close()
    dt_mt = float(np.median(mt[args.warmup:]))
    assert n_mt == count
    return {"metric": "tokenizer encode tokens/s (host, 1 core)", "value": count / dt, "unit": "tokens/s",
            "higher_is_better": True, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
            "bytes_per_s": nbytes / dt, "tokens_per_step": count, "n_gpus": 0, "gpu_launches": 0,
            "data": "synthetic (seeded text; 128256-token vocabulary around 700 trained merges)",
            "config": {"workload": "tokenize", "corpus_bytes": nbytes, "texts": len(corpus),
                       "method": "one pass of ijb_tokenizer_encode over the corpus per step, a fresh tokenizer "
                                 "(empty piece cache) each step, median step"},
            "batch_all_cores": {"value": count / dt_mt, "unit": "tokens/s", "cores": cores,
                                "method": "ijb_tokenizer_encode_batch over the corpus's texts, one fresh tokenizer "
                                          "per step, a piece cache per worker thread, median step"},
            "reference": ref_rec}


def run_ours(args):
    import torch
    if args.workload == "tokenize":
        return run_tokenize(args)
    if args.workload == "tp_lm_head":
        return run_tp_lm_head(args)
    if args.workload.startswith("gemv"):
        return run_gemv(args)
    if args.workload.startswith("gemm"):
        return run_gemm(args)
    world, rank, local = dist_setup(args.gpus)
    cuda = torch.device(f"cuda:{local}")
    peak, peak_src = hbm_peak()
    big = args.workload == "ragged256_3b"
    cfg = synth.LLAMA_3B if big else synth.LLAMA_1B
    t_setup = time.perf_counter()
    weights = synth.make_model(cfg, seed=0)
    from ijb200.engine import Engine
    if args.workload == "ragged64":
        batch, context = args.batch or 64, args.prompt_max + 256 + 16
        eng = Engine(cfg, weights, context=context, max_batch=batch, max_seqs=batch + 1, device=local)
        server = RaggedServer(eng, batch, seed=1000 + rank, prompt_max=args.prompt_max)
    elif big:
        pmax = min(args.prompt_max * 4, 4096)  # 4096 by default
        batch, context = args.batch or 256, pmax + 512 + 16
        eng = Engine(cfg, weights, context=context, max_batch=batch, max_seqs=batch + 1, device=local)
        server = RaggedServer(eng, batch, seed=2000 + rank, prompt_max=pmax, prompt_min=64, out_range=(64, 512))
    else:
        batch, context = 1, args.prompt + 16 + args.steps + args.warmup + 8
        eng = Engine(cfg, weights, context=context, max_batch=1, max_seqs=2, device=local)
        prompt = synth.prompt_tokens(args.prompt, seed=1)
        nxt = eng.prefill(prompt)
        pos = len(prompt)
    setup_s = time.perf_counter() - t_setup

    ragged = args.workload in ("ragged64", "ragged256_3b")

    def one_step():
        nonlocal nxt, pos
        if ragged:
            return server.step()
        t0 = time.perf_counter()
        nxt = eng.forward(nxt, pos, True)
        wall = time.perf_counter() - t0
        pos += 1
        return 1, eng.last_step_ms(), wall, pos

    sampler = make_clock_sampler(local)
    # warm-up (includes graph capture)
    for _ in range(args.warmup):
        one_step()
        if ragged:
            server.replace_finished()
    sampler.wait_first()
    replaced0 = server.replaced if ragged else 0
    barrier(world)
    sampler.mark_start()
    launches0 = ijblib.load().ijb_kernel_launches()
    tokens, dev_ms, wall_s, kv_tokens, replaced_s = 0, 0.0, 0.0, 0, 0.0
    t_region = time.perf_counter()
    for k in range(args.steps):
        if args.nvtx_step and k == args.steps - 1:
            torch.cuda.nvtx.range_push("step")
        n, ms, wall, ctx = one_step()
        if args.nvtx_step and k == args.steps - 1:
            torch.cuda.nvtx.range_pop()
        tokens += n
        dev_ms += ms
        wall_s += wall
        kv_tokens += ctx
        if ragged:
            t0 = time.perf_counter()
            server.replace_finished()
            replaced_s += time.perf_counter() - t0
    barrier(world)
    sampler.mark_end()
    region_s = time.perf_counter() - t_region
    launches = ijblib.load().ijb_kernel_launches() - launches0
    clocks = sampler.stop()
    if clocks.get("sm_mhz"):
        clocks["ms_per_step_x_sm_mhz"] = dev_ms / args.steps * clocks["sm_mhz"]

    value, e2e, max_dev_ms = job_throughput(world, tokens, dev_ms, wall_s)
    ms_per_step = max_dev_ms / args.steps

    # step roofline: quantised weights + norms, KV read for every live context
    # (K and V, fp16) and the new K/V written, per step
    w_bytes = cfg.weight_bytes()
    kv_per_tok = cfg.kv_bytes_per_token(2)
    step_bytes = w_bytes + kv_per_tok * (kv_tokens / args.steps)
    step_gbs = step_bytes / (ms_per_step * 1e-3) / 1e9

    result = None
    if rank == 0:
        extras = args.workload == "ragged64" and not args.no_extras
        kern = gemv_roofline(cuda, peak, GEMV_CASES + ((GEMV_B8_CASE,) if extras else ())) if (extras or not ragged) \
            else None
        att = attention_roofline(eng, server, peak, cfg.head_dim) if ragged else None
        if big:
            # K/V reads are ~97% of this step's bytes: the dominant kernel is the attention
            dom = dict(att, weight_bytes=None, per_matrix_alone=None)
            vocab = None
        elif ragged:
            dom = layer_roofline(cuda, peak, local)
            vocab = mma_vocab_roofline(eng, cuda, peak) if extras else None
        else:
            dom = dict(kern["q6k_lm_head_128256x2048"], traffic=None,
                       kernel="ijb_gemv_kernel (Q6_K lm_head 128256x2048, B=1)")
            vocab = None
        ctxs = ([int(c) for c in server.contexts()[:8]] if ragged else [pos] * 4)
        eng.close()
        eng = None
        torch.cuda.empty_cache()
        d1 = decode1_record(cuda, local, cfg, weights, peak, 32, 4) if extras else None
        cpu = cpu_extra = None
        if world == 1 and not args.no_cpu_baseline:
            nthreads = os.cpu_count() or 1
            tps, used = cpu_forward(cfg, weights, ctxs, nthreads)
            cpu = {"value": tps, "unit": "tokens/s", "cores": nthreads, "kind": "port",
                   "sample": f"oracle FastRunner::forward (INT8 path), one decode token at each context {used}, "
                             f"{nthreads} threads"}
            if extras:
                tps1, used1 = cpu_forward(cfg, weights, ctxs[:2], 1, budget_s=8.0)
                cpu_extra = {"forward_1_thread": {"value": tps1, "unit": "tokens/s", "cores": 1,
                                                  "sample": f"one decode token at each context {used1}"},
                             "gemv_1_thread": cpu_gemv(1), f"gemv_{nthreads}_threads": cpu_gemv(nthreads)}
        h2d = 4 * batch * 4  # token, seq, position, KV slot per entry (int32)
        metric = (f"decode tokens/s (3B Q4_K_M, batch {batch})" if big else
                  f"decode tokens/s (1B Q4_K_M, batch {batch})" if ragged else "decode tokens/s (1B Q4_K_M, batch 1)")
        workload = (f"llama-3.2-3b Q4_K_M ragged decode, {batch} seqs, prompts U[64,{server.prompt_max}], outputs "
                    "U[64,512], replacement, pre-aged population" if big else
                    f"llama-3.2-1b Q4_K_M ragged decode, {batch} seqs, prompts U[16,{args.prompt_max}], "
                    "outputs U[32,256], replacement, pre-aged population" if ragged
                    else f"llama-3.2-1b Q4_K_M decode, batch 1, {args.prompt}-token prompt")
        result = {
            "metric": metric,
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": DTYPE_TC if ragged else DTYPE_DP4A, "data": "synthetic (random-init weights, seeded)",
            "config": {"workload": workload,
                       "batch_per_gpu": batch, "page_size": 16, "kv": "fp16 paged",
                       "parallelism": f"replicas x{world}",
                       "l2": f"inputs larger than L2 ({w_bytes / 1e6:.0f} MB weights/step)",
                       "mean_context": kv_tokens / args.steps / batch,
                       "replaced_in_window": (server.replaced - replaced0) if ragged else 0},
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": 4 * batch + 4},  # next tokens + the device status word
            "gpu_launches": int(launches),
            "roofline": {"bound": "hbm", "achieved": dom["gbs"], "peak": peak, "unit": "GB/s",
                         "frac": dom["frac"], "traffic": dom["traffic"], "kernel": dom["kernel"],
                         "peak_source": peak_src,
                         **({k: dom[k] for k in ("us_per_layer", "weight_bytes", "algorithmic_bytes",
                                                 "traffic_source", "per_matrix_alone")} if ragged else
                            {"us_per_launch": dom["us_per_launch"]})},
            "step_roofline": {"bytes_per_step": step_bytes, "achieved_gbs": step_gbs, "frac": step_gbs / peak},
            "cpu_baseline": cpu,
            "clocks": clocks,
            "setup_s": setup_s,
            "region_wall_s": region_s,
        }
        if vocab:
            result["vocab_projection"] = vocab
        if att and not big:
            result["attention"] = {k: att[k] for k in ("kernel", "us_per_layer", "algorithmic_bytes", "gbs", "frac",
                                                        "traffic", "traffic_source")}
        if kern:
            result["gemv"] = kern
        if d1:
            result["decode1"] = d1
        if cpu_extra:
            result["cpu_baseline_extra"] = cpu_extra
        if extras:
            try:  # the host tokenizer (no GPU), one warm-up and three timed passes beside the reference's
                tk = run_tokenize(parse(["--workload", "tokenize", "--steps", "3", "--warmup", "1"]))
                result["tokenizer"] = {k: tk[k] for k in ("metric", "value", "unit", "bytes_per_s", "batch_all_cores",
                                                          "reference", "data", "config")}
            except Exception as ex:  # reported, not fatal
                result["tokenizer"] = {"error": repr(ex)}
            result["reference_cuda"] = {"gemv": reference_cuda_gemv()}
            try:
                result["reference_cuda"]["decode_3b_b1"] = decode_3b_b1(local)
            except Exception as ex:  # reported, not fatal
                result["reference_cuda"]["decode_3b_b1"] = {"error": repr(ex)}
        if ragged:
            result["prefill"] = {"tokens": server.prefill_tokens, "seconds": server.prefill_s,
                                 "tokens_per_s": server.prefill_tokens / max(server.prefill_s, 1e-9),
                                 "method": "wall time of the population's prefills (ijb_seq_prefill, chunks of "
                                           "max_batch tokens through the decode kernels), outside the timed steps"}
    if eng is not None:
        eng.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return result


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    if args.workload == "tokenize":
        return run_tokenize(args)
    import oracle as O
    big = args.workload == "ragged256_3b"
    cfg = synth.LLAMA_3B if big else synth.LLAMA_1B
    weights = synth.make_model(cfg, seed=0)
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    rng = np.random.default_rng(1000)
    if args.workload == "ragged64":
        # contexts of a steady ragged population: prompt U[16,1024] + generated so far
        ctxs = [int(rng.integers(16, 1025) + rng.integers(0, 257)) for _ in range(args.steps + args.warmup)]
    elif big:
        ctxs = [int(rng.integers(64, 4097) + rng.integers(0, 513)) for _ in range(args.steps + args.warmup)]
    else:
        ctxs = [512 + i for i in range(args.steps + args.warmup)]
    m = O.OracleModel(cfg, weights, max(ctxs) + 2, True, True)
    t_total = 0.0
    for i, ctx in enumerate(ctxs):
        st = m.new_state()
        st.fill_kv(ctx)
        t0 = time.perf_counter()
        st.forward(1, ctx, True)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            t_total += dt
        del st
    value = args.steps / t_total
    return {
        "impl": "reference", "metric": "decode tokens/s (3B Q4_K_M, batch 256)" if big else
        "decode tokens/s (1B Q4_K_M, batch 64)" if args.workload == "ragged64" else "decode tokens/s (1B Q4_K_M, batch 1)",
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t_total / args.steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8xq4/q6 dp4a, fp32 accumulate, fp32 KV", "data": "synthetic (random-init weights, seeded)",
        "config": {"workload": "llama-3.2-3b Q4_K_M ragged decode, 256 seqs" if big else
                   "llama-3.2-1b Q4_K_M ragged decode, 64 seqs" if args.workload == "ragged64"
                   else "llama-3.2-1b Q4_K_M decode, batch 1", "parallelism": "host cores"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"one decode token per step of one sequence at the workload's context lengths "
                                   f"({args.steps} timed steps), oracle restatement of FastRunner::forward"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    args = parse()
    if args.impl == "reference":
        r = run_reference(args)
    else:
        r = run_ours(args)
    if r is not None:
        print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
