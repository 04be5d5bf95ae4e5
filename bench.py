#!/usr/bin/env python3
"""Decode-throughput benchmark of the B200 hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload ragged64|decode1]

Workloads (seeded synthetic inputs; random-init weights, no checkpoint):
  ragged64  Llama-3.2-1B-architecture Q4_K_M, 64 concurrent sequences, prompts
            U[16,1024], targets U[32,256]; finished sequences are replaced
            from the same distributions; paged fp16 KV, 16-token pages.  A
            step is one packed decode step over the 64 live sequences.
  decode1   same model, one sequence: 512-token prompt (ids U[0,128000),
            seed 1), then greedy decode steps.
  gemm_q6k_b64  the dominant kernel of ragged64 alone: the tensor-core
            quantised GEMM (+ its activation prep) on the 1B vocab
            projection, Q6_K 128256x2048, 64 tokens, through ijb_matvec.
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


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=48)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["ragged64", "decode1", "gemv_q4k", "gemv_q6k", "gemm_q6k_b64"],
                    default="ragged64")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--prompt", type=int, default=512, help="decode1 prompt length")
    ap.add_argument("--prompt-max", type=int, default=1024,
                    help="ragged64 longest prompt (1024 in the BASELINE config; smaller for profiling captures)")
    ap.add_argument("--nvtx-step", action="store_true",
                    help="wrap the last timed step in an NVTX range 'step' (ncu --nvtx-include step/)")
    return ap.parse_args()


# --------------------------------------------------------------- helpers --

def hbm_peak():
    try:
        with open(MEASURED_PEAKS) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every 50 ms from before the
    warm-up; only the samples that arrive inside the timed region (mark_start /
    mark_end) are reported."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int, interval_ms: int = 50, cmd=None):
        self.index = index
        self.interval_ms = interval_ms
        self.cmd = cmd
        self.rows = []  # (arrival time, fields)
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
                self.rows.append((time.perf_counter(), parts))

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
        rows = [r for t, r in self.rows if t0 <= t <= t1]
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[2 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "interval_ms": self.interval_ms}


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
    """64 live sequences; replaces finished ones from the request stream."""

    def __init__(self, eng, batch, seed, vocab_limit=128000, prompt_max=1024):
        self.eng = eng
        self.prompt_max = prompt_max
        self.batch = batch
        self.rng = np.random.default_rng(seed)
        self.vocab_limit = vocab_limit
        self.live = []  # [seq_id, next_token, generated, target]
        self.prefill_tokens = 0
        self.prefill_s = 0.0
        for _ in range(batch):
            self.live.append(self._admit())

    def _admit(self):
        plen = int(self.rng.integers(16, self.prompt_max + 1))
        target = int(self.rng.integers(32, 257))
        prompt = self.rng.integers(0, self.vocab_limit, size=plen).astype(np.int32)
        s = self.eng.seq_open()
        t0 = time.perf_counter()
        nxt = self.eng.seq_prefill(s, prompt)
        self.prefill_s += time.perf_counter() - t0
        self.prefill_tokens += plen
        return [s, nxt, 0, target]

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


GEMV_CASES = (("q4k_ffn_gate_8192x2048", 12, 8192, 2048), ("q6k_lm_head_128256x2048", 14, 128256, 2048))


def gemv_roofline(cuda, peak, cases=GEMV_CASES, iters_min=20):
    """Dominant kernel (gemv_kernel, the fused quantised GEMV) timed alone with
    CUDA events on its stream: the 1B ffn_gate Q4_K shape
    and the Q6_K lm_head (config 1), weights rotated over > 4x L2."""
    import torch
    L = ijblib.load()
    out = {}
    rng = np.random.default_rng(0)
    for name, qtype, rows, cols in cases:
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
        x = torch.randn(cols, device=cuda)
        y = torch.empty(rows, device=cuda)
        stream = torch.cuda.current_stream().cuda_stream
        for i in range(3 * copies):
            ijblib.check(L.ijb_gemv(qtype, ws[i % copies].data_ptr(), x.data_ptr(), y.data_ptr(), cols, rows, 1, 1,
                                    ctypes.c_void_p(stream)))
        iters = max(iters_min, 4 * copies)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        for i in range(iters):
            ijblib.check(L.ijb_gemv(qtype, ws[i % copies].data_ptr(), x.data_ptr(), y.data_ptr(), cols, rows, 1, 1,
                                    ctypes.c_void_p(stream)))
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / iters
        algo = nbytes + cols * 4 + rows * 4
        out[name] = {"us_per_launch": ms * 1e3, "algorithmic_bytes": algo, "gbs": algo / (ms * 1e-3) / 1e9,
                     "frac": algo / (ms * 1e-3) / 1e9 / peak, "rotated_copies": copies}
        del ws, wd
        torch.cuda.empty_cache()
    return out


# dram__bytes_read.sum + dram__bytes_write.sum of one mma_gemm_kernel launch of
# the gemm_q6k_b64 workload, from an ncu capture of that launch
MMA_VOCAB_TRAFFIC = 215909120 + 8392704


def mma_roofline(eng, cuda, peak, iters=20, batch=64):
    """The tensor-core GEMM timed alone with CUDA events on its stream: the
    vocab projection (Q6_K 128256x2048, the largest launch of a decode step)
    for `batch` tokens through ijb_matvec, each launch = activation prep +
    mma_gemm_kernel.  Algorithmic bytes: the Q6_K weights as stored (unit
    layout), the fp32 activations read and the fp32 logits written."""
    import torch
    L = ijblib.load()
    cfg = eng.cfg
    idx = eng.tensor_index("token_embd.weight")
    cols, rows = cfg.dim, cfg.vocab
    x = torch.randn(batch, cols, device=cuda)
    y = torch.empty(batch, rows, device=cuda)
    side = torch.cuda.Stream(device=cuda)  # a real stream handle (0 would mean the engine's own stream)
    stream = side.cuda_stream
    def launch():
        ijblib.check(L.ijb_matvec(eng.h, idx, x.data_ptr(), y.data_ptr(), cols, rows, batch, ctypes.c_void_p(stream)),
                     eng.h)
    torch.cuda.synchronize()
    with torch.cuda.stream(side):
        for _ in range(3):
            launch()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(side)
        for _ in range(iters):
            launch()
        b.record(side)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / iters
    w_bytes = rows * L.ijb_q6k_planar_row_bytes(cols)
    algo = w_bytes + batch * cols * 4 + batch * rows * 4
    gbs = algo / (ms * 1e-3) / 1e9
    return {"us_per_launch": ms * 1e3, "algorithmic_bytes": algo, "gbs": gbs, "frac": gbs / peak,
            "kernel": f"mma_gemm_kernel + activation prep (Q6_K {rows}x{cols} vocab projection, {batch} tokens)",
            "traffic": MMA_VOCAB_TRAFFIC}


def run_gemm(args):
    """The dominant kernel of ragged64 alone (see mma_roofline)."""
    import torch
    world, rank, local = dist_setup(args.gpus)
    cuda = torch.device(f"cuda:{local}")
    peak, src = hbm_peak()
    full = synth.LLAMA_1B
    cfg = synth.ModelConfig("llama-3.2-1b-1layer", dim=full.dim, layers=1, heads=full.heads,
                            kv_heads=full.kv_heads, hidden=full.hidden, vocab=full.vocab)
    from ijb200.engine import Engine
    eng = Engine(cfg, synth.make_model(cfg, seed=0), context=32, max_batch=64, device=local)
    r = mma_roofline(eng, cuda, peak, iters=max(args.steps, 5))
    eng.close()
    if rank != 0:
        return None
    return {"metric": "GEMM HBM GB/s (Q6_K 128256x2048 vocab projection, 64 tokens)", "value": r["gbs"],
            "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": 3, "ms_per_step": r["us_per_launch"] / 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp16 x fp16 (exact dequant, int8-path activations), fp32 accumulate",
            "data": "synthetic (seeded)", "config": {"workload": "gemm_q6k_b64", "l2": "weights 216 MB > L2"},
            "roofline": {"bound": "hbm", "achieved": r["gbs"], "peak": peak, "unit": "GB/s", "frac": r["frac"],
                         "traffic": r["traffic"], "kernel": r["kernel"], "peak_source": src}}


def cpu_baseline(cfg, weights, contexts, threads, budget_s=20.0):
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
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 dp4a x q4/q6",
            "data": "synthetic (seeded)", "config": {"workload": case[0], "rotated_copies": r["rotated_copies"]},
            "roofline": {"bound": "hbm", "achieved": r["gbs"], "peak": peak, "unit": "GB/s", "frac": r["frac"],
                         "traffic": None, "peak_source": src}}


def run_ours(args):
    import torch
    if args.workload.startswith("gemv"):
        return run_gemv(args)
    if args.workload == "gemm_q6k_b64":
        return run_gemm(args)
    world, rank, local = dist_setup(args.gpus)
    cuda = torch.device(f"cuda:{local}")
    peak, peak_src = hbm_peak()
    cfg = synth.LLAMA_1B
    t_setup = time.perf_counter()
    weights = synth.make_model(cfg, seed=0)
    from ijb200.engine import Engine
    if args.workload == "ragged64":
        batch, context = 64, 1024 + 256 + 16
        eng = Engine(cfg, weights, context=context, max_batch=batch, max_seqs=batch + 1, device=local)
        server = RaggedServer(eng, batch, seed=1000 + rank, prompt_max=args.prompt_max)
    else:
        batch, context = 1, args.prompt + 16 + args.steps + args.warmup + 8
        eng = Engine(cfg, weights, context=context, max_batch=1, max_seqs=2, device=local)
        prompt = synth.prompt_tokens(args.prompt, seed=1)
        nxt = eng.prefill(prompt)
        pos = len(prompt)
    setup_s = time.perf_counter() - t_setup

    def one_step():
        nonlocal nxt, pos
        if args.workload == "ragged64":
            return server.step()
        t0 = time.perf_counter()
        nxt = eng.forward(nxt, pos, True)
        wall = time.perf_counter() - t0
        pos += 1
        return 1, eng.last_step_ms(), wall, pos

    sampler = ClockSampler(local)
    sampler.start()
    # warm-up (includes graph capture)
    for _ in range(args.warmup):
        one_step()
        if args.workload == "ragged64":
            server.replace_finished()
    sampler.wait_first()
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
        if args.workload == "ragged64":
            t0 = time.perf_counter()
            server.replace_finished()
            replaced_s += time.perf_counter() - t0
    barrier(world)
    sampler.mark_end()
    region_s = time.perf_counter() - t_region
    launches = ijblib.load().ijb_kernel_launches() - launches0
    clocks = sampler.stop()

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
        kern = gemv_roofline(cuda, peak)
        dom = mma_roofline(eng, cuda, peak) if args.workload == "ragged64" else dict(
            kern["q6k_lm_head_128256x2048"], kernel="gemv_kernel (Q6_K lm_head 128256x2048, B=1)", traffic=None)
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            ctxs = ([int(c) for c in server.contexts()[:8]] if args.workload == "ragged64" else [pos] * 4)
            nthreads = os.cpu_count() or 1
            tps, used = cpu_baseline(cfg, weights, ctxs, nthreads)
            cpu = {"value": tps, "unit": "tokens/s", "cores": nthreads, "kind": "port",
                   "sample": f"oracle FastRunner::forward (INT8 path), one decode token at each context {used}, "
                             f"{nthreads} threads"}
        h2d = 4 * batch * 4  # token, seq, position, KV slot per entry (int32)
        result = {
            "metric": "decode tokens/s (1B Q4_K_M, batch 64)" if args.workload == "ragged64"
            else "decode tokens/s (1B Q4_K_M, batch 1)",
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8xq4/q6 dp4a, fp32 accumulate, fp16 KV", "data": "synthetic (random-init weights, seeded)",
            "config": {"workload": f"llama-3.2-1b Q4_K_M ragged decode, 64 seqs, prompts U[16,{args.prompt_max}], "
                                   "outputs U[32,256], replacement" if args.workload == "ragged64"
                       else f"llama-3.2-1b Q4_K_M decode, batch 1, {args.prompt}-token prompt",
                       "batch_per_gpu": batch, "page_size": 16, "kv": "fp16 paged",
                       "parallelism": f"replicas x{world}", "l2": "inputs larger than L2 (836 MB weights/step)",
                       "mean_context": kv_tokens / args.steps / batch},
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4 * batch},
            "gpu_launches": int(launches),
            "roofline": {"bound": "hbm", "achieved": dom["gbs"], "peak": peak, "unit": "GB/s",
                         "frac": dom["frac"], "traffic": dom["traffic"], "kernel": dom["kernel"],
                         "us_per_launch": dom["us_per_launch"], "peak_source": peak_src},
            "step_roofline": {"bytes_per_step": step_bytes, "achieved_gbs": step_gbs, "frac": step_gbs / peak},
            "gemv": kern,
            "cpu_baseline": cpu,
            "clocks": clocks,
            "setup_s": setup_s,
            "region_wall_s": region_s,
        }
        if args.workload == "ragged64":
            result["prefill"] = {"tokens": server.prefill_tokens, "seconds": server.prefill_s}
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
    import oracle as O
    cfg = synth.LLAMA_1B
    weights = synth.make_model(cfg, seed=0)
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    rng = np.random.default_rng(1000)
    if args.workload == "ragged64":
        # contexts of a steady ragged population: prompt U[16,1024] + generated so far
        ctxs = [int(rng.integers(16, 1025) + rng.integers(0, 257)) for _ in range(args.steps + args.warmup)]
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
        "impl": "reference", "metric": "decode tokens/s (1B Q4_K_M, batch 64)" if args.workload == "ragged64"
        else "decode tokens/s (1B Q4_K_M, batch 1)",
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t_total / args.steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8xq4/q6 dp4a, fp32 accumulate, fp32 KV", "data": "synthetic (random-init weights, seeded)",
        "config": {"workload": "llama-3.2-1b Q4_K_M ragged decode, 64 seqs" if args.workload == "ragged64"
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
