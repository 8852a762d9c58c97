#!/usr/bin/env python3
"""Qwen3-0.6B int8 weight-only greedy decode throughput on N B200s.

Workload (the sharded batch configuration): 64 independent sequences, seeded
prompts of uniform length in [512, 4096], greedy decode, paged bf16 KV cache,
synthetic Qwen3-0.6B-shaped int8 weights (seeded normal(0, 0.02), norm weights
1.0). Sequences are split across the N GPUs (length-balanced, one process per
GPU, no collective on the hot path); total work is fixed, so scaling is
"strong". A step is one decode step of every sequence (64 tokens).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Timing: W untimed steps, then exactly K steps as on-device greedy generation
(CUDA graphs, argmax fed back on the device) between barrier + synchronize,
CUDA-event time on the library's stream, max over ranks. Each step reads the
0.6 GB of int8 weights and ~17 GB of KV cache, far above the 126 MB L2, so no
L2 flush is needed. `e2e` repeats the metric through the public C ABI call
zynfer_cu_decode_step with host token buffers (host->device inputs and the
device->host argmax inside the timed region). `roofline` comes from CUDA
events around every attention launch in an instrumented pass of the same
steps right after the timed region. `cpu_baseline` times the oracle
(the CPU restatement of the reference path) on a bounded sample.

    python bench.py --sweep gemv [--sweep-calls C] [--sweep-shape MxK]

prints one JSON line per case of the int8 linear sweep instead: matvecQ8 /
matmulQ8 (ops.zig:181-228) shapes 3072x1024 (QKV as 2048+512+512),
4096x1024 (the model's QKV, 2048+1024+1024), 1024x2048, 6144x1024, 1024x3072
and 151936x1024 at 1 and 8 activation rows, through zynfer_cu_linear with
device pointers. Each call reads another of R weight copies (R x m x k above
twice the L2), CUDA events around every call on the library's stream give
its time, and achieved GB/s = (m k + 4 m + 4 B k + 4 B m) / time.

At one GPU the line also carries three more workloads of the same model:
* "batch1" (one sequence, context 2048, 256 greedy tokens on the device):
  ms/token, tok/s and the fraction of the HBM roofline (weights + KV bytes
  per token / measured peak), with the argmax agreement of every timed token
  against the oracle (teacher-forced). The context is the seeded stand-in
  cache of zynfer_cu_kv_fill_synthetic (the oracle fills the same values):
  the same bytes and kernels as after a 2048-token prefill, without a CPU
  prefill.
* "prefill" (512 seeded tokens through a bf16-weight model, f32
  accumulate): ms per prefill from CUDA events, TFLOP/s of the algorithmic
  FLOPs against the measured bf16 peak, and the last-token logits of the
  reference tools' golden fixture prompt on the same kind of model.
* "linears" (the sweep's six shapes at 1 and 8 rows on the default kernel
  choice, 100 calls each): microseconds and GB/s per isolated call, and the
  oracle's single-thread time per call.

    python bench.py --case SEQS,CTX,LAYERS [--steps K] [--warmup W] [--schedule S]
                    [--path P] [--weights q8|bf16] [--window decode|prefill] [--phases]

times one fixed batch of SEQS sequences prefilled with CTX seeded tokens on
a model of LAYERS layers (a small case for profiler captures): K greedy steps
on the device, then per-kernel-class CUDA events; one JSON line.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Qwen3-0.6B int8 decode tok/s"
N_SEQS = 64
SEED = 20250601
KV_BYTES_PER_TOKEN_LAYER = 2 * 8 * 128 * 2  # K + V, 8 kv heads, d = 128, bf16
# Qwen3-0.6B int8 weights read per decode token: 28 x (QKV 4096x1024 + O
# 1024x2048 + gate/up 6144x1024 + down 1024x3072) int8, their f32 row scales,
# the four norm vectors per layer, the tied 151936x1024 LM head with its
# scales, and the final norm.
LINEAR_PARAMS_PER_LAYER = 4096 * 1024 + 1024 * 2048 + 6144 * 1024 + 1024 * 3072
WEIGHT_BYTES_PER_TOKEN = (28 * (LINEAR_PARAMS_PER_LAYER + 4 * (4096 + 1024 + 6144 + 1024) + 4 * (2 * 1024 + 2 * 128))
                          + 151936 * 1024 + 4 * 151936 + 4 * 1024)
BATCH1_CTX, BATCH1_STEPS = 2048, 256
PREFILL_T = 512
GOLDEN_SEED = 20251201
# An argmax differs from the oracle's only at a near tie: the oracle's top two
# logits within this bound (the stated bf16-KV logit tolerance of the tests).
ARGMAX_TIE = 1.5e-2
# DRAM bytes (read + write) per algorithmic byte of attn_decode_kernel, from one
# ncu capture of 32 sequences at context 2048 (profiles/attn_decode_b32_ctx2048.txt:
# 275.1 MB for 269.3 MB); the traffic grows with the KV bytes, so a launch of this
# workload moves about this ratio times its algorithmic bytes.
ATTN_TRAFFIC_RATIO = 275.06 / 269.3


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=120)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=16)
    ap.add_argument("--profile-steps", type=int, default=4)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sweep", choices=["gemv"], default=None)
    ap.add_argument("--sweep-calls", type=int, default=200)
    ap.add_argument("--sweep-shape", default=None, help="one shape of the sweep, as MxK")
    ap.add_argument("--no-batch1", action="store_true", help="skip the one-sequence context-2048 workload")
    ap.add_argument("--no-prefill", action="store_true", help="skip the 512-token bf16 prefill workload")
    ap.add_argument("--no-linears", action="store_true", help="skip the int8 linear sweep at 1 and 8 rows")
    ap.add_argument("--batch1-steps", type=int, default=BATCH1_STEPS)
    ap.add_argument("--case", default=None, help="SEQS,CTX,LAYERS: one fixed decode batch (profiling case)")
    ap.add_argument("--schedule", default="auto", help="--case: decode schedule (auto, kernels, persistent)")
    ap.add_argument("--path", default="auto", help="--case: linear kernel family (auto, gemv, mma, tcgen05, simt)")
    ap.add_argument("--weights", default="q8", choices=["q8", "bf16"], help="--case: weight storage")
    ap.add_argument("--window", default="decode", choices=["decode", "prefill"],
                    help="--case: what runs between cudaProfilerStart/Stop")
    ap.add_argument("--kv-f32", action="store_true",
                    help="--case: prefill attention over f32 K/V (the benchmark's prefill), not the cache's bf16 values")
    ap.add_argument("--phases", action="store_true",
                    help="--case with the persistent schedule: per-phase times from CTA 0's phase trace")
    return ap.parse_args()


def env_rank():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def measured_peak_tflops():
    """Burst bf16 tensor peak (a prefill is timed alone): measured, else the fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled while the timed
    region runs: NVML polled every 2 ms from a host thread (so even a
    30 ms region yields samples), nvidia-smi as the fallback. Read-only."""
    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.samples: list[tuple[float, float, set]] = []
        self.nvml = None
        self.proc = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.handle = pynvml.nvmlDeviceGetHandleByUUID(gpu_id)
            self.max_sm = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
            self.nvml = pynvml
        except Exception:
            self.nvml = None

    def _poll_nvml(self):
        p = self.nvml
        bits = [(name, getattr(p, attr, 0)) for name, attr in self.REASONS]
        while not self._stop.is_set():
            try:
                sm = float(p.nvmlDeviceGetClockInfo(self.handle, p.NVML_CLOCK_SM))
                r = p.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.samples.append((sm, self.max_sm, {name for name, b in bits if b and r & b}))
            except Exception:
                pass
            time.sleep(0.002)

    def _read_smi(self):
        names = [n for n, _ in self.REASONS]
        for ln in self.proc.stdout:
            f = [x.strip() for x in ln.strip().split(",")]
            if len(f) < 9:
                continue
            try:
                self.samples.append((float(f[1]), float(f[2]),
                                     {n for n, v in zip(names, f[5:9]) if v.lower() == "active"}))
            except ValueError:
                continue

    def start(self):
        if self.nvml:
            self._t = threading.Thread(target=self._poll_nvml, daemon=True)
            self._t.start()
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", self.gpu_id], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read_smi, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None

    def stop(self):
        if self.nvml:
            self._stop.set()
            self._t.join(timeout=2)
            source = "nvml"
        elif self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self._t.join(timeout=2)
            source = "nvidia-smi"
        else:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock source"], "samples": 0}
        sm = [x[0] for x in self.samples]
        reasons = set().union(*[x[2] for x in self.samples]) if self.samples else set()
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(x[1] for x in self.samples) if self.samples else None,
                "reasons": sorted(reasons), "samples": len(sm), "source": source}


def oracle_model(threads: int):
    """The oracle's int8 Qwen3-0.6B on the benchmark's seeded weights."""
    from oracle import oracle as O
    return O.Model(O.QWEN3_0_6B, O.W_Q8, kv_bf16=True, seed=SEED, w_std=0.02, norm_std=0.0, threads=threads)


def cpu_baseline(mean_ctx: int, n_seqs: int, steps: int, threads: int, warmup: int = 1, m=None):
    """Oracle int8 decode (the reference path restated in C, all host threads
    splitting each matvec's rows) on n_seqs sequences at context mean_ctx,
    whose caches are filled with seeded values instead of a CPU prefill."""
    own = m is None
    if own:
        m = oracle_model(threads)
    m.set_threads(threads)
    sessions = []
    for i in range(n_seqs):
        s = m.session(mean_ctx + steps + warmup + 2)
        s.fill_kv(mean_ctx, SEED + i)
        sessions.append(s)
    tok = [1 + i for i in range(n_seqs)]
    for _ in range(warmup):
        for i, s in enumerate(sessions):
            tok[i] = int(s.greedy(tok[i], 1)[0])
    t0 = time.perf_counter()
    for _ in range(steps):
        for i, s in enumerate(sessions):
            tok[i] = int(s.greedy(tok[i], 1)[0])
    dt = time.perf_counter() - t0
    for s in sessions:
        s.close()
    if own:
        m.close()
    return n_seqs * steps / dt, dt


def run_reference(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return
    from zynfer_b200 import workload
    lens = workload.prompt_lengths(N_SEQS, SEED)
    mean_ctx = int(round(sum(lens) / len(lens)))
    threads = os.cpu_count() or 1
    n_sample = 2 if args.steps + args.warmup <= 200 else 1
    value, dt = cpu_baseline(mean_ctx, n_sample, args.steps, threads, warmup=args.warmup)
    sample = (f"{n_sample} sequences x {args.steps} greedy steps at context {mean_ctx} "
              f"(mean prompt of the 64-sequence workload; caches seeded, no CPU prefill)")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * dt / args.steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "qwen3-0.6b int8 weight-only greedy decode, 64 seqs, prompts U[512,4096]",
                   "model": "Qwen3-0.6B-shaped (random init)", "global_batch": N_SEQS, "seq_len": mean_ctx,
                   "parallelism": "host threads split each matvec's output rows"},
        "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_batch1(model, gpu, oracle, slot: int, steps: int, warmup: int, peak: float):
    """One sequence at context 2048, `steps` greedy tokens on the device (the
    one-row GEMV graph), timed with CUDA events; then the oracle, fed the
    GPU's tokens, checks every timed argmax (a flip only at a near tie)."""
    import numpy as np

    TIE = ARGMAX_TIE
    first = 4242
    model.kv_fill_synthetic(slot, BATCH1_CTX, SEED)
    model.generate([slot], [first], warmup)                 # captures the batch-1 graph
    model.kv_fill_synthetic(slot, BATCH1_CTX, SEED)         # back to context 2048
    out, ms = model.generate([slot], [first], steps)
    path = gpu.last_path
    ids = out[:, 0]
    agree = near_ties = 0
    if oracle is not None:
        s = oracle.session(BATCH1_CTX + steps + 2)
        s.fill_kv(BATCH1_CTX, SEED)
        _, logits = s.greedy(first, steps, teacher=ids, want_logits=True)
        s.close()
        for i in range(steps):
            if int(np.argmax(logits[i])) == int(ids[i]):
                agree += 1
            else:
                top2 = np.sort(logits[i])[-2:]
                if top2[1] - top2[0] <= TIE and logits[i][int(ids[i])] >= top2[1] - TIE:
                    near_ties += 1
    mean_kv = BATCH1_CTX + (steps + 1) / 2.0                 # step i reads 2048 + i + 1 positions
    bytes_tok = WEIGHT_BYTES_PER_TOKEN + mean_kv * 28 * KV_BYTES_PER_TOKEN_LAYER
    ms_tok = ms / steps
    gbs = bytes_tok / (ms_tok / 1e3) / 1e9
    return {"workload": f"one sequence, context {BATCH1_CTX}, {steps} greedy tokens (int8 weights, bf16 KV)",
            "ms_per_token": round(ms_tok, 4), "tok_s": round(1e3 / ms_tok, 1),
            "roofline": {"bound": "hbm", "bytes_per_token": int(bytes_tok), "achieved": round(gbs, 1),
                         "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 4)},
            "argmax_vs_oracle": None if oracle is None else
            {"tokens": steps, "equal": agree, "near_tie_flips": near_ties, "mismatch": steps - agree - near_ties},
            "context_source": "seeded stand-in cache of 2048 positions (zynfer_cu_kv_fill_synthetic; the "
                              "oracle fills the same bf16 values)",
            "path": path}


def prefill_flops(T: int) -> float:
    """Algorithmic FLOPs of a T-token prefill: every linear of every layer on
    T rows, causal attention (QK and PV per visible pair), LM head on the last row."""
    linear = 2.0 * 28 * LINEAR_PARAMS_PER_LAYER * T
    attn = 28 * 16 * (T * (T + 1) / 2) * 128 * 4
    return linear + attn + 2.0 * 151936 * 1024


def run_prefill(local: int, runs: int = 5):
    """512 seeded tokens through a bf16-weight Qwen3-0.6B (f32 accumulate),
    CUDA-event time per prefill (median of `runs`), and the golden fixture."""
    import numpy as np

    from zynfer_b200 import cuda as zc
    from zynfer_b200 import workload
    gpu = zc.Gpu(local)
    try:
        m = zc.Model(gpu, zc.QWEN3_0_6B, zc.W_BF16, max_batch=1, max_seqs=1, max_seq_len=PREFILL_T,
                     max_prefill=PREFILL_T, prefill_kv_f32=True)
        m.fill_synthetic(GOLDEN_SEED, 0.02, 0.1)
        ids = workload.tokens(PREFILL_T, SEED, 3)
        for _ in range(2):
            m.prefill(0, ids, want_logits=False)
        times = []
        for _ in range(runs):
            m.prefill(0, ids, want_logits=False)
            times.append(gpu.last_step_ns / 1e6)
        path = gpu.last_path
        ms = statistics.median(times)
        g = np.load(os.path.join(ROOT, "tests", "golden", "qwen3_bf16_bos23.npz"))
        logits, _ = m.prefill(0, g["tokens"])
        err = max(float(np.max(np.abs(g["np_sample_vals"] - logits[g["np_sample_idx"]]))),
                  float(np.max(np.abs(g["np_top_vals"] - logits[g["np_top_ids"]]))))
    finally:
        gpu.close()
    flops = prefill_flops(PREFILL_T)
    tf = flops / (ms / 1e3) / 1e12
    peak, kind = measured_peak_tflops()
    return {"workload": f"{PREFILL_T}-token prefill, bf16 weights, f32 accumulate, last-token logits",
            "ms": round(ms, 4), "runs_ms": [round(t, 4) for t in times],
            "roofline": {"bound": "tensor", "flops": flops, "achieved": round(tf, 1), "peak": peak,
                         "peak_kind": kind, "unit": "TFLOP/s", "frac": round(tf / peak, 4)},
            "golden_fixture": {"prompt": [int(t) for t in g["tokens"]], "max_abs_vs_reference_numpy": err,
                               "bound": 2e-3, "ok": err <= 2e-3},
            "path": path}


def run_ours(args):
    import torch
    import torch.distributed as dist

    from zynfer_b200 import cuda as zc
    from zynfer_b200 import shard, workload

    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)

    def barrier():
        if world > 1:
            dist.barrier()

    lens = workload.prompt_lengths(N_SEQS, SEED)
    total_steps = args.warmup + args.steps + args.e2e_steps + args.profile_steps
    mine = shard.assign_sequences(lens, world, total_steps)[rank]
    B = len(mine)
    max_len = max(max(lens[i] for i in mine) + total_steps + 16, BATCH1_CTX + args.batch1_steps + 64)
    gpu = zc.Gpu(local)
    model = zc.Model(gpu, zc.QWEN3_0_6B, zc.W_Q8, max_batch=B, max_seqs=B, max_seq_len=max_len,
                     max_prefill=4096)
    model.fill_synthetic(SEED, 0.02, 0.0)
    t0 = time.perf_counter()
    first = []
    for slot, i in enumerate(mine):
        first.append(model.prefill(slot, workload.prompt(i, lens[i], SEED), want_logits=False))
    prefill_s = time.perf_counter() - t0
    slots = list(range(B))

    # warm-up (also captures the decode graph for this batch size)
    out, _ = model.generate(slots, first, args.warmup)
    nxt = out[-1].tolist()
    ctx_before = [model.seq_len(s) for s in slots]

    props = torch.cuda.get_device_properties(local)
    clocks = ClockSampler("GPU-" + str(props.uuid) if hasattr(props, "uuid") else str(local))
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    torch.cuda.profiler.start()  # a profiler run with --profile-from-start off sees the timed steps only
    out, dev_ms = model.generate(slots, nxt, args.steps)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    clk = clocks.stop()
    timed_path = gpu.last_path  # the kernels of the timed steps (the graph), before any instrumented pass
    barrier()
    nxt = out[-1].tolist()
    t_max = shard.max_over_ranks(dev_ms, dev)
    tokens = N_SEQS * args.steps
    value = tokens / (t_max / 1e3)
    launches = gpu.step_launches * args.steps

    # e2e through the public C ABI: host tokens in, argmax out, every step
    gpu.io_bytes(reset=True)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        nxt = model.decode_step(slots, nxt).tolist()
    e2e_s = time.perf_counter() - t0
    barrier()
    h2d, d2h = gpu.io_bytes(reset=True)
    e2e_max = shard.max_over_ranks(e2e_s, dev)
    h2d_all = shard.sum_over_ranks(h2d, dev) / max(1, args.e2e_steps)
    d2h_all = shard.sum_over_ranks(d2h, dev) / max(1, args.e2e_steps)
    e2e_value = N_SEQS * args.e2e_steps / e2e_max

    # instrumented pass: CUDA events around every kernel class
    ctx_prof = [model.seq_len(s) for s in slots]
    gpu.set_timing(True)
    model.generate(slots, nxt, args.profile_steps)
    n_attn, ms_attn = gpu.kernel_time(zc.K_ATTN)
    n_lin, ms_lin = gpu.kernel_time(zc.K_LINEAR)
    n_lm, ms_lm = gpu.kernel_time(zc.K_LMHEAD)
    n_oth, ms_oth = gpu.kernel_time(zc.K_OTHER)
    gpu.set_timing(False)
    # algorithmic bytes per attention launch (one layer): K+V of every cached
    # position (bf16) + q in and attention out (f32), averaged over the pass
    kv_tok = sum(sum(c + 1 + s for c in ctx_prof) for s in range(args.profile_steps)) / args.profile_steps
    attn_bytes = kv_tok * KV_BYTES_PER_TOKEN_LAYER + B * 2 * 2048 * 4
    attn_avg_ms = ms_attn / max(1, n_attn)
    achieved = attn_bytes / (attn_avg_ms / 1e3) / 1e9
    peak, peak_kind = measured_peaks()
    achieved_all = shard.sum_over_ranks(achieved, dev) / world
    per_step = lambda v: round(v / args.profile_steps, 4)  # noqa: E731
    mine_row = [float(B), dev_ms / args.steps, ms_attn / args.profile_steps, ms_lin / args.profile_steps,
                ms_lm / args.profile_steps, float(sum(ctx_before)) / max(1, B)]
    rows = shard.gather_over_ranks(mine_row, dev)

    cpu = batch1 = prefill = None
    oracle = None
    if rank == 0 and world == 1 and not (args.no_cpu_baseline and args.no_batch1):
        oracle = oracle_model(os.cpu_count() or 1)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        mean_ctx = int(round(sum(ctx_before) / len(ctx_before)))
        threads = os.cpu_count() or 1
        v, dt = cpu_baseline(mean_ctx, 2, 12, threads, m=oracle)
        v1, dt1 = cpu_baseline(mean_ctx, 1, 3, 1, m=oracle)
        cpu = {"value": round(v, 4), "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"2 sequences x 12 greedy steps at context {mean_ctx} (caches seeded, no CPU prefill)",
               "single_thread": {"value": round(v1, 4), "unit": "tok/s", "cores": 1,
                                 "sample": f"1 sequence x 3 greedy steps at context {mean_ctx}"}}
    if rank == 0 and world == 1 and not args.no_batch1:
        batch1 = run_batch1(model, gpu, oracle, 0, args.batch1_steps, max(3, args.warmup), peak)
    if oracle is not None:
        oracle.set_threads(1)
        oracle.close()
    if rank == 0 and world == 1 and not args.no_prefill:
        prefill = run_prefill(local)
    linears = run_linears(gpu) if rank == 0 and world == 1 and not args.no_linears else None

    if rank == 0:
        mean_ctx = sum(ctx_before) / len(ctx_before)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_max / args.steps, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "weights": "int8 per-row scale", "data": "synthetic",
            "config": {"workload": "qwen3-0.6b int8 weight-only greedy decode, 64 seqs, prompts U[512,4096], "
                                   "paged bf16 KV",
                       "model": "Qwen3-0.6B-shaped (random init)", "global_batch": N_SEQS,
                       "per_gpu_batch": B, "seq_len": round(mean_ctx, 1),
                       "parallelism": f"dp{world} (independent sequences, no collective)",
                       "l2": "per-step bytes (~0.6 GB weights + ~17 GB KV) far exceed the 126 MB L2"},
            "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": int(h2d_all),
                    "d2h_bytes_per_step": int(d2h_all), "steps": args.e2e_steps},
            "roofline": {"bound": "hbm", "kernel": "attn_decode_kernel", "achieved": round(achieved_all, 1),
                         "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(achieved_all / peak, 4),
                         "traffic": int(ATTN_TRAFFIC_RATIO * attn_bytes),
                         "traffic_source": "ncu dram read+write of a 32-sequence, context-2048 launch, "
                                           "scaled by KV bytes",
                         "bytes_per_launch": int(attn_bytes), "avg_launch_ms": round(attn_avg_ms, 5),
                         "launches_timed": n_attn,
                         "note": "CUDA events around each attention launch in an instrumented pass of "
                                 f"{args.profile_steps} steps right after the timed region"},
            "kernel_ms_per_step": {"attention": per_step(ms_attn), "linear": per_step(ms_lin),
                                   "lm_head": per_step(ms_lm), "other": per_step(ms_oth)},
            "per_rank": [{"rank": r, "batch": int(row[0]), "ms_per_step": round(row[1], 4),
                          "attention_ms": round(row[2], 4), "linear_ms": round(row[3], 4),
                          "lm_head_ms": round(row[4], 4), "mean_context": round(row[5], 1)}
                         for r, row in enumerate(rows)],
            "cpu_baseline": cpu,
            "clocks": clk, "gpu_launches": launches, "prefill_s": round(prefill_s, 2),
            "path": timed_path,
        }
        if batch1 is not None:
            line["batch1"] = batch1
        if prefill is not None:
            line["prefill"] = prefill
        if linears is not None:
            line["linears"] = linears
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    gpu.close()


KV_BYTES_PER_TOKEN_HEAD = 2 * 128 * 2  # K and V rows, bf16


def phase_breakdown(trace, layers: int) -> dict:
    """Mean per-layer microseconds of each phase of the last persistent step,
    as seen by CTA 0: "work" runs from the phase's start (its input staged)
    to its end (its outputs written), "wait" from its end to the next
    phase's start (the other CTAs' outputs arriving)."""
    import numpy as np

    t = trace.astype(np.int64)
    P = 5 * layers + 1
    if t.size < 4 + 10 * layers:
        return {}
    st, en = t[1:2 * P:2], t[2:2 * P + 1:2]
    nxt = np.append(st[1:], t[3 + 2 * (P - 1)])
    out = {}
    for k, name in enumerate(("qkv", "attention", "o", "gate_up", "down")):
        idx = np.arange(k, 5 * layers, 5)
        out[name] = {"work": round(float(np.mean(en[idx] - st[idx])) / 1e3, 2),
                     "wait": round(float(np.mean(nxt[idx] - en[idx])) / 1e3, 2)}
    out["lm_head"] = {"work": round(float(en[-1] - st[-1]) / 1e3, 2),
                      "finish": round(float(t[3 + 2 * (P - 1)] - en[-1]) / 1e3, 2)}
    return out


def run_case(args):
    """One fixed decode batch: SEQS sequences prefilled with CTX seeded tokens
    on a model of LAYERS layers (fewer layers keep a profiler capture of one
    layer's kernels to a few GB). Times `steps` greedy steps on the device,
    then every kernel class with per-launch events. The timed steps (or, with
    --window prefill, one more prefill) run between cudaProfilerStart/Stop,
    so a profiler started with --profile-from-start off sees only them."""
    import dataclasses

    import torch

    from zynfer_b200 import cuda as zc
    from zynfer_b200 import workload

    seqs, ctx, layers = (int(v) for v in args.case.split(","))
    arch = dataclasses.replace(zc.QWEN3_0_6B, layers=layers)
    B = seqs
    total = args.warmup + 2 * args.steps + 2
    gpu = zc.Gpu(0)
    wk = zc.W_Q8 if args.weights == "q8" else zc.W_BF16
    model = zc.Model(gpu, arch, wk, max_batch=B, max_seqs=B, max_seq_len=ctx + total + 16, max_prefill=ctx,
                     prefill_kv_f32=args.kv_f32)
    model.fill_synthetic(1, 0.02, 0.0)
    gpu.set_linear_path(args.path)
    gpu.set_decode_schedule(args.schedule)
    first = [model.prefill(s, workload.prompt(s, ctx, 1), want_logits=False) for s in range(B)]
    if args.window == "prefill":
        gpu.sync()
        torch.cuda.profiler.start()
        first[0] = model.prefill(0, workload.prompt(0, ctx, 1), want_logits=False)
        gpu.sync()
        torch.cuda.profiler.stop()
        print(json.dumps({"prefill_tokens": ctx, "layers": layers, "weights": args.weights,
                          "prefill_ms": round(gpu.last_step_ns / 1e6, 4), "path": gpu.last_path}), flush=True)
        gpu.close()
        return
    slots = list(range(B))
    out, _ = model.generate(slots, first, args.warmup)
    nxt = out[-1].tolist()
    gpu.sync()

    torch.cuda.profiler.start()
    out, ms = model.generate(slots, nxt, args.steps)
    torch.cuda.profiler.stop()
    path = gpu.last_path
    nxt = out[-1].tolist()

    ctxs = [model.seq_len(s) for s in slots]
    gpu.set_timing(True)
    model.generate(slots, nxt, args.steps)
    times = {name: gpu.kernel_time(cls) for name, cls in
             (("attention", zc.K_ATTN), ("linear", zc.K_LINEAR), ("lm_head", zc.K_LMHEAD), ("other", zc.K_OTHER))}
    phases = phase_breakdown(gpu.phase_trace(), layers) if args.phases and args.schedule == "persistent" else None
    gpu.set_timing(False)

    kv_tok = sum(sum(c + 1 + s for c in ctxs) for s in range(args.steps)) / args.steps
    attn_bytes = kv_tok * KV_BYTES_PER_TOKEN_HEAD * arch.n_kv + B * 2 * arch.n_q * arch.head_dim * 4
    n_attn, ms_attn = times["attention"]
    line = {
        "seqs": B, "ctx": ctx, "layers": layers, "steps": args.steps, "path": path,
        "ms_per_step": round(ms / args.steps, 4), "tok_s": round(B * args.steps / (ms / 1e3), 1),
        "launches_per_step": gpu.step_launches,
        "kernel_ms_per_step": {k: round(v[1] / args.steps, 4) for k, v in times.items()},
        "launches": {k: v[0] for k, v in times.items()},
        "attn_bytes_per_launch": int(attn_bytes),
        "attn_gbs": round(attn_bytes / (ms_attn / max(1, n_attn) / 1e3) / 1e9, 1) if n_attn else None,
    }
    if phases:
        line["phases_us"] = phases
    print(json.dumps(line), flush=True)
    gpu.close()


GEMV_SHAPES = [(3072, 1024), (4096, 1024), (1024, 2048), (6144, 1024), (1024, 3072), (151936, 1024)]
L2_BYTES = 126 * 2**20


def cpu_linear_us(m: int, k: int, batch: int, budget_s: float = 1.0) -> float:
    """Oracle matvecQ8 (one row) / matmulQ8 (batch columns), one host thread,
    microseconds per call over a bounded number of calls."""
    import numpy as np
    from oracle import oracle as O
    rng = np.random.default_rng(SEED)
    q = rng.integers(-127, 128, size=(m, k), dtype=np.int8)
    s = rng.random(m, dtype=np.float32) * np.float32(0.01)
    x = rng.standard_normal((k,) if batch == 1 else (k, batch)).astype(np.float32)
    calls, t0 = 0, time.perf_counter()
    while True:
        if batch == 1:
            O.matvec_q8(q, s, x)
        else:
            O.matmul_q8(q, s, x)
        calls += 1
        dt = time.perf_counter() - t0
        if dt > budget_s or calls >= 20:
            return dt / calls * 1e6


def linear_sweep(gpu, calls: int, shapes, paths_b8=("auto", "gemv", "mma", "tcgen05"), cpu_budget_s: float = 1.0):
    """Yield one record per (shape, rows, linear path) of the int8 linear sweep
    on an open context (device pointers through zynfer_cu_linear)."""
    import torch
    from zynfer_b200 import cuda as zc
    peak, peak_kind = measured_peaks()
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(SEED)
    for (m, k) in shapes:
        copies = max(2, -(-2 * L2_BYTES // (m * k)))
        w = torch.randint(-127, 128, (copies, m, k), dtype=torch.int8, device=dev, generator=g)
        sc = torch.rand((copies, m), device=dev, generator=g) * 0.01
        cpu_us = {}
        for batch in (1, 8):
            x = torch.randn((batch, k), device=dev, generator=g)
            y = torch.empty((batch, m), device=dev)
            ref = (x @ w[0].float().t()) * sc[0]
            for path in (("auto",) if batch == 1 else paths_b8):
                gpu.set_linear_path(path)
                for i in range(copies):  # warm-up: tensor maps, scratch
                    gpu.linear(zc.W_Q8, w[i], sc[i], x, batch, m, k, y)
                gpu.sync()
                gpu.linear(zc.W_Q8, w[0], sc[0], x, batch, m, k, y)
                gpu.sync()
                err = float(((y - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item())
                n_calls = max(calls, 2 * copies)
                gpu.set_timing(True)
                for i in range(n_calls):
                    gpu.linear(zc.W_Q8, w[i % copies], sc[i % copies], x, batch, m, k, y)
                n, ms = gpu.kernel_time(zc.K_LINEAR)
                gpu.set_timing(False)
                us = ms / max(1, n) * 1e3
                nbytes = m * k + 4 * m + 4 * batch * k + 4 * batch * m
                gbs = nbytes / (us * 1e-6) / 1e9
                if batch not in cpu_us:
                    cpu_us[batch] = cpu_linear_us(m, k, batch, cpu_budget_s)
                yield {
                    "sweep": "gemv", "m": m, "k": k, "batch": batch, "path": path, "kernel_path": gpu.last_path,
                    "us_per_call": round(us, 3), "bytes_per_call": nbytes, "achieved_gbs": round(gbs, 1),
                    "peak_gbs": peak, "peak_kind": peak_kind, "frac": round(gbs / peak, 4),
                    "rotation_copies": copies, "calls": n, "max_rel_err_vs_torch_f32": err,
                    "cpu_us_per_call": round(cpu_us[batch], 1), "cpu_threads": 1,
                    "cpu_kind": "port (oracle matvecQ8 / matmulQ8)"}
        del w, sc
        torch.cuda.empty_cache()
    gpu.set_linear_path("auto")


def run_linears(gpu) -> dict:
    """The int8 linear sweep's shapes at 1 and 8 rows on the default kernel
    choice, compactly, for the benchmark line."""
    cases = []
    for r in linear_sweep(gpu, 100, GEMV_SHAPES, paths_b8=("auto",), cpu_budget_s=0.5):
        cases.append({"m": r["m"], "k": r["k"], "rows": r["batch"], "kernel_path": r["kernel_path"],
                      "us_per_call": r["us_per_call"], "achieved_gbs": r["achieved_gbs"], "frac": r["frac"],
                      "max_rel_err_vs_torch_f32": r["max_rel_err_vs_torch_f32"],
                      "cpu_us_per_call": r["cpu_us_per_call"]})
    return {"workload": "matvecQ8 / matmulQ8 shapes of the model at 1 and 8 activation rows, one isolated call "
                        "each, weights rotated over copies larger than twice the L2",
            "bytes_per_call": "m k + 4 m + 4 rows k + 4 rows m", "cpu": "oracle, 1 host thread",
            "cases": cases}


def run_gemv_sweep(args):
    from zynfer_b200 import cuda as zc
    gpu = zc.Gpu(0)
    shapes = GEMV_SHAPES
    if args.sweep_shape:
        shapes = [tuple(int(v) for v in args.sweep_shape.lower().split("x"))]
    for rec in linear_sweep(gpu, args.sweep_calls, shapes):
        print(json.dumps(rec), flush=True)
    gpu.close()


def main():
    args = parse()
    if args.sweep == "gemv":
        run_gemv_sweep(args)
        return
    if args.case:
        run_case(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
