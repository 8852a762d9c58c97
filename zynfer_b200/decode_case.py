"""Decode microbenchmark: one fixed batch of sequences at one context length.

    python -m zynfer_b200.decode_case --seqs 32 --ctx 2048 --layers 2 --steps 3

Builds an int8 Qwen3-0.6B-shaped model (optionally with fewer layers, so a
profile of one layer's kernels holds only a few GB), prefills every sequence
with a seeded prompt of `ctx` tokens, warms the decode graph, then times
`steps` greedy steps on the device (CUDA events) and, in a second pass, every
kernel class with per-launch events. The steps run between
cudaProfilerStart/Stop, so a profiler started with `--profile-from-start off`
sees only the decode launches. Prints one JSON line.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import time

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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--seqs", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--path", default="auto", help="linear kernel family (auto, gemv, tcgen05, simt)")
    ap.add_argument("--schedule", default="auto", help="decode schedule (auto, kernels, persistent)")
    ap.add_argument("--phases", action="store_true",
                    help="persistent schedule: add the per-phase breakdown of CTA 0's phase trace (mean over layers)")
    ap.add_argument("--window", default="decode", choices=["decode", "prefill"],
                    help="what runs between cudaProfilerStart/Stop: the timed decode steps, or one more prefill")
    ap.add_argument("--weights", default="q8", choices=["q8", "bf16"])
    args = ap.parse_args()

    import torch

    from . import cuda as zc
    from . import workload

    arch = dataclasses.replace(zc.QWEN3_0_6B, layers=args.layers)
    B = args.seqs
    total = args.warmup + 2 * args.steps + 2
    gpu = zc.Gpu(0)
    wk = zc.W_Q8 if args.weights == "q8" else zc.W_BF16
    model = zc.Model(gpu, arch, wk, max_batch=B, max_seqs=B, max_seq_len=args.ctx + total + 16,
                     max_prefill=args.ctx)
    model.fill_synthetic(args.seed, 0.02, 0.0)
    gpu.set_linear_path(args.path)
    gpu.set_decode_schedule(args.schedule)
    first = [model.prefill(s, workload.prompt(s, args.ctx, args.seed), want_logits=False) for s in range(B)]
    if args.window == "prefill":
        gpu.sync()
        torch.cuda.profiler.start()
        t0 = time.perf_counter()
        first[0] = model.prefill(0, workload.prompt(0, args.ctx, args.seed), want_logits=False)
        gpu.sync()
        prefill_ms = (time.perf_counter() - t0) * 1e3
        torch.cuda.profiler.stop()
        print(json.dumps({"prefill_tokens": args.ctx, "layers": args.layers, "weights": args.weights,
                          "prefill_ms_wall": round(prefill_ms, 3)}), flush=True)
        gpu.close()
        return
    slots = list(range(B))
    out, _ = model.generate(slots, first, args.warmup)
    nxt = out[-1].tolist()
    gpu.sync()

    torch.cuda.profiler.start()
    out, ms = model.generate(slots, nxt, args.steps)
    torch.cuda.profiler.stop()
    nxt = out[-1].tolist()

    ctx = [model.seq_len(s) for s in slots]
    gpu.set_timing(True)
    model.generate(slots, nxt, args.steps)
    times = {name: gpu.kernel_time(cls) for name, cls in
             (("attention", zc.K_ATTN), ("linear", zc.K_LINEAR), ("lm_head", zc.K_LMHEAD), ("other", zc.K_OTHER))}
    phases = phase_breakdown(gpu.phase_trace(), args.layers) if args.phases and args.schedule == "persistent" else None
    gpu.set_timing(False)

    kv_tok = sum(sum(c + 1 + s for c in ctx) for s in range(args.steps)) / args.steps
    attn_bytes = kv_tok * KV_BYTES_PER_TOKEN_HEAD * arch.n_kv + B * 2 * arch.n_q * arch.head_dim * 4
    n_attn, ms_attn = times["attention"]
    line = {
        "seqs": B, "ctx": args.ctx, "layers": args.layers, "steps": args.steps, "path": args.path,
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


if __name__ == "__main__":
    main()
