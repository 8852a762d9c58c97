"""Command line of the `cuda` backend: the reference's commands that reach it.

    python -m zynfer_b200.cli backends
    python -m zynfer_b200.cli forward-golden MODEL.zynfer [--tokens 151643,2,3] [--golden LOGITS.f32] [--backend cuda]
    python -m zynfer_b200.cli decode-bench [--backend cuda] [--artifact MODEL.zynfer] [--batch B] [--prefill-tokens T]
                                           [--decode-steps S] [--warmup W] [--iters I]

`--backend` (else ZYNFER_BACKEND, else the default kind) resolves through the
reference's rules (src/main.zig:58-64,110-114; backend.zig:106-130, mirrored in
zynfer_b200/backend.py): an unknown name fails, and a kind this build does not
have fails too; there is no CPU fallback.

forward-golden follows runForwardGolden (main.zig:412-505): prefill the tokens
(default: bos, 2, 3) on a model loaded from the artifact, compare the last
row's logits with a golden f32 file under compare.zig's rule (atol 1e-3,
rtol 1e-2) and print the top 8 (topK, qwen_forward.zig:177-193). The per-layer
--dump of the CPU path is not available here (the cuda path keeps no per-layer
host copies) and is rejected.

decode-bench prints block-bench's report (main.zig:1150-1245) for the
Qwen3-shaped decode on the device: prefill time of `prefill_tokens` and decode
ns/token over `decode_steps` greedy steps, then "json" and one line with
block-bench's keys (backend, fixture, hidden, prefill_tokens, decode_steps,
warmup, iters, metal_init_ns, peak_rss_bytes, energy_per_token,
cpu_prefill_ns, cpu_decode_ns_per_token, apple_prefill_ns,
apple_decode_ns_per_token, apple_block_path) plus this backend's cuda_* keys.
Keys of backends that did not run are null, as block-bench prints them.
"""
from __future__ import annotations

import argparse
import json
import os
import resource
import sys
import time

import numpy as np

from . import backend

BLOCK_BENCH_KEYS = ("backend", "fixture", "hidden", "prefill_tokens", "decode_steps", "warmup", "iters",
                    "metal_init_ns", "peak_rss_bytes", "energy_per_token", "cpu_prefill_ns",
                    "cpu_decode_ns_per_token", "apple_prefill_ns", "apple_decode_ns_per_token", "apple_block_path")
CUDA_KEYS = ("cuda_init_ns", "cuda_prefill_ns", "cuda_decode_ns_per_token", "cuda_block_path", "cuda_batch",
             "cuda_launches_per_step")


class CliError(SystemExit):
    """Exit status 2 with a message on stderr (the reference's usage/failure exits)."""

    def __init__(self, msg: str):
        sys.stderr.write(msg.rstrip() + "\n")
        super().__init__(2)


def resolve(flag: str | None) -> backend.BackendKind:
    try:
        kind = backend.resolve_kind(flag)
    except backend.UnknownBackend as e:
        raise CliError(str(e))
    except backend.BackendUnavailable as e:
        raise CliError(str(e))
    if kind is not backend.BackendKind.cuda:
        raise CliError(f"backend {kind.value} is not part of this build (only cuda is)")
    return kind


def parse_tokens(text: str) -> list[int]:
    """parseTokenIds (main.zig): comma-separated ids."""
    try:
        ids = [int(t) for t in text.split(",") if t.strip()]
    except ValueError:
        raise CliError(f"bad --tokens: {text}")
    if not ids:
        raise CliError("--tokens is empty")
    return ids


def expect_close(expected: np.ndarray, actual: np.ndarray, atol: float, rtol: float) -> tuple[bool, float, int]:
    """compare.zig:14-59: the largest |a - e| (last index on ties) within atol + rtol |e| there."""
    d = np.abs(actual.astype(np.float64) - expected.astype(np.float64))
    idx = int(d.size - 1 - np.argmax(d[::-1]))
    ok = bool(d[idx] <= atol + rtol * abs(float(expected[idx])))
    return ok, float(d[idx]), idx


def top_k(logits: np.ndarray, k: int = 8) -> list[tuple[int, float]]:
    """topK (qwen_forward.zig:177-193): highest logits, lowest id first among equals."""
    order = np.lexsort((np.arange(logits.size), -logits.astype(np.float64)))[:k]
    return [(int(i), float(logits[i])) for i in order if logits[i] != -np.inf]


def _weights_kind(art) -> int:
    from . import artifact as A
    from . import cuda
    t = art.find("model.layers.0.self_attn.q_proj.weight")
    if t is None:
        raise CliError("forward-golden: TensorNotFound: model.layers.0.self_attn.q_proj.weight")
    return cuda.W_Q8 if t.dtype == A.DT_I8 else cuda.W_BF16


def forward_golden(args, out=None) -> int:
    out = out or sys.stdout
    resolve(args.backend)
    if args.dump:
        raise CliError("forward-golden: --dump (per-layer host copies) is not available on the cuda backend")
    from . import artifact as A
    from . import cuda
    try:
        art = A.Artifact(args.artifact)
    except A.ArtifactError as e:
        raise CliError(f"forward-golden: load failed ({args.artifact}): {e}")
    with art:
        m = art.meta()
        ids = parse_tokens(args.tokens) if args.tokens else [m.bos, 2, 3]
        gpu = cuda.Gpu(args.device)
        try:
            model = cuda.Model(gpu, art.arch(), _weights_kind(art), max_batch=1, max_seqs=1,
                               max_seq_len=max(len(ids), 16), max_prefill=max(len(ids), 16),
                               prefill_kv_f32=True)
            model.load_artifact(art)
            logits, _ = model.prefill(0, ids)
        finally:
            gpu.close()
    if args.golden:
        if not os.path.exists(args.golden):
            raise CliError(f"forward-golden: golden file not found ({args.golden})")
        gold = np.fromfile(args.golden, "<f4")
        if gold.size != logits.size:
            raise CliError(f"forward-golden: golden size mismatch (expected {logits.size * 4} bytes)")
        ok, d, idx = expect_close(gold, logits, 1e-3, 1e-2)
        if not ok:
            raise CliError(f"forward-golden: logits differ from the golden file: |d|={d} at {idx}")
        out.write(f"golden OK ({args.golden}, vocab={logits.size})\n")
    out.write(f"forward-golden: {args.artifact}\n")
    out.write(f"tokens: {len(ids)}\n")
    out.write("top logits (last token):\n")
    for i, v in top_k(logits, 8):
        out.write(f"  id={i} logit={v:.6f}\n")
    out.write("\n")
    return 0


def block_bench_json(*, kind: str, hidden: int, prefill_tokens: int, decode_steps: int, warmup: int, iters: int,
                     cuda_init_ns: int | None, cuda_prefill_ns: int | None, cuda_decode_ns_per_token: int | None,
                     cuda_block_path: str | None, batch: int, launches: int | None,
                     fixture: str = "qwen3-0.6b") -> dict:
    """block-bench's JSON object (main.zig:1211-1245) with this backend's fields."""
    rss = resource.getrusage(resource.RUSAGE_SELF).ru_maxrss * 1024
    line = {"backend": kind, "fixture": fixture, "hidden": hidden, "prefill_tokens": prefill_tokens,
            "decode_steps": decode_steps, "warmup": warmup, "iters": iters, "metal_init_ns": None,
            "peak_rss_bytes": rss, "energy_per_token": None, "cpu_prefill_ns": None,
            "cpu_decode_ns_per_token": None, "apple_prefill_ns": None, "apple_decode_ns_per_token": None,
            "apple_block_path": None, "cuda_init_ns": cuda_init_ns, "cuda_prefill_ns": cuda_prefill_ns,
            "cuda_decode_ns_per_token": cuda_decode_ns_per_token, "cuda_block_path": cuda_block_path,
            "cuda_batch": batch, "cuda_launches_per_step": launches}
    return line


def decode_bench(args, out=None) -> int:
    out = out or sys.stdout
    kind = resolve(args.backend)
    from . import cuda
    from . import workload
    t0 = time.perf_counter_ns()
    gpu = cuda.Gpu(args.device)
    init_ns = time.perf_counter_ns() - t0
    B, T, S = args.batch, args.prefill_tokens, args.decode_steps
    try:
        if args.artifact:
            from . import artifact as A
            with A.Artifact(args.artifact) as art:
                arch, wk = art.arch(), _weights_kind(art)
                model = cuda.Model(gpu, arch, wk, max_batch=B, max_seqs=B,
                                   max_seq_len=T + (args.warmup + args.iters) * S + 8, max_prefill=T)
                model.load_artifact(art)
        else:
            arch = cuda.QWEN3_0_6B
            model = cuda.Model(gpu, arch, cuda.W_Q8, max_batch=B, max_seqs=B,
                               max_seq_len=T + (args.warmup + args.iters) * S + 8, max_prefill=T)
            model.fill_synthetic(args.seed, 0.02, 0.0)
        slots = list(range(B))
        prefill_ns, decode_ns = [], []
        for it in range(args.warmup + args.iters):
            first = [model.prefill(s, workload.prompt(s, T, args.seed, arch.vocab), want_logits=False) for s in slots]
            p_ns = gpu.last_step_ns
            _, ms = model.generate(slots, first, S)
            if it >= args.warmup:
                prefill_ns.append(p_ns)
                decode_ns.append(ms * 1e6 / S)
        path = gpu.last_path
        launches = gpu.step_launches
    finally:
        gpu.close()
    p = int(np.median(prefill_ns)) if prefill_ns else None
    d = int(np.median(decode_ns)) if decode_ns else None
    out.write("zynfer decode-bench\n===================\n")
    out.write(f"backend={kind.value}  fixture=qwen3 hidden={arch.hidden} n_q={arch.n_q} n_kv={arch.n_kv} "
              f"head_dim={arch.head_dim} layers={arch.layers} batch={B}\n")
    out.write(f"prefill_tokens={T} decode_steps={S}\n")
    out.write(f"cuda prefill_ns={p} decode_ns_per_token={d} iters={args.iters} path={path}\n")
    out.write("\njson\n")
    line = block_bench_json(kind=kind.value, hidden=arch.hidden, prefill_tokens=T, decode_steps=S,
                            warmup=args.warmup, iters=args.iters, cuda_init_ns=init_ns, cuda_prefill_ns=p,
                            cuda_decode_ns_per_token=d, cuda_block_path=path, batch=B, launches=launches)
    out.write(json.dumps(line) + "\n")
    return 0


def backends(args, out=None) -> int:
    out = out or sys.stdout
    """printBackends (main.zig): every kind with whether this build has it."""
    for k in backend.BackendKind:
        out.write(f"{k.display:8s} buildable={str(backend.is_backend_buildable(k)).lower()}\n")
    out.write(f"default={backend.default_kind().display}\n")
    return 0


def parse(argv=None):
    ap = argparse.ArgumentParser(prog="zynfer", description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--backend", default=None)
    ap.add_argument("--device", type=int, default=0)
    sub = ap.add_subparsers(dest="cmd", required=True)
    sub.add_parser("backends")
    fg = sub.add_parser("forward-golden")
    fg.add_argument("artifact")
    fg.add_argument("--tokens", default=None)
    fg.add_argument("--golden", default=None)
    fg.add_argument("--dump", default=None)
    fg.add_argument("--backend", dest="backend_sub", default=None)
    db = sub.add_parser("decode-bench")
    db.add_argument("--artifact", default=None)
    db.add_argument("--batch", type=int, default=1)
    db.add_argument("--prefill-tokens", type=int, default=512)
    db.add_argument("--decode-steps", type=int, default=32)
    db.add_argument("--warmup", type=int, default=1)
    db.add_argument("--iters", type=int, default=3)
    db.add_argument("--seed", type=int, default=20250601)
    db.add_argument("--backend", dest="backend_sub", default=None)
    args = ap.parse_args(argv)
    if getattr(args, "backend_sub", None):
        args.backend = args.backend_sub
    return args


def main(argv=None) -> int:
    args = parse(argv)
    return {"backends": backends, "forward-golden": forward_golden, "decode-bench": decode_bench}[args.cmd](args)


if __name__ == "__main__":
    sys.exit(main())
