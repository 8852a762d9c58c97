#!/usr/bin/env python3
"""Generate the golden fixtures that pin the oracle to the reference's own tools.

Runs in the build container only (it needs the reference checkout, which the
GPU machines do not have). Steps:

1. Write a synthetic Qwen3-0.6B checkpoint: bf16 weights from the seeded
   generator (oracle/synth_np.py, the same values the oracle and the CUDA fill
   produce), as an HF directory (config.json + model.safetensors).
2. Run the reference's numpy forward, tools/fixtures/ref_forward_numpy.py,
   unmodified, on that checkpoint (per-layer last rows, final norm, logits).
3. Run the reference's golden-logit tool, tools/fixtures/gen_golden_logits.py,
   unmodified (Hugging Face Qwen3, f32, eager attention) on the same checkpoint.
4. Save compact fixtures under tests/golden/: all per-layer last rows, the
   final-normed row, the top-64 logits, 8192 strided logits and the logits'
   sum / sum of squares, from both tools.

    python tests/golden/make_golden.py --reference <reference checkout> [--work /tmp/zg]
"""
from __future__ import annotations

import argparse
import json
import os
import struct
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import synth_np  # noqa: E402
from oracle.oracle import QWEN3_0_6B  # noqa: E402

SEED = 20251201
CASES = {
    "bos23": [151643, 2, 3],  # the reference's default forward-golden tokens
    "rand16": None,           # 16 seeded ids, stream ZS_TOKENS
}
N_SAMPLE = 8192


def case_tokens(name):
    ids = CASES[name]
    if ids is None:
        ids = synth_np.tokens(16, SEED, synth_np.ZS_TOKENS, QWEN3_0_6B.vocab).tolist()
    return [int(i) for i in ids]


def write_checkpoint(d: Path):
    d.mkdir(parents=True, exist_ok=True)
    a = QWEN3_0_6B
    cfg = {
        "architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3",
        "vocab_size": a.vocab, "hidden_size": a.hidden, "intermediate_size": a.inter,
        "num_hidden_layers": a.layers, "num_attention_heads": a.n_q,
        "num_key_value_heads": a.n_kv, "head_dim": a.head_dim,
        "max_position_embeddings": a.max_pos, "rms_norm_eps": a.eps, "rope_theta": a.theta,
        "tie_word_embeddings": True, "hidden_act": "silu", "attention_bias": False,
        "attention_dropout": 0.0, "use_sliding_window": False, "bos_token_id": 151643,
        "eos_token_id": 151645, "torch_dtype": "bfloat16",
    }
    (d / "config.json").write_text(json.dumps(cfg, indent=1))
    header, blobs, off = {}, [], 0
    for name, w in synth_np.synth_weights(a, SEED, w_std=0.02, norm_std=0.1, bf16=True):
        raw = synth_np.bf16_bits(w).tobytes()
        header[name] = {"dtype": "BF16", "shape": list(w.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(d / "model.safetensors", "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)


def summarise(logits: np.ndarray):
    order = np.argsort(-logits, kind="stable")[:64]
    idx = np.linspace(0, logits.size - 1, N_SAMPLE).astype(np.int64)
    return {
        "top_ids": order.astype(np.int64), "top_vals": logits[order],
        "sample_idx": idx, "sample_vals": logits[idx],
        "sum": np.float64(logits.astype(np.float64).sum()),
        "sumsq": np.float64((logits.astype(np.float64) ** 2).sum()),
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True, help="checkout of the Zynfer reference")
    ap.add_argument("--work", type=Path, default=Path("/tmp/zynfer_golden"))
    args = ap.parse_args()
    ck = args.work / "ckpt"
    if not (ck / "model.safetensors").exists():
        print("writing synthetic checkpoint ...", flush=True)
        write_checkpoint(ck)
    fx = args.reference / "tools" / "fixtures"
    for case in CASES:
        toks = ",".join(str(t) for t in case_tokens(case))
        np_dir = args.work / f"np_{case}"
        print(f"[{case}] reference numpy forward ...", flush=True)
        subprocess.run([sys.executable, str(fx / "ref_forward_numpy.py"), "--model",
                        str(ck / "model.safetensors"), "--tokens", toks, "--out-dir", str(np_dir)],
                       check=True)
        hf_out = args.work / f"hf_{case}.f32"
        print(f"[{case}] reference HF golden logits ...", flush=True)
        subprocess.run([sys.executable, str(fx / "gen_golden_logits.py"), "--model", str(ck),
                        "--tokens", toks, "--out", str(hf_out)], check=True)
        layers = np.stack([np.fromfile(np_dir / f"layer{i:02d}.f32", "<f4") for i in range(28)])
        normed = np.fromfile(np_dir / "normed.f32", "<f4")
        np_logits = np.fromfile(np_dir / "logits.f32", "<f4")
        hf_logits = np.fromfile(hf_out, "<f4")
        out = {"tokens": np.array(case_tokens(case), np.uint32), "seed": np.uint64(SEED),
               "w_std": np.float32(0.02), "norm_std": np.float32(0.1),
               "np_layers": layers, "np_normed": normed}
        for k, v in summarise(np_logits).items():
            out["np_" + k] = v
        for k, v in summarise(hf_logits).items():
            out["hf_" + k] = v
        out["hf_at_np_top"] = hf_logits[out["np_top_ids"]]
        np.savez_compressed(HERE / f"qwen3_bf16_{case}.npz", **out)
        print(f"[{case}] saved; np top={out['np_top_ids'][:4]} hf top={out['hf_top_ids'][:4]}")


if __name__ == "__main__":
    main()
