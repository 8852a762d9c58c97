#!/usr/bin/env python3
"""Generate the `.zynfer` fixture that pins the artifact reader to the reference's converter.

Runs in the build container only (it needs the reference checkout). Writes a
tiny Qwen3-shaped checkpoint (config.json + model.safetensors, bf16 weights
from the seeded generator, oracle/synth_np.py) and converts it with the
reference's own tools/checkpoint/safetensors_to_zynfer.py, unmodified. The
result is tests/golden/mini_bf16.zynfer (a few KB); tests/test_artifact.py
reads it back through the library and rebuilds it byte for byte with
zynfer_b200.artifact.build.

    python tests/golden/make_artifact_golden.py --reference <reference checkout> [--work /tmp/zart]
"""
from __future__ import annotations

import argparse
import json
import struct
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import synth_np  # noqa: E402
from oracle.oracle import Arch  # noqa: E402

SEED = 20251202
# a tiny Qwen3 shape (the reference's stage-11 mini dims, qwen3.zig:69-84)
MINI = Arch(vocab=8, hidden=16, inter=32, layers=1, n_q=2, n_kv=1, head_dim=8, max_pos=32, eps=1e-6, theta=10_000.0)
CONFIG = {
    "architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "vocab_size": MINI.vocab,
    "hidden_size": MINI.hidden, "intermediate_size": MINI.inter, "num_hidden_layers": MINI.layers,
    "num_attention_heads": MINI.n_q, "num_key_value_heads": MINI.n_kv, "head_dim": MINI.head_dim,
    "max_position_embeddings": MINI.max_pos, "rms_norm_eps": MINI.eps, "rope_theta": MINI.theta,
    "tie_word_embeddings": True, "bos_token_id": 1, "eos_token_id": 2, "torch_dtype": "bfloat16",
}


def weights():
    """(name, f32 values rounded to bf16) of every tensor of the mini model."""
    return list(synth_np.synth_weights(MINI, SEED, w_std=0.02, norm_std=0.1, bf16=True))


def write_checkpoint(d: Path):
    d.mkdir(parents=True, exist_ok=True)
    (d / "config.json").write_text(json.dumps(CONFIG, indent=1))
    header, blobs, off = {}, [], 0
    for name, w in weights():
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True, help="checkout of the Zynfer reference")
    ap.add_argument("--work", type=Path, default=Path("/tmp/zynfer_artifact_golden"))
    args = ap.parse_args()
    ck = args.work / "ckpt"
    write_checkpoint(ck)
    out = HERE / "mini_bf16.zynfer"
    subprocess.run([sys.executable, str(args.reference / "tools" / "checkpoint" / "safetensors_to_zynfer.py"),
                    "--config", str(ck / "config.json"), "--weights", str(ck / "model.safetensors"),
                    "--out", str(out)], check=True)
    print(f"wrote {out} ({out.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
