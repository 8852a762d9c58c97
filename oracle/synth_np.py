"""numpy restatement of the synthetic-data generator (zynfer_b200/csrc/synth_rng.h).

Test infrastructure: checks that the C and CUDA generators agree with an
independent implementation, and writes fixture weights for the golden script.
"""
from __future__ import annotations

import numpy as np

M64 = np.uint64(0xFFFFFFFFFFFFFFFF)
IH4_SIGMA = 37837.2266

ZS_EMBED, ZS_FINAL_NORM, ZS_TOKENS, ZS_PROMPT_LENS, ZS_ACTIVATIONS = 1, 2, 3, 4, 5
LAYER_CODES = {
    "input_layernorm.weight": 1, "self_attn.q_norm.weight": 2, "self_attn.k_norm.weight": 3,
    "self_attn.q_proj.weight": 4, "self_attn.k_proj.weight": 5, "self_attn.v_proj.weight": 6,
    "self_attn.o_proj.weight": 7, "post_attention_layernorm.weight": 8,
    "mlp.gate_proj.weight": 9, "mlp.up_proj.weight": 10, "mlp.down_proj.weight": 11,
}


def _mix64(z):
    with np.errstate(over="ignore"):
        z = (z + np.uint64(0x9E3779B97F4A7C15)) & M64
        z = ((z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)) & M64
        z = ((z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)) & M64
        return z ^ (z >> np.uint64(31))


def key(seed: int, stream: int) -> np.uint64:
    s = np.array([stream], np.uint64)
    return _mix64(np.array([seed], np.uint64) ^ _mix64(s))[0]


def layer_stream(layer: int, code: int) -> int:
    return ((layer + 1) << 8) | code


def bits(k, start: int, n: int):
    idx = np.arange(start, start + n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return _mix64(np.uint64(k) + idx * np.uint64(0xD1B54A32D192ED03))


def normal(n: int, seed: int, stream: int, std: float, chunk: int = 1 << 24) -> np.ndarray:
    k = key(seed, stream)
    scale = np.float32(std / IH4_SIGMA)
    out = np.empty(n, np.float32)
    for s in range(0, n, chunk):
        h = bits(k, s, min(chunk, n - s))
        m = np.uint64(0xFFFF)
        tot = (h & m) + ((h >> np.uint64(16)) & m) + ((h >> np.uint64(32)) & m) + (h >> np.uint64(48))
        c = tot.astype(np.int64) - 131070
        out[s:s + h.size] = c.astype(np.float32) * scale
    return out


def tokens(n: int, seed: int, stream: int, vocab: int) -> np.ndarray:
    return (bits(key(seed, stream), 0, n) % np.uint64(vocab)).astype(np.uint32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """f32 -> bf16 (round to nearest even) -> f32, vectorised."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    lsb = (u >> np.uint64(16)) & np.uint64(1)
    r = ((u + np.uint64(0x7FFF) + lsb) >> np.uint64(16)) << np.uint64(16)
    return (r & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def synth_weights(arch, seed: int, w_std: float = 0.02, norm_std: float = 0.0, bf16: bool = False):
    """Yield (hf_name, f32 array in HF layout) for every tensor of a Qwen3 model,
    generated exactly as zo_model_create_synthetic and the CUDA fill do."""
    H, I, d = arch.hidden, arch.inter, arch.head_dim
    qd, kvd = arch.n_q * d, arch.n_kv * d

    def fin(a):
        return bf16_round(a) if bf16 else a

    def norm(n, stream):
        if norm_std == 0.0:
            return np.ones(n, np.float32)
        return np.float32(1.0) + normal(n, seed, stream, norm_std)

    yield "model.embed_tokens.weight", fin(normal(arch.vocab * H, seed, ZS_EMBED, w_std)).reshape(arch.vocab, H)
    yield "model.norm.weight", fin(norm(H, ZS_FINAL_NORM))
    shapes = {
        "self_attn.q_proj.weight": (qd, H), "self_attn.k_proj.weight": (kvd, H),
        "self_attn.v_proj.weight": (kvd, H), "self_attn.o_proj.weight": (H, qd),
        "mlp.gate_proj.weight": (I, H), "mlp.up_proj.weight": (I, H), "mlp.down_proj.weight": (H, I),
    }
    vec = {"input_layernorm.weight": H, "post_attention_layernorm.weight": H,
           "self_attn.q_norm.weight": d, "self_attn.k_norm.weight": d}
    for layer in range(arch.layers):
        for nm, code in LAYER_CODES.items():
            stream = layer_stream(layer, code)
            full = f"model.layers.{layer}.{nm}"
            if nm in vec:
                yield full, fin(norm(vec[nm], stream))
            else:
                r, c = shapes[nm]
                yield full, fin(normal(r * c, seed, stream, w_std)).reshape(r, c)
