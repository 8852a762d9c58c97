"""Pin the oracle to the reference's own tools (CPU).

tests/golden/*.npz were produced by tests/golden/make_golden.py, which ran the
reference's tools/fixtures/ref_forward_numpy.py and gen_golden_logits.py
(Hugging Face Qwen3, f32, eager attention) unmodified on a synthetic bf16
Qwen3-0.6B checkpoint written from the seeded generator. The oracle, built from
the same seed, must reproduce every layer's last row, the final-normed row and
the logits. Observed agreement is ~1e-5 (the tools use BLAS summation order
and f64 RoPE); the test allows 1e-4.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
ATOL = 1e-4


@pytest.fixture(scope="module")
def model():
    g = np.load(os.path.join(HERE, "golden", "qwen3_bf16_bos23.npz"))
    m = O.Model(O.QWEN3_0_6B, O.W_BF16, kv_bf16=False, seed=int(g["seed"]), w_std=float(g["w_std"]),
                norm_std=float(g["norm_std"]), threads=os.cpu_count() or 1)
    yield m
    m.close()


@pytest.mark.parametrize("case", ["bos23", "rand16"])
def test_oracle_matches_reference_tools(model, case):
    g = np.load(os.path.join(HERE, "golden", f"qwen3_bf16_{case}.npz"))
    s = model.session(64)
    logits, layers, normed = s.forward(g["tokens"], dump=True)
    assert np.max(np.abs(layers - g["np_layers"])) <= ATOL
    assert np.max(np.abs(normed - g["np_normed"])) <= ATOL
    for src in ("np", "hf"):
        assert np.max(np.abs(logits[g[f"{src}_sample_idx"]] - g[f"{src}_sample_vals"])) <= ATOL, src
        assert np.max(np.abs(logits[g[f"{src}_top_ids"]] - g[f"{src}_top_vals"])) <= ATOL, src
        assert abs(float(logits.astype(np.float64).sum()) - float(g[f"{src}_sum"])) <= 1e-2, src
    ids, _ = O.top_k(logits, 8)
    assert ids.tolist() == g["np_top_ids"][:8].tolist() == g["hf_top_ids"][:8].tolist()
