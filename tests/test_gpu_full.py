"""Full-size Qwen3-0.6B parity on the B200 against the oracle and the
reference tools' golden fixtures (B200 only; minutes of oracle CPU time).

Tolerances (tests/tolerances.py): F32_PATH (max_abs 2e-3, cosine 0.99999) for
the bf16-weight prefill with f32 K/V and the golden fixtures; BF16_KV for the
int8 model, whose K/V cache is bf16 on both sides; single-block outputs within
compare.zig's rule at atol = rtol = 2e-3.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from zynfer_b200 import cuda as zc

from tolerances import BF16_KV, F32_PATH, check_logits

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
THREADS = max(1, os.cpu_count() or 1)
GOLDEN_SEED = 20251201
LOGIT_ATOL = F32_PATH["atol"]






@pytest.fixture(scope="module")
def gpu():
    g = zc.Gpu(0)
    yield g
    g.close()


@pytest.fixture(scope="module")
def bf16_model(gpu):
    m = zc.Model(zc.Gpu(0), zc.QWEN3_0_6B, zc.W_BF16, max_batch=1, max_seqs=1, max_seq_len=1024,
                 max_prefill=1024, prefill_kv_f32=True)
    m.fill_synthetic(GOLDEN_SEED, 0.02, 0.1)
    yield m


@pytest.mark.parametrize("case", ["bos23", "rand16"])
def test_golden_fixture_on_gpu(bf16_model, case):
    """GPU logits vs the reference's own numpy forward and HF golden tool."""
    g = np.load(os.path.join(HERE, "golden", f"qwen3_bf16_{case}.npz"))
    assert int(g["seed"]) == GOLDEN_SEED
    logits, am = bf16_model.prefill(0, g["tokens"])
    for src in ("np", "hf"):
        ref = g[f"{src}_sample_vals"]
        got = logits[g[f"{src}_sample_idx"]]
        assert np.max(np.abs(ref - got)) <= LOGIT_ATOL, src
        assert np.max(np.abs(g[f"{src}_top_vals"] - logits[g[f"{src}_top_ids"]])) <= LOGIT_ATOL, src
    assert am == int(g["np_top_ids"][0])


def test_config2_prefill_512_matches_oracle(bf16_model):
    """BF16 weights, f32 accumulate, 512 seeded prompt tokens, last-token logits."""
    ids = O.synth_tokens(512, GOLDEN_SEED, 3, 151936)
    logits, _ = bf16_model.prefill(0, ids)
    ref_model = O.Model(O.QWEN3_0_6B, O.W_BF16, kv_bf16=False, seed=GOLDEN_SEED, w_std=0.02,
                        norm_std=0.1, threads=THREADS)
    ref = ref_model.session(512).prefill_last_logits(ids)
    ref_model.close()
    check_logits(ref, logits, "config 2", F32_PATH)


def test_config0_single_block_decode(gpu):
    """One Qwen3 block, kv_len 256 prefilled, one decode step (bf16-stored weights)."""
    arch = zc.Arch(layers=1)
    m = zc.Model(zc.Gpu(0), arch, zc.W_BF16, max_batch=1, max_seqs=1, max_seq_len=320)
    m.fill_synthetic(5, 0.02, 0.0)
    ref_model = O.Model(O.Arch(layers=1), O.W_BF16, kv_bf16=True, seed=5, w_std=0.02, norm_std=0.0,
                        threads=THREADS)
    s = ref_model.session(320)
    x = O.synth_normal(257 * 1024, 5, 5, 1.0).reshape(257, 1024)
    assert O.expect_close(s.block(0, x[:256]), m.block_forward(0, 0, x[:256]), 2e-3, 2e-3)
    exp = s.block(0, x[256:])
    got = m.block_forward(0, 0, x[256:])
    assert O.expect_close(exp, got, 2e-3, 2e-3)
    assert m.seq_len(0) == 257


@pytest.fixture(scope="module")
def q8_pair(gpu):
    m = zc.Model(zc.Gpu(0), zc.QWEN3_0_6B, zc.W_Q8, max_batch=16, max_seqs=16, max_seq_len=512)
    m.fill_synthetic(7, 0.02, 0.0)
    ref = O.Model(O.QWEN3_0_6B, O.W_Q8, kv_bf16=True, seed=7, w_std=0.02, norm_std=0.0, threads=THREADS)
    yield m, ref
    ref.close()


def test_full_q8_weights_bit_exact(q8_pair):
    m, ref = q8_pair
    for name, (r, c) in [("model.embed_tokens.weight", (151936, 1024)),
                         ("model.layers.0.self_attn.q_proj.weight", (2048, 1024)),
                         ("model.layers.13.self_attn.v_proj.weight", (1024, 1024)),
                         ("model.layers.27.mlp.up_proj.weight", (3072, 1024)),
                         ("model.layers.27.mlp.down_proj.weight", (1024, 3072))]:
        q, s = m.download_q8(name, r, c)
        q_ref, s_ref = ref.get_q8(name, r, c)
        assert np.array_equal(q, q_ref) and np.array_equal(s, s_ref), name


def test_config3_reduced_decode_matches_oracle(q8_pair):
    """int8 batch-1 decode: 256-token prompt, 24 teacher-forced greedy steps."""
    m, ref = q8_pair
    ids = O.synth_tokens(256, 7, 3, 151936)
    logits, am = m.prefill(0, ids)
    s = ref.session(512)
    check_logits(s.forward(ids), logits, "prefill")
    out, _ = m.generate([0], [am], 24)
    gpu_ids = [am] + out[:, 0].tolist()
    flips = 0
    for i in range(24):
        r = s.forward([gpu_ids[i]])
        top2 = np.sort(r)[-2:]
        if int(np.argmax(r)) != gpu_ids[i + 1]:
            flips += 1
            assert top2[1] - top2[0] <= BF16_KV["tie"], f"step {i}: argmax differs without a near tie"


def test_config4_reduced_batched_decode(q8_pair):
    """int8 batched decode over sequences of different lengths (gemv and GEMM paths)."""
    m, ref = q8_pair
    for batch in (8, 12):
        lens = [16 + 9 * i for i in range(batch)]
        sessions = []
        for sq, n in enumerate(lens):
            ids = O.synth_tokens(n, 70 + sq, 3, 151936)
            m.prefill(sq, ids, want_logits=False)
            ses = ref.session(512)
            ses.forward(ids, want_logits=False)
            sessions.append(ses)
        for step in range(2):
            toks = O.synth_tokens(batch, 200 + step, 3, 151936)
            am, logits = m.decode_step(list(range(batch)), toks, want_logits=True)
            for r in range(batch):
                check_logits(sessions[r].forward([toks[r]]), logits[r], f"B={batch} row {r}")
        for ses in sessions:
            ses.close()
