"""Model-level parity on a small Qwen3-shaped model (B200 only): the CUDA
prefill / decode / generate paths against the oracle session on the same
seeded weights, plus the reference's invariants and the error paths.

Tolerances are the stated ones in tests/tolerances.py: BF16_KV where both
sides keep a bf16 KV cache (the int8 model), F32_PATH where both keep f32 K/V
(the bf16-weight prefill).
"""
import numpy as np
import pytest

from oracle import oracle as O
from zynfer_b200 import cuda as zc

from tolerances import BF16_KV, F32_PATH, check_logits

pytestmark = pytest.mark.gpu

SMALL = dict(vocab=4096, hidden=512, inter=1024, layers=2, n_q=4, n_kv=2, head_dim=128, max_pos=4096,
             eps=1e-6, theta=1_000_000.0)
SEED, WSTD, NSTD = 11, 0.05, 0.1



@pytest.fixture(scope="module")
def gpu():
    g = zc.Gpu(0)
    yield g
    g.close()


@pytest.fixture(scope="module")
def small(gpu):
    m = zc.Model(gpu, zc.Arch(**SMALL), zc.W_Q8, max_batch=16, max_seqs=16, max_seq_len=512)
    m.fill_synthetic(SEED, WSTD, NSTD)
    return m


@pytest.fixture(scope="module")
def oracle_small():
    return O.Model(O.Arch(**SMALL), O.W_Q8, kv_bf16=True, seed=SEED, w_std=WSTD, norm_std=NSTD, threads=4)


def test_synthetic_weights_pack_bit_exact(small, oracle_small):  # ops.zig:145-162
    a = SMALL
    H, I, d = a["hidden"], a["inter"], a["head_dim"]
    shapes = {"self_attn.q_proj.weight": (a["n_q"] * d, H), "self_attn.k_proj.weight": (a["n_kv"] * d, H),
              "self_attn.v_proj.weight": (a["n_kv"] * d, H), "self_attn.o_proj.weight": (H, a["n_q"] * d),
              "mlp.gate_proj.weight": (I, H), "mlp.up_proj.weight": (I, H), "mlp.down_proj.weight": (H, I)}
    names = [("model.embed_tokens.weight", (a["vocab"], H))]
    for layer in range(a["layers"]):
        names += [(f"model.layers.{layer}.{n}", s) for n, s in shapes.items()]
    for name, (r, c) in names:
        q, s = small.download_q8(name, r, c)
        q_ref, s_ref = oracle_small.get_q8(name, r, c)
        assert np.array_equal(q, q_ref), name
        assert np.array_equal(s, s_ref), name


def test_prefill_logits_match_oracle(small, oracle_small):  # qwen_forward.zig:89-160
    ids = O.synth_tokens(37, SEED, 3, SMALL["vocab"])
    logits, am = small.prefill(0, ids)
    ref = oracle_small.session(64).prefill_last_logits(ids)
    check_logits(ref, logits, "prefill")
    assert small.seq_len(0) == 37


def test_prefill_kv_matches_oracle(small, oracle_small):  # kv_cache.zig:49-73 (bf16 pool)
    ids = O.synth_tokens(21, SEED, 7, SMALL["vocab"])
    small.prefill(1, ids, want_logits=False)
    s = oracle_small.session(64)
    s.forward(ids, want_logits=False)
    for layer in range(SMALL["layers"]):
        for which_v in (False, True):
            got = small.kv(1, layer, which_v)
            ref = s.kv(layer, which_v)
            assert got.shape == ref.shape
            # bf16 values: equal, or one bf16 step apart where the f32 inputs straddled a rounding edge
            np.testing.assert_allclose(got, ref, rtol=1.6e-2, atol=1e-3)
            assert np.mean(got == ref) > 0.95


def test_decode_teacher_forced_matches_oracle(small, oracle_small):
    ids = O.synth_tokens(30, SEED, 11, SMALL["vocab"])
    small.prefill(2, ids, want_logits=False)
    s = oracle_small.session(128)
    s.forward(ids, want_logits=False)
    feed = O.synth_tokens(12, SEED, 12, SMALL["vocab"])
    for i, tok in enumerate(feed):
        am, logits = small.decode_step([2], [tok], want_logits=True)
        ref = s.forward([tok])
        check_logits(ref, logits[0], f"step {i}")
    assert small.seq_len(2) == 30 + 12


@pytest.mark.parametrize("path", ["auto", "gemv", "mma", "tcgen05"])
def test_batched_decode_each_row_matches_oracle(gpu, small, oracle_small, path):
    # every linear family at a few rows (norm prologue, residual, SwiGLU and
    # argmax epilogues), past the GEMV's 8 rows, and at the few-row kernel's 16
    gpu.set_linear_path(path)
    try:
        for batch in (3, 8, 12, 16):
            lens = [5 + 13 * i for i in range(batch)]
            seqs = list(range(batch))
            sessions = []
            for sq, n in zip(seqs, lens):
                ids = O.synth_tokens(n, SEED + sq, 3, SMALL["vocab"])
                small.prefill(sq, ids, want_logits=False)
                ses = oracle_small.session(256)
                ses.forward(ids, want_logits=False)
                sessions.append(ses)
            for step in range(3):
                toks = O.synth_tokens(batch, 100 + step, 3, SMALL["vocab"])
                am, logits = small.decode_step(seqs, toks, want_logits=True)
                if path != "auto" and batch <= (8 if path == "gemv" else 16):
                    assert f"{path}" in gpu.last_path, gpu.last_path
                for r in range(batch):
                    check_logits(sessions[r].forward([toks[r]]), logits[r],
                                 f"{path} B={batch} row {r} step {step}")
                    assert int(am[r]) == int(np.argmax(logits[r]))
            for ses in sessions:
                ses.close()
    finally:
        gpu.set_linear_path("auto")


def test_few_row_decode_equals_tcgen05_decode(gpu, small):
    # the few-row MMA linears reproduce the tcgen05 linears bit for bit, so a
    # whole decode step (norms, residuals, SwiGLU, attention, LM head) does too
    logits = {}
    for path in ("mma", "tcgen05"):
        gpu.set_linear_path(path)
        try:
            for batch in (2, 7, 16):
                seqs = list(range(batch))
                for sq in seqs:
                    small.prefill(sq, O.synth_tokens(9 + 5 * sq, SEED + sq, 4, SMALL["vocab"]), want_logits=False)
                for step in range(2):
                    toks = O.synth_tokens(batch, 200 + step, 3, SMALL["vocab"])
                    _, lg = small.decode_step(seqs, toks, want_logits=True)
                    logits[(path, batch, step)] = lg.copy()
                if path == "mma":
                    assert "mma" in gpu.last_path, gpu.last_path
        finally:
            gpu.set_linear_path("auto")
    for (path, batch, step), lg in logits.items():
        if path == "mma":
            assert np.array_equal(lg, logits[("tcgen05", batch, step)]), (batch, step)


def test_generate_graph_equals_stepwise(small):
    ids = O.synth_tokens(40, SEED, 21, SMALL["vocab"])
    first = 17
    small.prefill(3, ids, want_logits=False)
    stepwise = []
    tok = first
    for _ in range(10):
        tok = int(small.decode_step([3], [tok])[0])
        stepwise.append(tok)
    small.prefill(3, ids, want_logits=False)
    out, ms = small.generate([3], [first], 10)
    assert out[:, 0].tolist() == stepwise
    assert ms > 0.0
    assert small.seq_len(3) == 50


def test_greedy_generate_matches_oracle(small, oracle_small):
    ids = O.synth_tokens(25, SEED, 31, SMALL["vocab"])
    small.prefill(4, ids, want_logits=False)
    out, _ = small.generate([4], [9], 16)
    s = oracle_small.session(128)
    s.forward(ids, want_logits=False)
    _, logits = s.greedy(9, 16, teacher=out[:, 0], want_logits=True)
    for i in range(16):  # teacher-forced on the GPU's own tokens
        top2 = np.sort(logits[i])[-2:]
        if top2[1] - top2[0] > BF16_KV["tie"]:
            assert int(np.argmax(logits[i])) == int(out[i, 0]), i


def test_prefill_equals_stepwise_decode_on_gpu(small):  # tiny_block.zig:352-383
    ids = O.synth_tokens(20, SEED, 41, SMALL["vocab"])
    pre, _ = small.prefill(5, ids)
    small.prefill(5, ids[:1], want_logits=False)
    for t in ids[1:-1]:
        small.decode_step([5], [t])
    _, step = small.decode_step([5], [ids[-1]], want_logits=True)
    check_logits(pre, step[0], "prefill vs stepwise")


def test_errors_are_reported_and_context_survives(small):
    with pytest.raises(zc.InvalidArgument):
        small.prefill(6, [SMALL["vocab"]])            # id >= vocab (ops.zig:406)
    with pytest.raises(zc.InvalidArgument):
        small.prefill(6, [])                          # empty prompt (qwen_forward.zig:101)
    with pytest.raises(zc.InvalidArgument):
        small.decode_step([6, 6], [1, 2])             # one sequence twice in a batch
    with pytest.raises(zc.InvalidArgument):
        small.prefill(99, [1])                        # slot out of range
    small.prefill(6, O.synth_tokens(510, 1, 1, SMALL["vocab"]), want_logits=False)
    small.decode_step([6], [1])
    small.decode_step([6], [1])
    with pytest.raises(zc.InvalidArgument):
        small.decode_step([6], [1])                   # KV cache full (qwen_block.zig:176)
    assert small.seq_len(6) == 512
    small.gpu.set_fail_at("launch")
    with pytest.raises(zc.LaunchFailed):
        small.prefill(6, [1, 2, 3])
    small.gpu.set_fail_at("upload")
    with pytest.raises(zc.Internal):
        small.upload_f32("model.norm.weight", np.ones(SMALL["hidden"], np.float32))
    logits, _ = small.prefill(6, [1, 2, 3])           # still usable
    assert np.isfinite(logits).all()


def test_injected_alloc_failure_at_init(gpu):
    g = zc.Gpu(0)
    g.set_fail_at("alloc:3")
    with pytest.raises(zc.OutOfMemory):
        zc.Model(g, zc.Arch(**SMALL), zc.W_Q8, max_batch=1, max_seqs=1, max_seq_len=64)
    g.close()


def test_bf16_model_prefill_matches_f32_oracle():
    gpu = zc.Gpu(0)  # one model per context
    m = zc.Model(gpu, zc.Arch(**SMALL), zc.W_BF16, max_batch=2, max_seqs=2, max_seq_len=256,
                 prefill_kv_f32=True)
    m.fill_synthetic(SEED, WSTD, NSTD)
    ref_model = O.Model(O.Arch(**SMALL), O.W_BF16, kv_bf16=False, seed=SEED, w_std=WSTD, norm_std=NSTD)
    ids = O.synth_tokens(64, SEED, 51, SMALL["vocab"])
    logits, _ = m.prefill(0, ids)
    check_logits(ref_model.session(128).prefill_last_logits(ids), logits, "bf16 prefill", F32_PATH)


@pytest.mark.parametrize("T", [1, 31, 100, 200])
def test_bf16_prefill_ragged_lengths_match_f32_oracle(T):  # qwen_forward.zig:89-160
    # f32 K/V (hi and lo terms), key tiles cut short by T, the attention also
    # writing the O projection's activation planes (the GEMV takes O at T = 1)
    gpu = zc.Gpu(0)
    try:
        m = zc.Model(gpu, zc.Arch(**SMALL), zc.W_BF16, max_batch=2, max_seqs=2, max_seq_len=256,
                     max_prefill=256, prefill_kv_f32=True)
        m.fill_synthetic(SEED, WSTD, NSTD)
        ref_model = O.Model(O.Arch(**SMALL), O.W_BF16, kv_bf16=False, seed=SEED, w_std=WSTD, norm_std=NSTD)
        ids = O.synth_tokens(T, SEED, 52 + T, SMALL["vocab"])
        logits, am = m.prefill(0, ids)
        check_logits(ref_model.session(256).prefill_last_logits(ids), logits, f"bf16 prefill T={T}", F32_PATH)
        assert int(am) == int(np.argmax(logits))
        ref_model.close()
    finally:
        gpu.close()


def test_block_forward_matches_oracle_block():  # qwen_block.zig:161-235, one layer
    arch = dict(SMALL, layers=1)
    gpu = zc.Gpu(0)
    m = zc.Model(gpu, zc.Arch(**arch), zc.W_BF16, max_batch=1, max_seqs=1, max_seq_len=128)
    m.fill_synthetic(SEED, 0.02, NSTD)
    ref = O.Model(O.Arch(**arch), O.W_BF16, kv_bf16=True, seed=SEED, w_std=0.02, norm_std=NSTD)
    s = ref.session(128)
    x = O.synth_normal(65 * arch["hidden"], 3, 5, 1.0).reshape(65, arch["hidden"])
    got_pre = m.block_forward(0, 0, x[:64])
    ref_pre = s.block(0, x[:64])
    assert O.expect_close(ref_pre, got_pre, 2e-3, 2e-3)
    got = m.block_forward(0, 0, x[64:])
    exp = s.block(0, x[64:])
    assert O.expect_close(exp, got, 2e-3, 2e-3)


def test_decode_allocates_nothing(small):  # tiny_block.zig:385-401
    """After the first decode of a batch size (which captures its graph), decode
    steps and generate calls of that batch size allocate neither device memory
    nor host containers."""
    torch = pytest.importorskip("torch")
    slots = [7, 8, 9, 10]
    for sq in slots:
        small.prefill(sq, O.synth_tokens(20, SEED, 60 + sq, SMALL["vocab"]), want_logits=False)
    toks = [1, 2, 3, 4]
    small.decode_step(slots, toks)                     # captures the batch-4 graph
    small.decode_step(slots, toks, want_logits=True)
    small.generate(slots, toks, 2)
    torch.cuda.synchronize()
    before = small.gpu.alloc_events()
    free_before = torch.cuda.mem_get_info(0)[0]
    for i in range(64):
        small.decode_step(slots, toks, want_logits=(i % 8 == 0))
    small.generate(slots, toks, 8)
    torch.cuda.synchronize()
    assert small.gpu.alloc_events() == before
    assert torch.cuda.mem_get_info(0)[0] == free_before
