"""The persistent decode schedule against the oracle and against the
multi-kernel schedule (B200 only): one cooperative dataflow kernel per step
(weights and KV blocks streamed into shared memory ahead of the layer chain,
tagged activations instead of grid barriers).

The kernel is built for Qwen3-0.6B widths (hidden 1024,
intermediate 3072, 16 x 128 query dims, 8 kv heads), so these tests use those
widths with 2 layers and a 8192-token vocabulary, which keeps the oracle fast.
Tolerances: BF16_KV (both sides keep a bf16 KV cache).
"""
import numpy as np
import pytest

from oracle import oracle as O
from zynfer_b200 import cuda as zc

from tolerances import BF16_KV, check_logits

pytestmark = pytest.mark.gpu

WIDE = dict(vocab=8192, hidden=1024, inter=3072, layers=2, n_q=16, n_kv=8, head_dim=128, max_pos=4096,
            eps=1e-6, theta=1_000_000.0)
SEED, WSTD, NSTD = 5, 0.02, 0.1


@pytest.fixture(scope="module")
def sched():
    return "persistent"


@pytest.fixture(scope="module")
def gpu():
    g = zc.Gpu(0)
    yield g
    g.close()


@pytest.fixture(scope="module")
def wide(gpu, sched):
    m = zc.Model(gpu, zc.Arch(**WIDE), zc.W_Q8, max_batch=8, max_seqs=13, max_seq_len=1536)
    m.fill_synthetic(SEED, WSTD, NSTD)
    gpu.set_decode_schedule(sched)
    return m


@pytest.fixture(scope="module")
def oracle_wide():
    return O.Model(O.Arch(**WIDE), O.W_Q8, kv_bf16=True, seed=SEED, w_std=WSTD, norm_std=NSTD, threads=8)


def test_single_sequence_teacher_forced(wide, oracle_wide, sched):  # qwen_block.zig:161-235 per layer, t = 1
    ids = O.synth_tokens(27, SEED, 3, WIDE["vocab"])
    wide.prefill(0, ids, want_logits=False)
    s = oracle_wide.session(128)
    s.forward(ids, want_logits=False)
    feed = O.synth_tokens(9, SEED, 4, WIDE["vocab"])  # crosses the 32-token block boundary
    for i, tok in enumerate(feed):
        am, logits = wide.decode_step([0], [tok], want_logits=True)
        assert wide.gpu.last_path == f"decode:{sched}"
        ref = s.forward([tok])
        check_logits(ref, logits[0], f"step {i}")
        assert int(am[0]) == int(np.argmax(logits[0]))
    assert wide.seq_len(0) == 36


def test_kv_append_matches_oracle(wide, oracle_wide):  # kv_cache.zig:49-73
    ids = O.synth_tokens(14, SEED, 5, WIDE["vocab"])
    wide.prefill(1, ids, want_logits=False)
    s = oracle_wide.session(64)
    s.forward(ids, want_logits=False)
    for tok in O.synth_tokens(4, SEED, 6, WIDE["vocab"]):
        wide.decode_step([1], [tok])
        s.forward([tok], want_logits=False)
    for layer in range(WIDE["layers"]):
        for which_v in (False, True):
            got, ref = wide.kv(1, layer, which_v), s.kv(layer, which_v)
            # bf16 values: equal, or one bf16 step apart where the f32 inputs of the
            # two sides straddle a rounding edge (more of them at this width)
            np.testing.assert_allclose(got, ref, rtol=1.6e-2, atol=1e-3)
            assert np.mean(got == ref) > 0.9


@pytest.mark.parametrize("batch", [2, 5, 8])
def test_batched_rows_match_oracle(wide, oracle_wide, batch):
    seqs = list(range(2, 2 + batch))
    sessions = []
    for j, sq in enumerate(seqs):
        ids = O.synth_tokens(3 + 17 * j, SEED + sq, 7, WIDE["vocab"])
        wide.prefill(sq, ids, want_logits=False)
        ses = oracle_wide.session(256)
        ses.forward(ids, want_logits=False)
        sessions.append(ses)
    for step in range(3):
        toks = O.synth_tokens(batch, 200 + step, 3, WIDE["vocab"])
        am, logits = wide.decode_step(seqs, toks, want_logits=True)
        for r in range(batch):
            check_logits(sessions[r].forward([toks[r]]), logits[r], f"B={batch} row {r} step {step}")


def test_long_context_rows_match_oracle(wide, oracle_wide):
    """Contexts of ~1000 and ~600 tokens: every (row, kv head) spans many CTAs'
    block ranges, so the cross-CTA merge of partial softmax states runs."""
    seqs, lens = [12, 11], [1000, 600]
    sessions = []
    for sq, n in zip(seqs, lens):
        ids = O.synth_tokens(n, SEED + sq, 8, WIDE["vocab"])
        wide.prefill(sq, ids, want_logits=False)
        ses = oracle_wide.session(1100)
        ses.forward(ids, want_logits=False)
        sessions.append(ses)
    for step in range(3):
        toks = O.synth_tokens(2, 300 + step, 3, WIDE["vocab"])
        am, logits = wide.decode_step(seqs, toks, want_logits=True)
        for r in range(2):
            check_logits(sessions[r].forward([toks[r]]), logits[r], f"long row {r} step {step}")


def test_device_wait_timeout_is_reported(wide, oracle_wide):
    """A device wait that runs out ends the step with DeviceTimeout and leaves
    the context usable. Injected on the host (ZYNFER_CUDA_FAIL_AT=wait): one
    layer input is polled with a tag that nothing writes, so the kernel's
    bounded wait gives up, every CTA stops through the abort flag, and no
    fault or hang is involved. The next step of the same sequence then
    matches the oracle (the failed step advanced nothing)."""
    ids = O.synth_tokens(30, SEED, 41, WIDE["vocab"])
    wide.prefill(9, ids, want_logits=False)
    s = oracle_wide.session(64)
    s.forward(ids, want_logits=False)
    wide.gpu.set_fail_at("wait")
    with pytest.raises(zc.DeviceTimeout):
        wide.decode_step([9], [7])
    assert wide.seq_len(9) == 30
    am, logits = wide.decode_step([9], [7], want_logits=True)
    check_logits(s.forward([7]), logits[0], "step after the timeout")
    assert int(am[0]) == int(np.argmax(logits[0]))


def test_generate_equals_stepwise(wide, sched):
    ids = O.synth_tokens(40, SEED, 21, WIDE["vocab"])
    wide.prefill(10, ids, want_logits=False)
    stepwise, tok = [], 17
    for _ in range(12):
        tok = int(wide.decode_step([10], [tok])[0])
        stepwise.append(tok)
    wide.prefill(10, ids, want_logits=False)
    out, ms = wide.generate([10], [17], 12)
    assert wide.gpu.last_path == f"generate:{sched}"
    assert out[:, 0].tolist() == stepwise
    assert ms > 0.0


def test_single_kernel_and_kernel_schedules_agree(wide, sched):
    ids = O.synth_tokens(50, SEED, 23, WIDE["vocab"])
    feed = O.synth_tokens(6, SEED, 24, WIDE["vocab"])
    runs = {}
    for name in (sched, "kernels"):
        wide.gpu.set_decode_schedule(name)
        wide.prefill(11, ids, want_logits=False)
        runs[name] = [wide.decode_step([11], [t], want_logits=True)[1][0] for t in feed]
    wide.gpu.set_decode_schedule(sched)
    for i, (a, b) in enumerate(zip(runs[sched], runs["kernels"])):
        check_logits(b, a, f"schedules step {i}", BF16_KV)


def test_schedule_names_and_shape_limits(gpu, wide):
    with pytest.raises(zc.InvalidArgument):
        gpu.set_decode_schedule("bogus")
    g2 = zc.Gpu(0)
    small = dict(WIDE, hidden=512, inter=1024, n_q=4, n_kv=2)
    zc.Model(g2, zc.Arch(**small), zc.W_Q8, max_batch=1, max_seqs=1, max_seq_len=64)
    with pytest.raises(zc.Unsupported):
        g2.set_decode_schedule("persistent")
    g2.set_decode_schedule("kernels")
    g2.close()


def test_phase_trace_covers_every_phase(wide):
    """With timing on, the persistent step records (start, end) of every phase
    as globaltimer ns: 4 + 10 L entries, each phase starting after the previous
    one ended, and the per-class totals of kernel_time add up to the step."""
    gpu = wide.gpu
    ids = O.synth_tokens(20, SEED, 31, WIDE["vocab"])
    wide.prefill(11, ids, want_logits=False)
    gpu.set_timing(True)
    try:
        wide.decode_step([11], [5])
        t = gpu.phase_trace().astype(np.int64)
        n_att, ms_att = gpu.kernel_time(zc.K_ATTN)
        n_lin, ms_lin = gpu.kernel_time(zc.K_LINEAR)
        n_head, ms_head = gpu.kernel_time(zc.K_LMHEAD)
    finally:
        gpu.set_timing(False)
    L = WIDE["layers"]
    assert t.size == 4 + 10 * L
    phases = 5 * L + 1
    starts, ends = t[1:2 * phases:2], t[2:2 * phases + 1:2]
    assert (ends >= starts).all()
    assert (starts[1:] >= ends[:-1]).all()
    assert t[3 + 2 * (phases - 1)] >= ends[-1]
    assert (n_att, n_lin, n_head) == (L, 4 * L, 1)
    total_ms = (t[3 + 2 * (phases - 1)] - t[1]) / 1e6
    assert abs((ms_att + ms_lin + ms_head) - total_ms) < 1e-3
