"""Prefix reuse over the paged KV pool (B200 only): zynfer_cu_seq_fork shares a
sequence's whole blocks and copies its partial last block, zynfer_cu_extend
appends tokens after a shared prefix, and blocks return to the pool when the
last sequence holding them is reset. Each forked sequence must decode exactly
as an oracle session that computed its whole history itself (BF16_KV: both
sides keep a bf16 cache and round their own K/V)."""
import numpy as np
import pytest

from oracle import oracle as O
from zynfer_b200 import cuda as zc

from tolerances import BF16_KV, check_logits

pytestmark = pytest.mark.gpu

SMALL = dict(vocab=4096, hidden=512, inter=1024, layers=2, n_q=4, n_kv=2, head_dim=128, max_pos=4096, eps=1e-6,
             theta=1_000_000.0)
SEED, WSTD, NSTD = 11, 0.05, 0.1


@pytest.fixture(scope="module")
def pair():
    gpu = zc.Gpu(0)
    m = zc.Model(gpu, zc.Arch(**SMALL), zc.W_Q8, max_batch=4, max_seqs=8, max_seq_len=128)
    m.fill_synthetic(SEED, WSTD, NSTD)
    ref = O.Model(O.Arch(**SMALL), O.W_Q8, kv_bf16=True, seed=SEED, w_std=WSTD, norm_std=NSTD, threads=4)
    yield m, ref
    ref.close()
    gpu.close()


@pytest.mark.parametrize("n", [41, 32])   # a partial last block (copied), and whole blocks only (all shared)
def test_forks_decode_like_independent_sessions(pair, n):
    m, ref = pair
    V = SMALL["vocab"]
    prompt = O.synth_tokens(41, SEED, 90, V)
    free0, _ = m.pool_stats()
    m.prefill(0, prompt, want_logits=False)
    m.seq_fork(1, 0, n)
    m.seq_fork(2, 0, n)
    assert m.seq_len(1) == n and m.seq_len(2) == n
    free, shared = m.pool_stats()
    assert shared == n // 16                                   # the whole blocks, held three times
    assert free0 - free == 3 + 2 * (1 if n % 16 else 0)        # src's blocks + one copied block per fork
    for layer in range(SMALL["layers"]):
        for which_v in (False, True):
            k0 = m.kv(0, layer, which_v)[:, :n]
            assert np.array_equal(m.kv(1, layer, which_v), k0) and np.array_equal(m.kv(2, layer, which_v), k0)
    sessions = []
    for s in range(3):
        ses = ref.session(128)
        ses.forward(prompt[:41 if s == 0 else n], want_logits=False)
        sessions.append(ses)
    for step in range(3):
        toks = O.synth_tokens(3, 91 + step, 3, V)
        _, logits = m.decode_step([0, 1, 2], toks, want_logits=True)
        for s in range(3):
            check_logits(sessions[s].forward([int(toks[s])]), logits[s], f"seq {s} step {step}", BF16_KV)
    m.seq_reset(0)                                             # the forks keep the shared blocks
    toks = O.synth_tokens(2, 95, 3, V)
    _, logits = m.decode_step([1, 2], toks, want_logits=True)
    for i, s in enumerate((1, 2)):
        check_logits(sessions[s].forward([int(toks[i])]), logits[i], f"seq {s} after the source's reset", BF16_KV)
    m.seq_reset(1)
    m.seq_reset(2)
    assert m.pool_stats() == (free0, 0)                        # every block is back in the pool
    for ses in sessions:
        ses.close()


def test_extend_after_a_shared_prefix_equals_a_full_prefill(pair):
    m, ref = pair
    V = SMALL["vocab"]
    a = O.synth_tokens(48, SEED, 92, V)
    b = np.concatenate([a[:32], O.synth_tokens(9, SEED, 93, V)])   # shares the first 32 tokens with a
    m.prefill(3, a, want_logits=False)
    m.seq_fork(4, 3, 32)
    logits, am = m.extend(4, b[32:])
    assert m.seq_len(4) == len(b)
    want = ref.session(128).prefill_last_logits(b)
    check_logits(want, logits, "prefix reuse + extend", BF16_KV)
    with pytest.raises(zc.InvalidArgument):
        m.seq_fork(5, 3, 49)                                   # longer than the source
    with pytest.raises(zc.InvalidArgument):
        m.seq_fork(3, 3, 10)                                   # a sequence onto itself
    m.seq_reset(3)
    m.seq_reset(4)
