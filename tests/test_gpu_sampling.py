"""Sampling on the device (B200 only) against the oracle's zo_sample_row on the
same logits: temperature only (Gumbel-max over the vocabulary), top-k, and
top-k + top-p, in isolation (zynfer_cu_sample on device logits) and inside
decode_step / generate (zynfer_cu_set_sampling), where the draws are keyed by
(seed, sequence slot, position) and so repeat exactly.

Equality is exact except at a draw that falls within f32 rounding of a
decision boundary (the device's and the host's log / exp may differ in the
last bit); such a case is accepted only when recomputing both candidates'
scores on the host shows them within 1e-5.
"""
import numpy as np
import pytest

from oracle import oracle as O
from zynfer_b200 import cuda as zc

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SMALL = dict(vocab=4096, hidden=512, inter=1024, layers=2, n_q=4, n_kv=2, head_dim=128, max_pos=4096, eps=1e-6,
             theta=1_000_000.0)
RULES = [(0.7, 0, 1.0), (1.0, 40, 1.0), (1.3, 0, 0.9), (0.8, 20, 0.85), (1.0, 1, 1.0)]


def _gumbel_score(logits, v, temp, seed, slot, pos):
    """The Gumbel-max score of vocabulary entry v, recomputed on the host (f32)."""
    from oracle import synth_np
    V = logits.size
    key = synth_np.key(seed, 0x5A5A000000000000 | slot)
    bits = synth_np.bits(key, pos * (V + 1) + v, 1)[0]
    u = np.float32((np.float32(bits >> np.uint64(41)) + np.float32(0.5)) * np.float32(2.0 ** -23))
    g = -np.log(-np.log(np.float64(u)))
    return float(logits[v]) / temp + g


def _agree(logits, got, want, temp, top_k, top_p, seed, slot, pos):
    if got == want:
        return True
    if top_k == 0 and top_p >= 1.0:
        return abs(_gumbel_score(logits, got, temp, seed, slot, pos) - _gumbel_score(logits, want, temp, seed, slot, pos)) < 1e-5
    return abs(float(logits[got]) - float(logits[want])) < 1e-5  # neighbouring candidates at a boundary


@pytest.fixture(scope="module")
def small():
    gpu = zc.Gpu(0)
    m = zc.Model(gpu, zc.Arch(**SMALL), zc.W_Q8, max_batch=16, max_seqs=16, max_seq_len=128)
    m.fill_synthetic(11, 0.05, 0.1)
    yield m
    gpu.close()


@pytest.mark.parametrize("temp,top_k,top_p", RULES)
def test_device_sampler_equals_oracle(small, temp, top_k, top_p):
    rows, V = 16, 151936
    rng = np.random.default_rng(int(temp * 100) + top_k)
    logits = (rng.standard_normal((rows, V)) * 2.5).astype(np.float32)
    slots = np.arange(rows, dtype=np.uint32)
    pos = (np.arange(rows, dtype=np.uint32) * 37 + 5)
    got = small.gpu.sample(torch.from_numpy(logits).cuda(), rows, V, slots, pos, temp, top_k, top_p, seed=77)
    for r in range(rows):
        want = O.sample_row(logits[r], temp, top_k, top_p, 77, int(slots[r]), int(pos[r]))
        assert _agree(logits[r], int(got[r]), want, temp, top_k, top_p, 77, int(slots[r]), int(pos[r])), (r, got[r], want)


def test_decode_with_sampling_matches_oracle_on_its_own_logits(small):
    V = SMALL["vocab"]
    for (temp, top_k, top_p) in RULES:
        small.gpu.set_sampling(temp, top_k, top_p, seed=5)
        for s in range(4):
            small.prefill(s, O.synth_tokens(9 + s, 3, 40 + s, V), want_logits=False)
        for step in range(3):
            positions = [small.seq_len(s) for s in range(4)]
            toks = O.synth_tokens(4, 50 + step, 3, V)
            ids, logits = small.decode_step(list(range(4)), toks, want_logits=True)
            for s in range(4):
                want = O.sample_row(logits[s], temp, top_k, top_p, 5, s, positions[s])
                assert _agree(logits[s], int(ids[s]), want, temp, top_k, top_p, 5, s, positions[s]), (temp, s, step)
    small.gpu.set_sampling(0.0)


def test_generate_with_sampling_repeats_and_differs_by_seed(small):
    V = SMALL["vocab"]
    prompt = O.synth_tokens(12, 3, 60, V)

    def run(seed, temp=0.9):
        small.gpu.set_sampling(temp, 0, 1.0, seed)
        small.prefill(0, prompt, want_logits=False)
        small.prefill(1, prompt, want_logits=False)
        out, _ = small.generate([0, 1], [5, 5], 12)
        return out

    a, b, c = run(1), run(1), run(2)
    assert np.array_equal(a, b)                      # same seed, slots and positions: the same tokens
    assert not np.array_equal(a, c)                  # another seed draws differently
    assert not np.array_equal(a[:, 0], a[:, 1])      # the two slots draw independently
    greedy = run(0, temp=0.0)
    small.gpu.set_sampling(0.0)
    small.prefill(0, prompt, want_logits=False)
    small.prefill(1, prompt, want_logits=False)
    ref, _ = small.generate([0, 1], [5, 5], 12)
    assert np.array_equal(greedy, ref) and np.array_equal(greedy[:, 0], greedy[:, 1])
    with pytest.raises(zc.InvalidArgument):
        small.gpu.set_sampling(1.0, 65, 1.0, 0)
    with pytest.raises(zc.InvalidArgument):
        small.gpu.set_sampling(1.0, 0, 0.0, 0)
