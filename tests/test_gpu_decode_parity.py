"""Parity on the benchmarked decode configurations (B200 only; about two
minutes of oracle CPU time).

Both sides start from bit-identical caches: zynfer_cu_kv_fill_synthetic on the
GPU and zo_session_fill_kv in the oracle write the same seeded bf16 K/V for
positions [0, n) of every layer, so a long context costs no CPU prefill. The
decode steps after it are teacher-forced: the oracle is fed the GPU's tokens,
and every GPU argmax must equal the oracle's unless the oracle's top-2 gap is
within the stated tie bound (topK, qwen_forward.zig:177-193).

Runs the "kernels" schedule, the one bench.py times: graph launches
(decode_step without logits, generate) and eager launches (decode_step with
logits) of the same kernels.

* Batch 64 at the benchmark's contexts: workload.prompt_lengths(64, 20250601)
  (prompts uniform in [512, 4096]) with one row at 4221, so that the steps
  below reach 4224, the longest context of the 128-step benchmark.
* Config 3: one sequence at context 2048, 64 greedy steps on the device.
* The longest attention split: one sequence at the model's last position.

Tolerance: FULL_DECODE (tests/tolerances.py: max_abs 2e-3, cosine 0.99999,
the bar for f32-accumulate paths). The measured worst max_abs of each case is
printed (pytest -s) and recorded beside the bound there.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from zynfer_b200 import cuda as zc
from zynfer_b200 import workload

from tolerances import FULL_DECODE, check_logits

pytestmark = pytest.mark.gpu

SEED = 20250601
THREADS = max(1, os.cpu_count() or 1)
MAX_SEQ_LEN = 4232
VOCAB = 151936


@pytest.fixture(scope="module")
def pair():
    gpu = zc.Gpu(0)
    m = zc.Model(gpu, zc.QWEN3_0_6B, zc.W_Q8, max_batch=64, max_seqs=64, max_seq_len=MAX_SEQ_LEN)
    m.fill_synthetic(SEED, 0.02, 0.0)
    ref = O.Model(O.QWEN3_0_6B, O.W_Q8, kv_bf16=True, seed=SEED, w_std=0.02, norm_std=0.0, threads=THREADS)
    yield m, ref
    ref.close()
    gpu.close()


def _argmax_ok(ref_logits, got_id, what):
    """GPU argmax equals the oracle's, or the oracle's top two are within the tie bound."""
    top = int(np.argmax(ref_logits))
    if top == int(got_id):
        return 0
    srt = np.sort(ref_logits)
    gap = float(srt[-1] - srt[-2])
    assert gap <= FULL_DECODE["tie"], f"{what}: argmax {got_id} vs oracle {top} with top-2 gap {gap}"
    assert ref_logits[int(got_id)] >= srt[-1] - FULL_DECODE["tie"], what
    return 1


def test_batch64_benchmark_contexts(pair):
    m, ref = pair
    lens = workload.prompt_lengths(64, SEED)
    lens[int(np.argmax(lens))] = 4221  # one row past 4096: the steps below reach 4224
    slots = list(range(64))
    for i, n in enumerate(lens):
        m.kv_fill_synthetic(i, n, SEED + i)
        assert m.seq_len(i) == n
    toks0 = workload.tokens(64, SEED, 77)
    a0 = m.decode_step(slots, toks0)                            # graph
    a1, logits1 = m.decode_step(slots, a0, want_logits=True)    # eager, logits
    out, _ = m.generate(slots, a1, 2)                           # graph, two steps on the device
    assert m.gpu.last_path.startswith("generate:") and m.gpu.last_path.endswith(":graph")
    worst, flips = 0.0, 0
    for i, n in enumerate(lens):
        s = ref.session(n + 8)
        s.fill_kv(n, SEED + i)
        flips += _argmax_ok(s.forward([int(toks0[i])]), a0[i], f"row {i} step 0")
        r1 = s.forward([int(a0[i])])
        check_logits(r1, logits1[i], f"row {i} (context {n + 1}) step 1", FULL_DECODE)
        worst = max(worst, O.diff(r1, logits1[i]).max_abs)
        flips += _argmax_ok(r1, a1[i], f"row {i} step 1")
        flips += _argmax_ok(s.forward([int(a1[i])]), out[0, i], f"row {i} step 2")
        flips += _argmax_ok(s.forward([int(out[0, i])]), out[1, i], f"row {i} step 3")
        s.close()
    print(f"batch 64, contexts {min(lens)}..{max(lens) + 4}: worst logit max_abs {worst:.3e}, near-tie flips {flips}")


def test_config3_context_2048_greedy_64(pair):
    m, ref = pair
    n, steps, first = 2048, 64, 4242
    m.kv_fill_synthetic(0, n, SEED)
    out, _ = m.generate([0], [first], steps)                   # batch-1 graph: one-row GEMVs
    ids = out[:, 0]
    _, last_logits = m.decode_step([0], [int(ids[-1])], want_logits=True)
    s = ref.session(n + steps + 8)
    s.fill_kv(n, SEED)
    _, logits = s.greedy(first, steps, teacher=ids, want_logits=True)
    flips = sum(_argmax_ok(logits[i], ids[i], f"step {i}") for i in range(steps))
    r = s.forward([int(ids[-1])])
    check_logits(r, last_logits[0], "config 3 step 65", FULL_DECODE)
    s.close()
    print(f"config 3 (context 2048, {steps} greedy steps): near-tie flips {flips}, "
          f"step-65 logit max_abs {O.diff(r, last_logits[0]).max_abs:.3e}")


def test_longest_attention_split(pair):
    """Context at the model's last position: one (row, kv head) spans the most
    KV blocks and so the most warp shares and CTA records of the split."""
    m, ref = pair
    n = MAX_SEQ_LEN - 1
    m.kv_fill_synthetic(1, n, SEED + 1)
    m.kv_fill_synthetic(2, 37, SEED + 2)      # a short row beside it moves the split boundaries
    am, logits = m.decode_step([1, 2], [11, 12], want_logits=True)
    for slot, ctx, tok in ((1, n, 11), (2, 37, 12)):
        s = ref.session(ctx + 2)
        s.fill_kv(ctx, SEED + slot)
        r = s.forward([tok])
        check_logits(r, logits[slot - 1], f"slot {slot} context {ctx + 1}", FULL_DECODE)
        _argmax_ok(r, am[slot - 1], f"slot {slot}")
        s.close()
    with pytest.raises(zc.InvalidArgument):
        m.decode_step([1], [1])                # the cache is full now (qwen_block.zig:176)
