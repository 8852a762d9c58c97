"""The oracle against the reference's own known-answer tests.

Each test restates one test of the reference (cited file:line) with the same
inputs and the same tolerance, run through the oracle library.
"""
import math

import numpy as np
import pytest

from oracle import oracle as O
from oracle import synth_np


def iota(shape, start, step):
    n = int(np.prod(shape))
    return (np.float32(start) + np.float32(step) * np.arange(n, dtype=np.float32)).reshape(shape)


def test_add_and_silu_mul_tiny():  # ops.zig:459-477
    a = np.array([1, 2], np.float32)
    b = np.array([3, 4], np.float32)
    c = np.empty(2, np.float32)
    O.lib().zo_add(c, a, b, 2)
    assert c.tolist() == [4.0, 6.0]
    c = O.silu_mul(a, b)
    expected0 = O.lib().zo_silu_scalar(1.0) * np.float32(3)
    assert O.expect_close([expected0], c[:1], 1e-6, 1e-6)
    assert abs(c[0] - 3.0 / (1.0 + math.exp(-1.0))) < 1e-6


def test_softmax_sums_to_one():  # ops.zig:479-492
    y = O.softmax(np.array([[1, 2, 3, 4]], np.float32))
    assert abs(float(y.sum()) - 1.0) <= 1e-6


def test_matmul_identity():  # ops.zig:494-508
    a = iota((2, 2), 1, 1)
    c = O.matmul(a, np.eye(2, dtype=np.float32))
    assert O.expect_close(a, c, 1e-6, 0)


def test_rope_position_zero_is_identity():  # ops.zig:510-519
    x = iota((1, 2, 4), 0.25, 0.25)
    assert O.expect_close(x, O.rope(x, 0, 10_000.0), 1e-6, 0)


def test_rope_d2_pos1_hand_values():  # ops.zig:521-530
    x = np.array([[[1.0, 0.0]]], np.float32)
    y = O.rope(x, 1, 10_000.0)
    assert O.expect_close([math.cos(1.0), math.sin(1.0)], y.ravel(), 1e-6, 1e-6)


def test_causal_attention_masks_the_future():  # ops.zig:532-553
    q = np.zeros((1, 2, 2), np.float32)
    k = np.zeros((1, 2, 2), np.float32)
    v = np.array([[[1, 0], [0, 1]]], np.float32)
    q[0, 0, 0] = 1
    q[0, 1, 0] = 1
    o = O.attention_into(q, k, v, kv_len=2)
    assert abs(o[0, 0, 0] - 1) <= 1e-5
    assert abs(o[0, 0, 1] - 0) <= 1e-5


def test_attention_reads_strided_kv():  # ops.zig:555-596
    q = iota((2, 1, 2), 0.25, 0.25)
    pk = iota((2, 2, 2), 0.1, 0.1)
    pv = iota((2, 2, 2), 0.2, 0.2)
    k = np.zeros((2, 4, 2), np.float32)
    v = np.zeros((2, 4, 2), np.float32)
    k[:, :2] = pk
    v[:, :2] = pv
    o_packed = O.attention_into(q, pk, pv, kv_len=2)
    o_stride = O.attention_into(q, k, v, kv_len=2)
    assert O.expect_close(o_packed, o_stride, 1e-6, 0)


def test_attention_rejects_bad_shapes():  # ops.zig:302-304
    q = np.zeros((3, 1, 2), np.float32)
    k = np.zeros((2, 4, 2), np.float32)
    with pytest.raises(ValueError):
        O.attention_into(q, k, k, kv_len=2)  # n_q % n_kv != 0
    q = np.zeros((2, 3, 2), np.float32)
    with pytest.raises(ValueError):
        O.attention_into(q, k, k, kv_len=2)  # q_len > kv_len


def test_head_time_permute_round_trips():  # ops.zig:598-609
    x = iota((3, 2, 4), 0, 1)
    mid = np.empty((2, 3, 4), np.float32)
    out = np.empty_like(x)
    O.lib().zo_tokens_heads_to_heads_tokens(mid, x, 3, 2, 4)
    O.lib().zo_heads_tokens_to_tokens_heads(out, mid, 2, 3, 4)
    assert np.array_equal(out, x)


def test_matvec_matches_matmul_n1():  # ops.zig:611-633 (seeded inputs, same property)
    rng = np.random.default_rng(7)
    a = (rng.random((5, 3), dtype=np.float32) * 2 - 1)
    x = (rng.random(3, dtype=np.float32) * 2 - 1)
    y = O.matvec(a, x)
    c = O.matmul(a, x.reshape(3, 1))
    assert O.expect_close(y, c.ravel(), 1e-5, 1e-5)


def test_pack_row_q8_matvec_approximates_f32():  # ops.zig:635-657
    w = iota((8, 16), 0.01, 0.02)
    x = iota((16,), 0.1, 0.05)
    y_f = O.matvec(w, x)
    q, s = O.pack_row_q8(w)
    y_q = O.matvec_q8(q, s, x)
    assert O.expect_close(y_f, y_q, 0.15, 0.05)


def test_pack_tensor_q8_matmul_approximates_f32():  # ops.zig:659-680
    w = iota((6, 8), 0.02, 0.01)
    b = iota((8, 5), 0.05, 0.02)
    c_f = O.matmul(w, b)
    q, s = O.pack_tensor_q8(w)
    c_q = O.matmul_q8(q, s, b)
    assert O.expect_close(c_f, c_q, 0.2, 0.08)


def test_rms_norm_plus_minus_one():  # tests/numerical/ops.zig:16-32
    y = O.rms_norm(np.array([[1, -1, 1, -1]], np.float32), np.ones(4, np.float32), 1e-6)
    assert abs(y[0, 0] - 1) <= 1e-5 and abs(y[0, 1] + 1) <= 1e-5


def test_pack_row_q8_rules():  # ops.zig:145-162: zero row scale 1, clamp, half away from zero
    w = np.zeros((3, 4), np.float32)
    w[1] = [127.0, -63.5, 0.5, -0.5]  # scale 1: round half away from zero
    w[2] = [2.0, -1.0, 0.0, 1.0]
    q, s = O.pack_row_q8(w)
    assert s[0] == 1.0 and q[0].tolist() == [0, 0, 0, 0]
    assert s[1] == np.float32(127.0) / np.float32(127.0)
    assert q[1].tolist() == [127, -64, 1, -1]
    assert s[2] == np.float32(2.0) / np.float32(127.0)
    assert q[2].tolist() == [127, -64, 0, 64]


def test_top_k_orders_and_prefers_lowest_index():  # qwen_forward.zig:177-193
    ids, vals = O.top_k(np.array([0.5, 2.0, 2.0, -1.0, 1.0], np.float32), 3)
    assert ids.tolist() == [1, 2, 4]
    assert vals.tolist() == [2.0, 2.0, 1.0]


def test_bf16_widen_known_value():  # bf16.zig:21-27
    assert abs(O.lib().zo_bf16_to_f32(0x3F80) - 1.0) < 1e-3


def test_bf16_rne_matches_numpy_restatement():
    x = O.synth_normal(4096, 11, 99, 1.0)
    assert np.array_equal(O.bf16_round(x[:256]), synth_np.bf16_round(x[:256]))
    # ties to even: 1 + 2^-8 is halfway between bf16 neighbours 1 and 1 + 2^-7
    t = np.array([1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -8], np.float32)
    assert O.bf16_round(t).tolist() == [1.0, 1.0 + 2.0 ** -6]


def test_diff_reports_last_max_index():  # compare.zig:14-41 (>= keeps the last)
    d = O.diff([1, 2, 3], [1.5, 2, 3.5])
    assert d.failing_index == 2 and abs(d.max_abs - 0.5) < 1e-7


def test_synth_generator_c_matches_numpy():
    for stream in (1, 5, synth_np.layer_stream(3, 7)):
        c = O.synth_normal(10_000, 1234, stream, 0.02)
        n = synth_np.normal(10_000, 1234, stream, 0.02)
        assert np.array_equal(c, n)
    t_c = O.synth_tokens(5000, 9, synth_np.ZS_TOKENS, 151936)
    t_n = synth_np.tokens(5000, 9, synth_np.ZS_TOKENS, 151936)
    assert np.array_equal(t_c, t_n)
    big = synth_np.normal(1 << 20, 5, 1, 1.0)
    assert abs(float(big.mean())) < 5e-3 and abs(float(big.std()) - 1.0) < 5e-3


def test_sampler_rule():  # extension: temperature / top-k / top-p sampling (zo_sample_row)
    rng = np.random.default_rng(1)
    logits = (rng.standard_normal(1000) * 3).astype(np.float32)
    top = int(np.argmax(logits))
    assert O.sample_row(logits, 1e-4, 0, 1.0, 5, 0, 0) == top      # a cold temperature is the argmax
    assert O.sample_row(logits, 1.0, 1, 1.0, 5, 0, 0) == top       # top-1 is the argmax
    assert O.sample_row(logits, 1.0, 0, 1e-6, 5, 0, 0) == top      # a tiny nucleus keeps only the top
    # the draws are keyed by (seed, slot, position): repeatable, and independent across slots
    assert O.sample_row(logits, 1.0, 0, 1.0, 9, 3, 7) == O.sample_row(logits, 1.0, 0, 1.0, 9, 3, 7)
    p = np.exp(logits.astype(np.float64) - logits.max())
    p /= p.sum()
    n = 3000
    full = np.bincount([O.sample_row(logits, 1.0, 0, 1.0, s, 0, 0) for s in range(n)], minlength=1000) / n
    best = np.argsort(-p)[:3]
    assert np.all(np.abs(full[best] - p[best]) < 4 * np.sqrt(p[best] / n) + 1e-3)
    k5 = np.bincount([O.sample_row(logits, 1.0, 5, 1.0, s, 1, 0) for s in range(n)], minlength=1000) / n
    assert set(np.nonzero(k5)[0]) <= set(np.argsort(-logits, kind="stable")[:5].tolist())
    q = np.sort(p)[::-1][:5] / np.sort(p)[::-1][:5].sum()
    assert np.all(np.abs(np.sort(k5[k5 > 0])[::-1][:len(q)] - q[:np.count_nonzero(k5)]) < 0.05)
