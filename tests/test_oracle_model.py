"""Model-level oracle tests: the reference's own invariants for the Qwen3
forward and the block-level decode, restated (citations per test)."""
import numpy as np
import pytest

from oracle import oracle as O

SMALL = O.Arch(vocab=512, hidden=64, inter=96, layers=2, n_q=4, n_kv=2, head_dim=16,
               max_pos=256, eps=1e-6, theta=10_000.0)


def mini_model():
    """qwen_forward.zig:195-300: the Stage 11 mini artifact's deterministic fills."""
    a = O.STAGE11_MINI
    m = O.Model(a, O.W_F32)

    def vec(n, seed):  # fillVec, qwen_forward.zig:285-287
        return np.float32(seed) * np.float32(0.01) + np.arange(n, dtype=np.float32) * np.float32(0.001)

    def mat(r, c, seed):  # fillMatrixHF, qwen_forward.zig:290-300
        i = np.arange(r)[:, None] + np.arange(c)[None, :]
        return np.float32(seed) * np.float32(0.002) + i.astype(np.float32) * np.float32(0.0003)

    H, I, d = a.hidden, a.inter, a.head_dim
    qd, kvd = a.n_q * d, a.n_kv * d
    m.set_tensor("model.embed_tokens.weight", mat(a.vocab, H, 1))
    m.set_tensor("model.norm.weight", vec(H, 100))
    s = 200
    p = "model.layers.0."
    m.set_tensor(p + "input_layernorm.weight", vec(H, s + 1))
    m.set_tensor(p + "self_attn.q_norm.weight", vec(d, s + 2))
    m.set_tensor(p + "self_attn.k_norm.weight", vec(d, s + 3))
    m.set_tensor(p + "self_attn.q_proj.weight", mat(qd, H, s + 4))
    m.set_tensor(p + "self_attn.k_proj.weight", mat(kvd, H, s + 5))
    m.set_tensor(p + "self_attn.v_proj.weight", mat(kvd, H, s + 6))
    m.set_tensor(p + "self_attn.o_proj.weight", mat(H, qd, s + 7))
    m.set_tensor(p + "post_attention_layernorm.weight", vec(H, s + 8))
    m.set_tensor(p + "mlp.gate_proj.weight", mat(I, H, s + 9))
    m.set_tensor(p + "mlp.up_proj.weight", mat(I, H, s + 10))
    m.set_tensor(p + "mlp.down_proj.weight", mat(H, I, s + 11))
    return m


def test_mini_forward_is_deterministic_and_ordered():  # qwen_forward.zig:302-329
    m1, m2 = mini_model(), mini_model()
    l1 = m1.session(8).prefill_last_logits([2, 3])
    l2 = m2.session(8).prefill_last_logits([2, 3])
    assert O.expect_close(l1, l2, 0, 0)
    ids, vals = O.top_k(l1, 3)
    assert vals[0] >= vals[1]


def test_mini_forward_is_nonzero():  # qwen_forward.zig:331-346
    logits = mini_model().session(8).prefill_last_logits([1, 2, 3])
    assert float(np.abs(logits).sum()) > 0


def test_prefill_rejects_empty_and_oversize():  # qwen_forward.zig:101, qwen_block.zig:175-176
    s = mini_model().session(4)
    with pytest.raises(ValueError):
        s.prefill_last_logits([])
    with pytest.raises(ValueError):
        s.prefill_last_logits([1, 2, 3, 4, 5])
    with pytest.raises(ValueError):
        s.prefill_last_logits([8])  # id >= vocab (ops.zig:406)


@pytest.mark.parametrize("wkind,kv_bf16", [(O.W_F32, False), (O.W_Q8, False), (O.W_Q8, True)])
def test_prefill_matches_stepwise_decode(wkind, kv_bf16):  # tiny_block.zig:352-383
    m = O.Model(SMALL, wkind, kv_bf16=kv_bf16, seed=5, w_std=0.05, norm_std=0.1)
    ids = O.synth_tokens(12, 5, 3, SMALL.vocab)
    s = m.session(32)
    _, pre_layers, _ = s.forward(ids, dump=True)
    pre_logits = s.forward([7])  # one more token on top of the prefill
    s.reset()
    for i, t in enumerate(ids):
        _, step_layers, _ = s.forward([t], dump=True)
    step_logits = s.forward([7])
    assert s.used == 13
    assert O.expect_close(pre_layers, step_layers, 1e-5, 1e-5)
    assert O.expect_close(pre_logits, step_logits, 1e-5, 1e-5)


def test_cache_overflow_is_reported():  # tiny_block.zig:403-421, kv_cache.zig:94-106
    m = O.Model(SMALL, O.W_F32, seed=1)
    s = m.session(2)
    s.forward([1, 2])
    with pytest.raises(ValueError):
        s.forward([3])
    assert s.used == 2


def test_kv_append_layout_and_bf16_rounding():  # kv_cache.zig:49-73 + bf16 extension
    m32 = O.Model(SMALL, O.W_Q8, kv_bf16=False, seed=3)
    m16 = O.Model(SMALL, O.W_Q8, kv_bf16=True, seed=3)
    s32, s16 = m32.session(16), m16.session(16)
    s32.forward([4, 5, 6])
    s16.forward([4, 5, 6])
    assert s32.used == 3
    # layer 0 sees identical inputs, so its bf16 cache is the rounded f32 cache
    for which_v in (False, True):
        k32 = s32.kv(0, which_v)
        k16 = s16.kv(0, which_v)
        assert k32.shape == (SMALL.n_kv, 3, SMALL.head_dim)
        assert np.array_equal(O.bf16_round(k32[:, :, :8]), k16[:, :, :8])


def test_q8_model_packs_bit_exact():  # ops.zig:145-162 applied to every linear
    from oracle import synth_np
    m = O.Model(SMALL, O.W_Q8, seed=21, w_std=0.02)
    for name, w in synth_np.synth_weights(SMALL, 21, w_std=0.02):
        if w.ndim != 2:
            continue
        q, s = m.get_q8(name, *w.shape)
        q_ref, s_ref = O.pack_row_q8(w)
        assert np.array_equal(q, q_ref), name
        assert np.array_equal(s, s_ref), name


def test_greedy_decode_teacher_forced_equals_free_run():
    m = O.Model(SMALL, O.W_Q8, kv_bf16=True, seed=8, w_std=0.05)
    s = m.session(64)
    s.forward(O.synth_tokens(10, 8, 3, SMALL.vocab))
    free = s.greedy(17, 8)
    s.reset()
    s.forward(O.synth_tokens(10, 8, 3, SMALL.vocab))
    forced = s.greedy(17, 8, teacher=free)
    assert np.array_equal(free, forced)
    assert s.used == 18
