"""Op-level parity of the attention-side exports against the oracle (B200 only):
zynfer_cu_attn_decode (attentionInto, ops.zig:285-354, with the per-head
norms, RoPE and the K/V append it fuses), zynfer_cu_rmsnorm_qk_rope (ops.zig:
49-67 + 233-261 per head) and zynfer_cu_swiglu (siluMul, ops.zig:36-42), and
zynfer_cu_kv_fill_synthetic against zo_session_fill_kv.

Tolerances (compare.zig rule max_abs <= atol + rtol |expected|):
* cached K/V from the seeded fill: bit-exact;
* attention output: atol = rtol = 1e-4 (q split into two bf16 terms, exact
  products with bf16 K/V, f32 softmax and accumulation); the reference side
  appends the host's bf16 K/V row, which can sit one bf16 step from the
  GPU's where the RMSNorm sums (different order) straddle a rounding edge;
  at kv_len 1 the output is the appended V row, bit-exact;
* q/k norm + RoPE: atol = rtol = 1e-5 (the RMS sum order; the RoPE angles are
  the same f32 values);
* siluMul: atol = 1e-6, rtol = 1e-5 (device expf against the host's).
"""
import numpy as np
import pytest

from oracle import oracle as O
from zynfer_b200 import cuda as zc

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

ARCH1 = zc.Arch(layers=1)
MAX_SEQ_LEN = 4232
LONG_SEQ_LEN = 11008
THETA = 1_000_000.0


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _one_layer(max_batch, max_seq_len):
    gpu = zc.Gpu(0)
    m = zc.Model(gpu, ARCH1, zc.W_Q8, max_batch=max_batch, max_seqs=max_batch, max_seq_len=max_seq_len)
    m.fill_synthetic(3, 0.02, 0.0)
    qn = (1.0 + O.synth_normal(128, 5, 1, 0.1)).astype(np.float32)
    kn = (1.0 + O.synth_normal(128, 5, 2, 0.1)).astype(np.float32)
    m.upload_f32("model.layers.0.self_attn.q_norm.weight", qn)
    m.upload_f32("model.layers.0.self_attn.k_norm.weight", kn)
    oracle = O.Model(O.Arch(layers=1), O.W_Q8, kv_bf16=True, seed=3, w_std=0.02, norm_std=0.0, threads=4)
    return gpu, (m, qn, kn, oracle)


@pytest.fixture(scope="module")
def one_layer():
    gpu, t = _one_layer(64, MAX_SEQ_LEN)
    yield t
    t[3].close()
    gpu.close()


@pytest.fixture(scope="module")
def one_layer_long():
    gpu, t = _one_layer(1, LONG_SEQ_LEN)
    yield t
    t[3].close()
    gpu.close()


def test_kv_fill_matches_oracle_fill(one_layer):
    m, _, _, oracle = one_layer
    for n in (1, 16, 17, 300):
        m.kv_fill_synthetic(5, n, 900 + n)
        s = oracle.session(n + 1)
        s.fill_kv(n, 900 + n)
        for which in (False, True):
            assert np.array_equal(m.kv(5, 0, which), s.kv(0, which)), (n, which)
        s.close()


def _check_attn_decode(one_layer, lens, qkv_seed):
    m, qn, kn, oracle = one_layer
    batch = len(lens)
    seqs = list(range(batch))
    for i, L in enumerate(lens):
        m.kv_fill_synthetic(i, L - 1, 7000 + L + i)
    qkv = O.synth_normal(batch * 4096, 11, qkv_seed, 1.0).reshape(batch, 4096)
    out = torch.empty((batch, 16, 128), dtype=torch.float32, device="cuda")
    m.attn_decode(0, seqs, dev(qkv), out)
    got = out.cpu().numpy()
    for i, L in enumerate(lens):
        pos = L - 1
        assert m.seq_len(i) == pos  # the decode step advances lengths, not the op
        q = O.rope(O.rms_norm(qkv[i, :2048].reshape(1, 16, 128), qn), pos, THETA)[0]
        k_new = O.rope(O.rms_norm(qkv[i, 2048:3072].reshape(1, 8, 128), kn), pos, THETA)[0]
        v_new = qkv[i, 3072:].reshape(8, 128)
        s = oracle.session(L)
        s.fill_kv(pos, 7000 + L + i)
        K = np.concatenate([s.kv(0, False), O.bf16_round(k_new)[:, None, :]], axis=1)
        V = np.concatenate([s.kv(0, True), O.bf16_round(v_new)[:, None, :]], axis=1)
        s.close()
        ref = O.attention_into(q[:, None, :], K, V, L)[:, 0]
        d = O.diff(ref, got[i])
        assert O.expect_close(ref, got[i], 1e-4, 1e-4), (i, L, d.max_abs, d.failing_index)
        if L == 1:  # one position: the output is the appended V row itself, both heads of each group
            assert np.array_equal(got[i], np.repeat(O.bf16_round(v_new), 2, axis=0)), i


@pytest.mark.parametrize("batch", [1, 8, 64])
def test_attn_decode_matches_attention_into(one_layer, batch):
    kv_lens = [1, 257, 2304, 4224]
    _check_attn_decode(one_layer, [kv_lens[(i + batch) % 4] for i in range(batch)], batch)


# One sequence runs as one cluster of 8 CTAs (64 warps) per kv head, the CTAs'
# records merged in the first CTA's shared memory. Lengths: one warp holds the
# whole row (1, 2, 16 positions), one CTA holds it (17, 128), all 64 warps one
# block each (1024), shares of 2 and 3 blocks (1025, 2049, 3072) and the
# cache's last position (4232: shares of 5 blocks, 7 CTAs with records).
@pytest.mark.parametrize("kv_len", [1, 2, 16, 17, 128, 1024, 1025, 2049, 3072, MAX_SEQ_LEN])
def test_attn_decode_one_sequence(one_layer, kv_len):
    _check_attn_decode(one_layer, [kv_len], 100 + kv_len)


# Past 640 blocks (10240 positions) one sequence is spread over every SM
# instead (the batched kernel's split with one-row settings); both sides of
# the switch and a longer context.
@pytest.mark.parametrize("kv_len", [10240, 10241, LONG_SEQ_LEN])
def test_attn_decode_one_long_sequence(one_layer_long, kv_len):
    _check_attn_decode(one_layer_long, [kv_len], 200 + kv_len)


@pytest.mark.parametrize("pos0", [0, 4219])
def test_rmsnorm_qk_rope_matches_oracle(one_layer, pos0):
    m, _, _, _ = one_layer
    T = 5
    qkv = O.synth_normal(T * 4096, 12, pos0 + 1, 1.0).reshape(T, 4096)
    qn = (1.0 + O.synth_normal(128, 13, 1, 0.1)).astype(np.float32)
    kn = (1.0 + O.synth_normal(128, 13, 2, 0.1)).astype(np.float32)
    q_out = torch.empty((16, T, 128), dtype=torch.float32, device="cuda")
    k_out = torch.empty((8, T, 128), dtype=torch.float32, device="cuda")
    m.rmsnorm_qk_rope(dev(qkv), T, dev(qn), dev(kn), pos0, q_out, k_out)
    q_ref = O.rope(O.rms_norm(qkv[:, :2048].reshape(T, 16, 128), qn), pos0, THETA).transpose(1, 0, 2)
    k_ref = O.rope(O.rms_norm(qkv[:, 2048:3072].reshape(T, 8, 128), kn), pos0, THETA).transpose(1, 0, 2)
    assert O.expect_close(q_ref, q_out.cpu().numpy(), 1e-5, 1e-5)
    assert O.expect_close(k_ref, k_out.cpu().numpy(), 1e-5, 1e-5)
    with pytest.raises(zc.InvalidArgument):
        m.rmsnorm_qk_rope(dev(qkv), T, dev(qn), dev(kn), MAX_SEQ_LEN - 2, q_out, k_out)


def test_swiglu_matches_silu_mul(one_layer):
    m, _, _, _ = one_layer
    n = 3072 * 8 + 5
    g = O.synth_normal(n, 14, 1, 3.0)
    u = O.synth_normal(n, 14, 2, 1.0)
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    m.gpu.swiglu(dev(g), dev(u), n, out)
    m.gpu.sync()
    assert O.expect_close(O.silu_mul(g, u), out.cpu().numpy(), 1e-6, 1e-5)
