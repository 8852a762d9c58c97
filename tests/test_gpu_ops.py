"""Op-level parity of the CUDA kernels against the oracle (B200 only).

Tolerances: int8 packing is bit-exact; f32-accumulate linears and norms use
the reference's GPU-vs-CPU tolerance for reductions (docs/numerics.md:24-28,
q8 GEMV 2e-4) with the compare.zig rule max_abs <= atol + rtol * |expected|.
"""
import numpy as np
import pytest

from oracle import oracle as O
from zynfer_b200 import cuda as zc

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def gpu():
    g = zc.Gpu(0)
    yield g
    g.close()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.cpu().numpy()


def test_caps(gpu):
    c = gpu.caps()
    assert c.sm_major == 10 and c.sm_count >= 132
    assert c.tcgen05 == 1 and c.bulk_copy == 1


def test_pack_q8_device_is_bit_exact(gpu):  # ops.zig:145-162
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((257, 1024)) * 0.02).astype(np.float32)
    w[0] = 0.0                                        # zero row: scale 1
    w[1, :4] = [127.0, -63.5, 0.5, -0.5]              # ties round away from zero
    w[1, 4:] = 0.0
    w[2] = np.float32(1e-30)                          # tiny values
    q_ref, s_ref = O.pack_row_q8(w)
    wd = dev(w)
    qd = torch.empty((257, 1024), dtype=torch.int8, device="cuda")
    sd = torch.empty(257, dtype=torch.float32, device="cuda")
    gpu.pack_q8(wd, 257, 1024, qd, sd)
    gpu.sync()
    assert np.array_equal(host(qd), q_ref)
    assert np.array_equal(host(sd), s_ref)


SHAPES = [(3072, 1024), (4096, 1024), (1024, 2048), (6144, 1024), (1024, 3072), (151936, 1024)]


@pytest.mark.parametrize("m,k", SHAPES)
@pytest.mark.parametrize("batch", [1, 8])
def test_linear_q8_matches_matvec_q8(gpu, m, k, batch):  # ops.zig:181-197
    w = O.synth_normal(m * k, 77, 1000 + m + k, 0.02).reshape(m, k)
    q, s = O.pack_row_q8(w)
    x = O.synth_normal(batch * k, 78, 5, 1.0).reshape(batch, k)
    y = torch.empty((batch, m), dtype=torch.float32, device="cuda")
    gpu.linear(zc.W_Q8, dev(q), dev(s), dev(x), batch, m, k, y)
    gpu.sync()
    got = host(y)
    for b in range(batch):
        ref = O.matvec_q8(q, s, x[b], threads=8)
        d = O.diff(ref, got[b])
        assert O.expect_close(ref, got[b], 2e-4, 2e-4), (b, d.max_abs, d.failing_index)


@pytest.mark.parametrize("batch", [2, 3, 5, 9, 16, 64, 100])
def test_linear_q8_batches(gpu, batch):  # gemv (<= 8 rows) and the tiled GEMM (> 8 rows)
    m, k = 1024, 3072
    w = O.synth_normal(m * k, 9, 9, 0.02).reshape(m, k)
    q, s = O.pack_row_q8(w)
    x = O.synth_normal(batch * k, 10, 5, 1.0).reshape(batch, k)
    y = torch.empty((batch, m), dtype=torch.float32, device="cuda")
    gpu.linear(zc.W_Q8, dev(q), dev(s), dev(x), batch, m, k, y)
    gpu.sync()
    got = host(y)
    for b in range(batch):
        assert O.expect_close(O.matvec_q8(q, s, x[b]), got[b], 2e-4, 2e-4), b


@pytest.mark.parametrize("path", ["tcgen05", "simt", "gemv"])
@pytest.mark.parametrize("m,k,batch", [(4096, 1024, 1), (4096, 1024, 5), (1024, 3072, 8), (4096, 1024, 16),
                                       (6144, 1024, 48), (1024, 2048, 64), (3072, 1024, 100), (1024, 1024, 200)])
def test_linear_q8_each_path(gpu, path, m, k, batch):  # ops.zig:181-197 on every kernel family
    if path == "gemv" and batch > 8:
        pytest.skip("the GEMV takes at most 8 rows")
    w = O.synth_normal(m * k, 31, m + k, 0.02).reshape(m, k)
    q, s = O.pack_row_q8(w)
    x = O.synth_normal(batch * k, 32, batch, 1.0).reshape(batch, k)
    x[0, :7] *= 50.0  # one large-magnitude row: exercises the per-row fixed-point exponent
    y = torch.empty((batch, m), dtype=torch.float32, device="cuda")
    gpu.set_linear_path(path)
    try:
        gpu.linear(zc.W_Q8, dev(q), dev(s), dev(x), batch, m, k, y)
        gpu.sync()
        assert gpu.last_path == {"tcgen05": "linear:tcgen05", "simt": "linear:simt", "gemv": "linear:gemv"}[path]
    finally:
        gpu.set_linear_path("auto")
    got = host(y)
    for b in range(batch):
        ref = O.matvec_q8(q, s, x[b])
        d = O.diff(ref, got[b])
        assert O.expect_close(ref, got[b], 2e-4, 2e-4), (path, b, d.max_abs, d.failing_index)


@pytest.mark.parametrize("m,k,batch,expect", [(4096, 1024, 1, "linear:gemv"), (1024, 3072, 1, "linear:gemv"),
                                              (4096, 1024, 2, "linear:mma"), (1024, 3072, 6, "linear:mma"),
                                              (1024, 1024, 7, "linear:mma"), (1024, 2048, 7, "linear:tcgen05"),
                                              (1024, 1024, 9, "linear:tcgen05"), (1024, 1024, 16, "linear:tcgen05"),
                                              (4096, 1024, 17, "linear:tcgen05"), (16512, 1024, 1, "linear:tcgen05"),
                                              (16512, 1024, 4, "linear:tcgen05")])
def test_linear_q8_auto_reports_the_kernel_it_ran(gpu, m, k, batch, expect):  # ops.zig:181-197
    # auto: the GEMV for one activation row, the few-row MMA kernel for 2..6
    # rows (2..8 when k <= 1024), each for at most 16384 outputs; tcgen05 otherwise
    w = O.synth_normal(m * k, 33, m + k, 0.02).reshape(m, k)
    q, s = O.pack_row_q8(w)
    x = O.synth_normal(batch * k, 34, batch, 1.0).reshape(batch, k)
    y = torch.empty((batch, m), dtype=torch.float32, device="cuda")
    gpu.set_linear_path("auto")
    gpu.linear(zc.W_Q8, dev(q), dev(s), dev(x), batch, m, k, y)
    gpu.sync()
    assert gpu.last_path == expect
    got = host(y)
    for b in range(batch):
        ref = O.matvec_q8(q, s, x[b])
        assert O.expect_close(ref, got[b], 2e-4, 2e-4), (b, O.diff(ref, got[b]).max_abs)


@pytest.mark.parametrize("m,k", [(4096, 1024), (6144, 1024), (1024, 2048), (1024, 3072), (3072, 1024), (512, 4096)])
@pytest.mark.parametrize("batch", [2, 5, 8, 9, 16])
def test_linear_q8_few_rows_equals_tcgen05_and_oracle(gpu, m, k, batch):  # ops.zig:200-228
    # the few-row MMA kernel builds the plane kernel's digits itself and sums
    # them exactly: its outputs equal the tcgen05 path's bit for bit
    w = O.synth_normal(m * k, 41, m + k, 0.02).reshape(m, k)
    q, s = O.pack_row_q8(w)
    x = O.synth_normal(batch * k, 42, batch, 1.0).reshape(batch, k)
    x[-1, :5] *= 80.0  # one row with a larger fixed-point exponent
    x[0, :] = 0.0      # and an all-zero row
    fits = k <= (3072 if batch <= 8 else 1024)  # the activation rows it holds in registers
    got = {}
    for path in ("mma", "tcgen05"):
        y = torch.full((batch, m), float("nan"), dtype=torch.float32, device="cuda")
        gpu.set_linear_path(path)
        try:
            gpu.linear(zc.W_Q8, dev(q), dev(s), dev(x), batch, m, k, y)
            gpu.sync()
            assert gpu.last_path == f"linear:{path if fits else 'tcgen05'}"
        finally:
            gpu.set_linear_path("auto")
        got[path] = host(y)
    assert np.array_equal(got["mma"], got["tcgen05"])
    for b in range(batch):
        ref = O.matvec_q8(q, s, x[b])
        d = O.diff(ref, got["mma"][b])
        assert O.expect_close(ref, got["mma"][b], 2e-4, 2e-4), (b, d.max_abs, d.failing_index)


@pytest.mark.parametrize("m,k", [(4096, 1024), (6144, 1024), (1024, 2048), (1024, 3072)])
def test_linear_q8_tile_shapes_agree(gpu, m, k):  # ops.zig:200-228
    # 9, 16, 24 and 40 rows run 16-, 32- and 64-token tiles with different
    # cluster splits of K; each output row depends only on its own activation
    # row and the sums are exact, so the shared rows agree bit for bit
    w = O.synth_normal(m * k, 51, m + k, 0.02).reshape(m, k)
    q, s = O.pack_row_q8(w)
    x = O.synth_normal(40 * k, 52, 40, 1.0).reshape(40, k)
    x[3, :9] *= 60.0
    got = {}
    gpu.set_linear_path("tcgen05")
    try:
        for batch in (40, 24, 16, 9):
            y = torch.full((batch, m), float("nan"), dtype=torch.float32, device="cuda")
            gpu.linear(zc.W_Q8, dev(q), dev(s), dev(x[:batch]), batch, m, k, y)
            gpu.sync()
            got[batch] = host(y)
    finally:
        gpu.set_linear_path("auto")
    for batch in (24, 16, 9):
        assert np.array_equal(got[batch], got[40][:batch]), batch
    for b in range(0, 40, 7):
        assert O.expect_close(O.matvec_q8(q, s, x[b]), got[40][b], 2e-4, 2e-4), b


@pytest.mark.parametrize("k,batch", [(1024, 17), (1024, 24), (2048, 9), (4096, 2)])
def test_linear_q8_few_rows_falls_back_where_it_cannot_run(gpu, k, batch):
    # more than 16 rows, or more activation values than it holds in registers:
    # the tcgen05 path runs instead
    m = 1024
    w = O.synth_normal(m * k, 43, 1, 0.02).reshape(m, k)
    q, s = O.pack_row_q8(w)
    x = O.synth_normal(batch * k, 44, batch, 1.0).reshape(batch, k)
    y = torch.empty((batch, m), dtype=torch.float32, device="cuda")
    gpu.set_linear_path("mma")
    try:
        gpu.linear(zc.W_Q8, dev(q), dev(s), dev(x), batch, m, k, y)
        gpu.sync()
        assert gpu.last_path == "linear:tcgen05"
    finally:
        gpu.set_linear_path("auto")
    got = host(y)
    for b in range(batch):
        assert O.expect_close(O.matvec_q8(q, s, x[b]), got[b], 2e-4, 2e-4), b


@pytest.mark.parametrize("path", ["tcgen05", "simt"])
@pytest.mark.parametrize("batch", [5, 64, 200])
def test_linear_bf16_each_path(gpu, path, batch):  # ops.zig:133-141 on bf16-widened weights
    from oracle import synth_np
    m, k = 2048, 1024
    w = synth_np.bf16_round(O.synth_normal(m * k, 6, 6, 0.02)).reshape(m, k)
    bits = synth_np.bf16_bits(w)
    x = O.synth_normal(batch * k, 7, 7, 1.0).reshape(batch, k)
    y = torch.empty((batch, m), dtype=torch.float32, device="cuda")
    gpu.set_linear_path(path)
    try:
        gpu.linear(zc.W_BF16, dev(bits.view(np.int16)), None, dev(x), batch, m, k, y)
        gpu.sync()
    finally:
        gpu.set_linear_path("auto")
    got = host(y)
    for b in range(batch):
        assert O.expect_close(O.matvec(w, x[b]), got[b], 1e-4, 1e-4), (path, b)


@pytest.mark.parametrize("batch", [1, 4, 24])
def test_linear_bf16_matches_matvec(gpu, batch):  # ops.zig:133-141 on bf16-widened weights
    from oracle import synth_np
    m, k = 2048, 1024
    w = synth_np.bf16_round(O.synth_normal(m * k, 4, 4, 0.02)).reshape(m, k)
    bits = synth_np.bf16_bits(w)
    x = O.synth_normal(batch * k, 5, 5, 1.0).reshape(batch, k)
    y = torch.empty((batch, m), dtype=torch.float32, device="cuda")
    gpu.linear(zc.W_BF16, dev(bits.view(np.int16)), None, dev(x), batch, m, k, y)
    gpu.sync()
    got = host(y)
    for b in range(batch):
        assert O.expect_close(O.matvec(w, x[b]), got[b], 1e-4, 1e-4), b


def test_rmsnorm_matches_oracle(gpu):  # ops.zig:49-67
    x = O.synth_normal(37 * 1024, 1, 2, 1.0).reshape(37, 1024)
    w = 1.0 + O.synth_normal(1024, 1, 3, 0.1)
    y = torch.empty((37, 1024), dtype=torch.float32, device="cuda")
    gpu.rmsnorm(dev(x), dev(w), 37, 1024, 1e-6, y)
    gpu.sync()
    assert O.expect_close(O.rms_norm(x, w), host(y), 1e-5, 1e-5)


def test_rmsnorm_plus_minus_one(gpu):  # tests/numerical/ops.zig:16-32
    x = np.tile(np.array([1, -1], np.float32), 64).reshape(1, 128)
    y = torch.empty((1, 128), dtype=torch.float32, device="cuda")
    gpu.rmsnorm(dev(x), dev(np.ones(128, np.float32)), 1, 128, 1e-6, y)
    gpu.sync()
    out = host(y)
    assert abs(out[0, 0] - 1) <= 1e-5 and abs(out[0, 1] + 1) <= 1e-5


def test_injected_launch_fault_then_recovers(gpu):
    m, k = 512, 512
    q = dev(np.ones((m, k), np.int8))
    s = dev(np.ones(m, np.float32))
    x = dev(np.ones((1, k), np.float32))
    y = torch.empty((1, m), dtype=torch.float32, device="cuda")
    gpu.set_fail_at("launch")
    with pytest.raises(zc.LaunchFailed):
        gpu.linear(zc.W_Q8, q, s, x, 1, m, k, y)
    gpu.linear(zc.W_Q8, q, s, x, 1, m, k, y)
    gpu.sync()
    assert np.all(host(y) == 512.0)


def test_linear_rejects_bad_k(gpu):
    y = torch.empty((1, 8), dtype=torch.float32, device="cuda")
    with pytest.raises(zc.Unsupported):
        gpu.linear(zc.W_Q8, y, y, y, 1, 8, 100, y)
