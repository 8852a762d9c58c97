"""The allocation-free int8 linear (zynfer_cu_linear_q8_static) through the C ABI.

It exists for callers that cannot call cudaMalloc (an embedder that owns all
device memory, a custom allocator that must not be bypassed). Its scratch and
its device error word are library-owned device arrays, so this checks, against
the oracle's matvecQ8 (ops.zig:181-197) within the linear tolerance used
elsewhere (compare.zig rule, atol = rtol = 2e-4):
* calls in a row with different shapes, a 64-row call before a 5-row call of
  another k (stale pad rows of the shared planes never reach stored outputs),
  and k = 640 and 128, which its multiple-of-128 rule admits;
* that a bounded device wait which runs out (armed on the host: no CTA loads
  its first K stage) is reported by zynfer_cu_linear_q8_static_status, and the
  next call is correct again;
* that sizes and alignments beyond its limits are rejected.
Collected last on purpose.
"""
import numpy as np
import pytest

from oracle import oracle as O
from zynfer_b200 import cuda as zc

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _case(m, k, batch, seed):
    w = O.synth_normal(m * k, seed, 1, 0.02).reshape(m, k)
    q, s = O.pack_row_q8(w)
    x = O.synth_normal(batch * k, seed, 2, 1.0).reshape(batch, k)
    return q, s, x


def _run(q, s, x):
    m, k = q.shape
    batch = x.shape[0]
    y = torch.full((batch, m), float("nan"), dtype=torch.float32, device="cuda")
    zc.linear_q8_static(torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda(), torch.from_numpy(x).cuda(),
                        batch, m, k, y)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def _check(q, s, x, got, what):
    assert np.isfinite(got).all(), what
    for b in range(x.shape[0]):
        ref = O.matvec_q8(q, s, x[b], threads=4)
        assert O.expect_close(ref, got[b], 2e-4, 2e-4), (what, b, O.diff(ref, got[b]).max_abs)


def test_static_linear_matches_matvec_q8_in_a_row():
    assert zc.linear_q8_static_status() == zc.OK
    for (m, k, batch, seed) in [(1024, 1024, 5, 3), (2048, 3072, 64, 4), (1024, 640, 5, 5), (256, 128, 1, 6),
                                (1024, 4096, 3, 7)]:
        q, s, x = _case(m, k, batch, seed)
        _check(q, s, x, _run(q, s, x), (m, k, batch))
    assert zc.linear_q8_static_status() == zc.OK


def test_static_linear_reports_a_device_wait_that_ran_out():
    q, s, x = _case(1024, 1024, 2, 8)
    zc.arm_static_wait_fault()
    _run(q, s, x)                                   # launches; its waits give up after a few seconds
    assert zc.linear_q8_static_status(clear=True) == zc.TIMEOUT
    assert zc.linear_q8_static_status() == zc.OK     # cleared
    _check(q, s, x, _run(q, s, x), "after the timeout")
    assert zc.linear_q8_static_status() == zc.OK


def test_static_linear_rejects_sizes_beyond_its_scratch():
    q, s, x = _case(128, 128, 1, 9)
    qd, sd, xd = torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda(), torch.from_numpy(x).cuda()
    y = torch.empty((1, 128), dtype=torch.float32, device="cuda")
    big = torch.empty((zc.STATIC_MAX_ROWS + 1, 128), dtype=torch.float32, device="cuda")
    with pytest.raises(zc.InvalidArgument):
        zc.linear_q8_static(qd, sd, big, zc.STATIC_MAX_ROWS + 1, 128, 128, big)
    with pytest.raises(zc.InvalidArgument):
        zc.linear_q8_static(qd, sd, xd, 1, 128, zc.STATIC_MAX_K + 128, y)
    with pytest.raises(zc.InvalidArgument):
        zc.linear_q8_static(qd, sd, xd, 1, 100, 128, y)
    with pytest.raises(zc.InvalidArgument):
        zc.linear_q8_static(qd, sd, xd, 1, 1 << 31, 128, y)      # rows beyond the kernels' int range
    with pytest.raises(zc.InvalidArgument):
        zc.linear_q8_static(qd, sd, xd.data_ptr() + 4, 1, 128, 128, y)   # x not 16-byte aligned
    with pytest.raises(zc.InvalidArgument):
        zc.linear_q8_static(qd, sd, xd, 1, 128, 128, y.data_ptr() + 2)   # y not 4-byte aligned
    assert zc.linear_q8_static_status() == zc.OK
