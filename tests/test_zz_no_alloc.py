"""The allocation-free int8 linear (zynfer_cu_linear_q8_static) through the C ABI.

It exists for callers that cannot call cudaMalloc (an embedder that owns all
device memory, a custom allocator that must not be bypassed). Its scratch is a
library-owned device array, so this checks that two calls in a row, with
different shapes, both match the regular entry point zynfer_cu_linear within
the linear tolerance used elsewhere (compare.zig rule, atol = rtol = 2e-4),
and that the size limits are enforced. Collected last on purpose.
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
    return (torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda(), torch.from_numpy(x).cuda())


def test_static_linear_matches_regular_entry_point_twice():
    gpu = zc.Gpu(0)
    try:
        for (m, k, batch, seed) in [(1024, 1024, 5, 3), (2048, 3072, 64, 4)]:
            q, s, x = _case(m, k, batch, seed)
            y_ref = torch.empty((batch, m), dtype=torch.float32, device="cuda")
            y = torch.full((batch, m), float("nan"), dtype=torch.float32, device="cuda")
            gpu.linear(zc.W_Q8, q, s, x, batch, m, k, y_ref)
            gpu.sync()
            zc.linear_q8_static(q, s, x, batch, m, k, y)
            torch.cuda.synchronize()
            ref, got = y_ref.cpu().numpy(), y.cpu().numpy()
            assert np.isfinite(got).all()
            for b in range(batch):
                d = O.diff(ref[b], got[b])
                assert O.expect_close(ref[b], got[b], 2e-4, 2e-4), (m, k, batch, b, d.max_abs)
    finally:
        gpu.close()


def test_static_linear_rejects_sizes_beyond_its_scratch():
    q, s, x = _case(128, 128, 1, 5)
    y = torch.empty((1, 128), dtype=torch.float32, device="cuda")
    big = torch.empty((zc.STATIC_MAX_ROWS + 1, 128), dtype=torch.float32, device="cuda")
    with pytest.raises(zc.InvalidArgument):
        zc.linear_q8_static(q, s, big, zc.STATIC_MAX_ROWS + 1, 128, 128, big)
    with pytest.raises(zc.InvalidArgument):
        zc.linear_q8_static(q, s, x, 1, 128, zc.STATIC_MAX_K + 128, y)
    with pytest.raises(zc.InvalidArgument):
        zc.linear_q8_static(q, s, x, 1, 100, 128, y)
