"""CPU checks of bench.py's int8 linear sweep mode (no GPU): the shapes it
covers and its CPU leg (the oracle's matvecQ8 / matmulQ8, ops.zig:181-228)."""
import sys

import bench


def test_sweep_covers_the_linear_shapes():
    # QKV as specified (2048+512+512) and as the model has it (2048+1024+1024),
    # then O, gate/up, down and the tied LM head
    assert bench.GEMV_SHAPES == [(3072, 1024), (4096, 1024), (1024, 2048), (6144, 1024), (1024, 3072),
                                 (151936, 1024)]
    for m, k in bench.GEMV_SHAPES:
        assert m % 128 == 0 and k % 512 == 0  # zynfer_cu_linear's int8 shape rules


def test_sweep_rotation_exceeds_l2():
    for m, k in bench.GEMV_SHAPES:
        copies = max(2, -(-2 * bench.L2_BYTES // (m * k)))
        assert copies * m * k >= 2 * bench.L2_BYTES


def test_sweep_arguments(monkeypatch):
    monkeypatch.setattr(sys, "argv", ["bench.py", "--sweep", "gemv", "--sweep-shape", "6144x1024",
                                      "--sweep-calls", "10"])
    args = bench.parse()
    assert args.sweep == "gemv" and args.sweep_shape == "6144x1024" and args.sweep_calls == 10
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    assert bench.parse().sweep is None  # the default run stays the one-line benchmark


def test_cpu_leg_times_one_and_eight_rows():
    assert 0.0 < bench.cpu_linear_us(1024, 1024, 1, budget_s=0.05)
    assert 0.0 < bench.cpu_linear_us(1024, 1024, 8, budget_s=0.05)
