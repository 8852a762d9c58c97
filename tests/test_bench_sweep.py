"""CPU checks of bench.py (no GPU): the int8 linear sweep mode (the shapes it
covers and its CPU leg, the oracle's matvecQ8 / matmulQ8, ops.zig:181-228),
the byte and FLOP counts behind the batch-1 and prefill roofline figures, and
the --case arguments."""
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


def test_decode_bytes_per_token():
    # 598.2 MB of int8 weights, scales and norms per token; KV 114,688 B per position
    assert abs(bench.WEIGHT_BYTES_PER_TOKEN / 1e6 - 598.2) < 0.1
    assert 28 * bench.KV_BYTES_PER_TOKEN_LAYER == 114688
    # one sequence at context 2048 + 256 steps: mean 2176.5 positions -> 847.8 MB per token
    mean_kv = bench.BATCH1_CTX + (bench.BATCH1_STEPS + 1) / 2.0
    assert mean_kv == 2176.5
    assert abs((bench.WEIGHT_BYTES_PER_TOKEN + mean_kv * 114688) / 1e6 - 847.8) < 0.1


def test_prefill_flops_512():
    # linears 2 x 440.4 M params x 512, causal attention 30.1 GFLOP, LM head on the last row
    f = bench.prefill_flops(512)
    assert abs(f / 1e9 - 481.4) < 0.5
    assert 28 * bench.LINEAR_PARAMS_PER_LAYER == 440401920


def test_case_arguments(monkeypatch):
    monkeypatch.setattr(sys, "argv", ["bench.py", "--case", "32,2048,2", "--steps", "2", "--warmup", "3",
                                      "--schedule", "persistent", "--phases"])
    a = bench.parse()
    assert a.case == "32,2048,2" and a.steps == 2 and a.schedule == "persistent" and a.phases
    assert tuple(int(v) for v in a.case.split(",")) == (32, 2048, 2)


def test_clock_sampler_reports_missing_sources():
    # without NVML and without nvidia-smi the line says so instead of inventing clocks
    s = bench.ClockSampler("GPU-00000000-0000-0000-0000-000000000000")
    s.nvml = None
    import subprocess
    orig = subprocess.Popen

    def no_smi(*a, **k):
        raise FileNotFoundError("nvidia-smi")
    subprocess.Popen = no_smi
    try:
        s.start()
        out = s.stop()
    finally:
        subprocess.Popen = orig
    assert out["samples"] == 0 and out["sm_mhz"] is None and out["reasons"] == ["no clock source"]


def test_clock_sampler_summarises_samples():
    s = bench.ClockSampler("GPU-00000000-0000-0000-0000-000000000000")
    s.nvml = None
    s.proc = None
    s.samples = [(1965.0, 1965.0, set()), (1800.0, 1965.0, {"sw_power_cap"}), (1965.0, 1965.0, set())]
    s.nvml = object()  # take the NVML branch of stop(): no thread to join
    s._t = type("T", (), {"join": lambda self, timeout=None: None})()
    out = s.stop()
    assert out["sm_mhz"] == 1965.0 and out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"] and out["samples"] == 3
