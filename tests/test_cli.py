"""The command line (zynfer_b200/cli.py) on the CPU: backend resolution as the
reference's main.zig does it (unknown names and unbuilt kinds fail, no CPU
fallback), decode-bench's JSON key set against block-bench's
(main.zig:1211-1245), compare.zig's rule and topK's order as forward-golden
uses them (main.zig:412-505)."""
import io
import json

import numpy as np
import pytest

from zynfer_b200 import cli


def test_backend_resolution_fails_loudly(monkeypatch):
    monkeypatch.delenv("ZYNFER_BACKEND", raising=False)
    assert cli.resolve("cuda").value == "cuda"
    with pytest.raises(SystemExit) as e:
        cli.resolve("bogus")
    assert e.value.code == 2
    with pytest.raises(SystemExit):
        cli.resolve("cpu")            # the reference's CPU kind is not part of this build: no fallback
    monkeypatch.setenv("ZYNFER_BACKEND", "metal")
    with pytest.raises(SystemExit):
        cli.resolve(None)             # the environment switch resolves the same way


def test_decode_bench_json_carries_block_bench_keys():
    line = cli.block_bench_json(kind="cuda", hidden=1024, prefill_tokens=512, decode_steps=32, warmup=1, iters=3,
                                cuda_init_ns=5, cuda_prefill_ns=4_000_000, cuda_decode_ns_per_token=900_000,
                                cuda_block_path="generate:gemv+tcgen05:graph", batch=1, launches=144)
    for k in cli.BLOCK_BENCH_KEYS + cli.CUDA_KEYS:
        assert k in line, k
    assert line["apple_prefill_ns"] is None and line["metal_init_ns"] is None and line["energy_per_token"] is None
    assert line["peak_rss_bytes"] > 0
    assert json.loads(json.dumps(line)) == line


def test_expect_close_is_compare_zig():
    e = np.array([1.0, -2.0, 3.0], np.float32)
    ok, d, i = cli.expect_close(e, e + np.float32(0.25), 0.3, 0.0)
    assert ok and i == 2 and d == 0.25        # the last index among equal differences
    ok, d, i = cli.expect_close(e, np.array([1.0, -2.5, 3.0], np.float32), 1e-3, 1e-2)
    assert not ok and i == 1 and abs(d - 0.5) < 1e-6


def test_top_k_orders_like_the_reference():
    logits = np.array([0.5, 2.0, -np.inf, 2.0, 1.0], np.float32)
    assert cli.top_k(logits, 3) == [(1, 2.0), (3, 2.0), (4, 1.0)]   # first maximum first
    assert len(cli.top_k(logits, 8)) == 4                              # -inf never listed


def test_forward_golden_rejects_dump_and_bad_artifacts(tmp_path):
    with pytest.raises(SystemExit):
        cli.main(["forward-golden", "x.zynfer", "--dump", str(tmp_path), "--backend", "cuda"])
    p = tmp_path / "bad.zynfer"
    p.write_bytes(b"XYNF" + b"\x00" * 200)
    with pytest.raises(SystemExit):
        cli.main(["forward-golden", str(p), "--backend", "cuda"])


def test_backends_lists_every_kind():
    out = io.StringIO()
    cli.backends(None, out)
    text = out.getvalue()
    for k in ("cpu", "apple", "amd-hip", "cuda"):
        assert k in text
