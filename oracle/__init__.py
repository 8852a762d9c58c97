"""The oracle: a CPU restatement of the Zynfer reference's f32 Qwen3 path.

TEST INFRASTRUCTURE ONLY. tests/, ``__graft_entry__.smoke()`` and bench.py's
CPU-baseline leg load it as the checker; the product package ``zynfer_b200``
never imports it and has no CPU fallback.
"""
