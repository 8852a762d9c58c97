"""`.zynfer` artifacts loaded straight to the device (B200 only): a small
Qwen3-shaped model written as an artifact (f32, bf16, and int8 + scales in
format version 2) and uploaded by zynfer_cu_load_artifact gives the same
weights, and so bit-identical logits, as the same seeded weights generated on
the device by zynfer_cu_fill_synthetic (Weights.load, qwen_weights.zig:61-175;
the int8 path packs with packRowQ8's arithmetic on either side)."""
import os

import numpy as np
import pytest

from oracle import oracle as O
from oracle import synth_np
from zynfer_b200 import artifact as A
from zynfer_b200 import cuda as zc

pytestmark = pytest.mark.gpu

SMALL = dict(vocab=4096, hidden=512, inter=1024, layers=2, n_q=4, n_kv=2, head_dim=128, max_pos=4096, eps=1e-6,
             theta=1_000_000.0)
SEED, WSTD, NSTD = 11, 0.05, 0.1
# the device generator derives its scale from the f32 std the C ABI receives;
# the host generator gets the same f32 value, so both produce identical weights
WSTD32, NSTD32 = float(np.float32(WSTD)), float(np.float32(NSTD))


def _meta():
    a = SMALL
    return A.Meta(vocab_size=a["vocab"], hidden_size=a["hidden"], intermediate_size=a["inter"],
                  num_hidden_layers=a["layers"], num_attention_heads=a["n_q"], num_key_value_heads=a["n_kv"],
                  head_dim=a["head_dim"], max_position_embeddings=a["max_pos"], rope_theta=a["theta"],
                  rms_norm_eps=a["eps"])


def _write(path, dtype, bf16_values):
    ts = []
    for name, w in synth_np.synth_weights(O.Arch(**SMALL), SEED, w_std=WSTD32, norm_std=NSTD32, bf16=bf16_values):
        if dtype == A.DT_BF16:
            ts.append(A.Tensor(name, A.DT_BF16, list(w.shape), synth_np.bf16_bits(w).tobytes()))
        elif dtype == A.DT_I8 and w.ndim == 2:
            q, s = A.pack_row_q8(w)
            ts.append(A.Tensor(name, A.DT_I8, list(w.shape), q.tobytes()))
            ts.append(A.Tensor(name + ".scale", A.DT_F32, [w.shape[0]], s.tobytes()))
        else:
            ts.append(A.Tensor(name, A.DT_F32, list(w.shape), np.ascontiguousarray(w, np.float32).tobytes()))
    with open(path, "wb") as f:
        f.write(A.build(_meta(), ts))


def _logits(model, ids):
    logits, _ = model.prefill(0, ids)
    am = model.decode_step([0], [7], want_logits=True)[1][0]
    return logits, am


@pytest.mark.parametrize("kind", ["f32", "int8"])
def test_int8_model_from_artifact_equals_device_fill(tmp_path, kind):
    path = str(tmp_path / f"small_{kind}.zynfer")
    _write(path, A.DT_F32 if kind == "f32" else A.DT_I8, bf16_values=False)
    ids = O.synth_tokens(29, SEED, 3, SMALL["vocab"])
    ref = zc.Model(zc.Gpu(0), zc.Arch(**SMALL), zc.W_Q8, max_batch=1, max_seqs=1, max_seq_len=64)
    ref.fill_synthetic(SEED, WSTD, NSTD)
    want = _logits(ref, ids)
    with A.Artifact(path) as art:
        assert art.meta().format_version == (2 if kind == "int8" else 1)
        m = zc.Model(zc.Gpu(0), art.arch(), zc.W_Q8, max_batch=1, max_seqs=1, max_seq_len=64)
        m.load_artifact(art)
    for name, (r, c) in [("model.embed_tokens.weight", (4096, 512)), ("model.layers.1.mlp.down_proj.weight", (512, 1024))]:
        q, s = m.download_q8(name, r, c)
        q2, s2 = ref.download_q8(name, r, c)
        assert np.array_equal(q, q2) and np.array_equal(s, s2), name
    got = _logits(m, ids)
    assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1])


def test_bf16_model_from_artifact_equals_device_fill(tmp_path):
    path = str(tmp_path / "small_bf16.zynfer")
    _write(path, A.DT_BF16, bf16_values=True)
    ids = O.synth_tokens(17, SEED, 5, SMALL["vocab"])
    ref = zc.Model(zc.Gpu(0), zc.Arch(**SMALL), zc.W_BF16, max_batch=1, max_seqs=1, max_seq_len=64)
    ref.fill_synthetic(SEED, WSTD, NSTD)
    with A.Artifact(path) as art:
        m = zc.Model(zc.Gpu(0), art.arch(), zc.W_BF16, max_batch=1, max_seqs=1, max_seq_len=64)
        m.load_artifact(art)
    a, b = _logits(ref, ids), _logits(m, ids)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def test_missing_tensor_and_wrong_architecture_are_reported(tmp_path):
    path = str(tmp_path / "partial.zynfer")
    ts = [A.Tensor(n, A.DT_F32, list(w.shape), np.ascontiguousarray(w, np.float32).tobytes())
          for n, w in synth_np.synth_weights(O.Arch(**SMALL), SEED, w_std=WSTD32, norm_std=NSTD32)
          if n != "model.layers.1.self_attn.k_norm.weight"]
    with open(path, "wb") as f:
        f.write(A.build(_meta(), ts))
    gpu = zc.Gpu(0)
    m = zc.Model(gpu, zc.Arch(**SMALL), zc.W_Q8, max_batch=1, max_seqs=1, max_seq_len=64)
    with A.Artifact(path) as art:
        with pytest.raises(zc.InvalidArgument, match="TensorNotFound: model.layers.1.self_attn.k_norm.weight"):
            m.load_artifact(art)
    other = zc.Model(zc.Gpu(0), zc.Arch(**dict(SMALL, layers=1)), zc.W_Q8, max_batch=1, max_seqs=1,
                     max_seq_len=64)
    with A.Artifact(path) as art:
        with pytest.raises(zc.InvalidArgument, match="ShapeMismatch"):
            other.load_artifact(art)
    os.remove(path)


def test_cli_forward_golden_and_decode_bench(tmp_path, capsys):
    """zynfer forward-golden / decode-bench --backend cuda (main.zig:412-505, 1150-1245)."""
    import json

    from zynfer_b200 import cli
    path = str(tmp_path / "small_bf16.zynfer")
    _write(path, A.DT_BF16, bf16_values=True)
    ids = [int(t) for t in O.synth_tokens(9, SEED, 7, SMALL["vocab"])]
    ref = O.Model(O.Arch(**SMALL), O.W_BF16, kv_bf16=False, seed=SEED, w_std=WSTD, norm_std=NSTD)
    want = ref.session(16).prefill_last_logits(ids)
    ref.close()
    gold = str(tmp_path / "golden.f32")
    want.astype("<f4").tofile(gold)
    assert cli.main(["forward-golden", path, "--tokens", ",".join(map(str, ids)), "--golden", gold,
                     "--backend", "cuda"]) == 0
    out = capsys.readouterr().out
    assert "golden OK" in out
    top = out.split("top logits (last token):\n")[1].splitlines()[0]
    assert top.strip().startswith(f"id={int(np.argmax(want))} ")
    assert cli.main(["decode-bench", "--backend", "cuda", "--artifact", path, "--batch", "2",
                     "--prefill-tokens", "32", "--decode-steps", "4", "--warmup", "1", "--iters", "2"]) == 0
    out = capsys.readouterr().out
    line = json.loads(out.split("json\n")[1].splitlines()[0])
    assert line["backend"] == "cuda" and line["cuda_batch"] == 2
    assert line["cuda_decode_ns_per_token"] > 0 and line["cuda_prefill_ns"] > 0
    assert all(k in line for k in cli.BLOCK_BENCH_KEYS)
