"""`.zynfer` artifacts on the CPU (no GPU): the library's reader against a file
written by the reference's own converter (tests/golden/mini_bf16.zynfer, made
by tests/golden/make_artifact_golden.py), the writer against the same bytes,
the reader's rejections in the reference's order and with its error names
(validate, src/model/artifact.zig:487-532; its tests at :560-613), and the
int8 extension (format version 2) with the host packRowQ8 against the oracle's."""
import os
import struct

import numpy as np
import pytest

from oracle import oracle as O
from oracle import synth_np
from zynfer_b200 import artifact as A

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden", "mini_bf16.zynfer")
SEED = 20251202
MINI = O.Arch(vocab=8, hidden=16, inter=32, layers=1, n_q=2, n_kv=1, head_dim=8, max_pos=32, eps=1e-6,
              theta=10_000.0)


def mini_meta():
    return A.Meta(vocab_size=8, hidden_size=16, intermediate_size=32, num_hidden_layers=1, num_attention_heads=2,
                  num_key_value_heads=1, head_dim=8, max_position_embeddings=32, bos_token_id=1, eos_token_id=2,
                  rope_theta=10_000.0, rms_norm_eps=1e-6, tie_word_embeddings=True)


def mini_tensors():
    return [A.Tensor(n, A.DT_BF16, list(w.shape), synth_np.bf16_bits(w).tobytes())
            for n, w in synth_np.synth_weights(MINI, SEED, w_std=0.02, norm_std=0.1, bf16=True)]


def test_reads_the_reference_converters_file():
    with A.Artifact(GOLDEN) as art:
        m = art.meta()
        assert m.model_id == b"qwen3-0.6b" and m.format_version == 1
        assert (m.vocab, m.hidden, m.inter, m.layers, m.n_q, m.n_kv, m.head_dim) == (8, 16, 32, 1, 2, 1, 8)
        assert m.tie_word_embeddings == 1 and m.tensor_count == 13
        want = dict(synth_np.synth_weights(MINI, SEED, w_std=0.02, norm_std=0.1, bf16=True))
        names = sorted(want)
        for i, t in enumerate(art.tensors()):
            assert t.tensor_id == i + 1 and t.name.decode() == names[i]   # ids 1..N in sorted-name order
            assert t.dtype == A.DT_BF16
            assert np.array_equal(t.array().reshape(-1), synth_np.bf16_bits(want[names[i]]).reshape(-1))
        assert art.find_id(3).name.decode() == names[2] and art.find(names[2]).tensor_id == 3
        assert art.find_id(99) is None and art.find("missing") is None
        assert art.arch().hidden == 16


def test_writer_reproduces_the_reference_converter_bytes():
    with open(GOLDEN, "rb") as f:
        ref = f.read()
    assert A.build(mini_meta(), mini_tensors()) == ref


def test_stage10_fixture_round_trip(tmp_path):  # artifact.zig:534-579
    emb = np.array([0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8], np.float32)
    lm = np.array([1.0, 0.0, -1.0, 0.5], np.float32)
    p = tmp_path / "s10.zynfer"
    p.write_bytes(A.build(A.Meta(), [A.Tensor("fixture.embed", A.DT_F32, [2, 4], emb.tobytes()),
                                     A.Tensor("fixture.lm_head", A.DT_F32, [2, 2], lm.tobytes())]))
    with A.Artifact(str(p)) as art:
        assert art.meta().layers == 28 and art.meta().tensor_count == 2
        e = art.find_id(1)
        assert e.nbytes == 32 and e.array()[0, 0] == np.float32(0.1) and e.array()[1, 3] == np.float32(0.8)
        assert art.find_id(2).name == b"fixture.lm_head"


def _rehash(b: bytearray) -> bytes:
    import hashlib
    b[56:88] = b"\x00" * 32
    b[56:88] = hashlib.sha256(bytes(b)).digest()
    return bytes(b)


def _rejected(tmp_path, blob: bytes) -> str:
    p = tmp_path / "bad.zynfer"
    p.write_bytes(blob)
    with pytest.raises(A.ArtifactError) as e:
        A.Artifact(str(p))
    return str(e.value)


def test_rejections_carry_the_reference_error_names(tmp_path):
    good = bytearray(open(GOLDEN, "rb").read())
    b = bytearray(good)
    b[0:1] = b"X"                                     # magic is checked before the checksum
    assert _rejected(tmp_path, bytes(b)).startswith("InvalidMagic")
    b = bytearray(good)
    b[-1] ^= 0xFF
    assert _rejected(tmp_path, bytes(b)).startswith("ChecksumMismatch")
    b = bytearray(good)
    struct.pack_into("<H", b, 4, 3)
    assert _rejected(tmp_path, _rehash(b)).startswith("UnsupportedVersion")
    b = bytearray(good)
    b[6] = 2
    assert _rejected(tmp_path, _rehash(b)).startswith("BadEndian")
    b = bytearray(good)
    struct.pack_into("<I", b, 12, 92)                 # meta_offset
    assert _rejected(tmp_path, _rehash(b)).startswith("BadHeader")
    b = bytearray(good)
    struct.pack_into("<Q", b, 40, struct.unpack_from("<Q", b, 40)[0] + 8)
    assert _rejected(tmp_path, _rehash(b)).startswith("BadAlignment")
    assert _rejected(tmp_path, bytes(good[:-64])).startswith("Truncated")
    assert _rejected(tmp_path, bytes(good[:40])).startswith("Truncated")
    d0 = 88 + 116                                      # first directory entry
    b = bytearray(good)
    b[d0 + 69] = 0                                     # rank 0
    assert _rejected(tmp_path, _rehash(b)).startswith("InvalidRank")
    b = bytearray(good)
    b[d0 + 68] = A.DT_I8                               # int8 in a version-1 file
    assert _rejected(tmp_path, _rehash(b)).startswith("InvalidDtype")
    b = bytearray(good)
    b[d0:d0 + 64] = b"\x00" * 64                       # empty name
    assert _rejected(tmp_path, _rehash(b)).startswith("InvalidName")
    b = bytearray(good)
    struct.pack_into("<I", b, d0 + 64, 0)              # tensor id 0
    assert _rejected(tmp_path, _rehash(b)).startswith("InvalidName")
    b = bytearray(good)
    struct.pack_into("<I", b, d0 + 120 + 64, 1)        # entry 2 takes id 1 too
    assert _rejected(tmp_path, _rehash(b)).startswith("DuplicateTensorId")


def test_host_pack_row_q8_is_bit_exact():  # ops.zig:145-162
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((67, 300)) * 0.02).astype(np.float32)
    w[0] = 0.0
    w[1, :4] = [127.0, -63.5, 0.5, -0.5]
    w[1, 4:] = 0.0
    w[2] = np.float32(1e-30)
    w[3, ::2] = -w[3, 1::2]
    q, s = A.pack_row_q8(w)
    q_ref, s_ref = O.pack_row_q8(w)
    assert np.array_equal(q, q_ref) and np.array_equal(s, s_ref)


def test_quantize_writes_version_2_int8_with_scales(tmp_path):
    dst = tmp_path / "mini_q8.zynfer"
    info = A.quantize(GOLDEN, str(dst))
    assert info["int8"] == 8                            # embedding + 7 linears
    want = dict(synth_np.synth_weights(MINI, SEED, w_std=0.02, norm_std=0.1, bf16=True))
    with A.Artifact(str(dst)) as art:
        assert art.meta().format_version == 2
        for name, w in want.items():
            t = art.find(name)
            if w.ndim == 2:
                q, s = O.pack_row_q8(w)
                sc = art.find(name + ".scale")
                assert t.dtype == A.DT_I8 and np.array_equal(t.array(), q), name
                assert sc.dtype == A.DT_F32 and np.array_equal(sc.array(), s), name
            else:
                assert t.dtype == A.DT_BF16 and np.array_equal(t.array(), synth_np.bf16_bits(w)), name
    with pytest.raises(ValueError):
        A.build(mini_meta(), [A.Tensor("x", A.DT_I8, [1, 16], b"\x00" * 16)], version=1)
