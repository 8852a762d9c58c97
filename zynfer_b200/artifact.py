"""`.zynfer` model artifacts: writer, int8 converter and the device loader's binding.

The file format is the reference's (src/model/artifact.zig:42-66), written
byte for byte as its converter writes it (tools/checkpoint/safetensors_to_zynfer.py:
175-235: 88-byte header, 116-byte model record, 120-byte entries with tensor
ids 1..N in sorted-name order, 64-byte-aligned payload, SHA-256 of the file
with its own field zeroed). Format version 2 adds dtype tag 3 = int8: an int8
matrix "X" stores packRowQ8's f32 row scales (src/backends/cpu/ops.zig:145-162)
in the tensor "X.scale" [rows]. The layout is unchanged, so a version-2 file
differs only in the version field and those tensors, and the reference's own
validate() rejects it with UnsupportedVersion, as a format bump should.

Reading goes through the library (zynfer_cu_artifact_open maps and validates
the file; zynfer_cu_load_artifact uploads it to a model on the device):
`open_artifact` / `Artifact` below.

    python -m zynfer_b200.artifact inspect MODEL.zynfer
    python -m zynfer_b200.artifact quantize IN.zynfer OUT.zynfer   # every 2-D weight to int8 + scales
"""
from __future__ import annotations

import argparse
import ctypes as C
import hashlib
import struct
import sys
from dataclasses import dataclass, field

import numpy as np

MAGIC = b"ZYNF"
ENDIAN = 1
PAYLOAD_ALIGN = 64
HEADER_SIZE, META_SIZE, ENTRY_SIZE = 88, 116, 120
DT_F32, DT_F16, DT_BF16, DT_I8 = 0, 1, 2, 3
DT_SIZE = {DT_F32: 4, DT_F16: 2, DT_BF16: 2, DT_I8: 1}


def align_up(v: int, a: int) -> int:
    return (v + a - 1) // a * a


@dataclass
class Meta:
    """Meta (artifact.zig:68-99); field names follow the HF config."""
    vocab_size: int = 151936
    hidden_size: int = 1024
    intermediate_size: int = 3072
    num_hidden_layers: int = 28
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 128
    max_position_embeddings: int = 40960
    bos_token_id: int = 151643
    eos_token_id: int = 151645
    rope_theta: float = 1_000_000.0
    rms_norm_eps: float = 1e-6
    tie_word_embeddings: bool = True
    model_id: str = "qwen3-0.6b"

    def pack(self) -> bytes:
        mid = self.model_id.encode()
        return struct.pack("<64s10I2fB3x", mid + b"\x00" * (64 - len(mid)), self.vocab_size, self.hidden_size,
                           self.intermediate_size, self.num_hidden_layers, self.num_attention_heads,
                           self.num_key_value_heads, self.head_dim, self.max_position_embeddings, self.bos_token_id,
                           self.eos_token_id, float(self.rope_theta), float(self.rms_norm_eps),
                           1 if self.tie_word_embeddings else 0)


@dataclass
class Tensor:
    name: str
    dtype: int
    shape: list[int]
    data: bytes = field(repr=False)


def build(meta: Meta, tensors: list[Tensor], version: int | None = None) -> bytes:
    """The file image: tensors sorted by name, ids 1..N in that order (the
    converter's rule), every payload 64-byte aligned, SHA-256 last."""
    ts = sorted(tensors, key=lambda t: t.name)
    if version is None:
        version = 2 if any(t.dtype == DT_I8 for t in ts) else 1
    if version not in (1, 2) or (version == 1 and any(t.dtype == DT_I8 for t in ts)):
        raise ValueError("int8 tensors need format version 2")
    dir_bytes = len(ts) * ENTRY_SIZE
    dir_offset = HEADER_SIZE + META_SIZE
    payload_offset = align_up(dir_offset + dir_bytes, PAYLOAD_ALIGN)
    entries, payload, cursor = bytearray(), bytearray(), 0
    for i, t in enumerate(ts):
        raw = bytes(t.data)
        name = t.name.encode()
        if not name or len(name) >= 64 or not 1 <= len(t.shape) <= 8:
            raise ValueError(f"bad tensor {t.name!r}")
        if len(raw) != int(np.prod(t.shape)) * DT_SIZE[t.dtype]:
            raise ValueError(f"size mismatch for {t.name}")
        off = align_up(cursor, PAYLOAD_ALIGN)
        payload.extend(b"\x00" * (off - cursor))
        payload.extend(raw)
        cursor = off + len(raw)
        entries.extend(struct.pack("<64sIBB2x8IQQ", name + b"\x00" * (64 - len(name)), i + 1, t.dtype, len(t.shape),
                                   *(list(t.shape) + [0] * (8 - len(t.shape))), off, len(raw)))
    hdr = bytearray(HEADER_SIZE)
    struct.pack_into("<4sHBB", hdr, 0, MAGIC, version, ENDIAN, 0)
    struct.pack_into("<IIIIII", hdr, 8, HEADER_SIZE, HEADER_SIZE, META_SIZE, dir_offset, dir_bytes, len(ts))
    struct.pack_into("<I", hdr, 32, 0)
    struct.pack_into("<QQ", hdr, 40, payload_offset, len(payload))
    body = bytearray(hdr) + meta.pack() + entries
    body.extend(b"\x00" * (payload_offset - len(body)))
    body.extend(payload)
    body[56:88] = hashlib.sha256(bytes(body)).digest()
    return bytes(body)


def pack_row_q8(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """packRowQ8 (ops.zig:145-162) on the host, bit-exact: scale = max|w| / 127
    (1 for an all-zero row), inv = 1 / scale, q = round-half-away(w * inv)
    clamped to +-127, every step one f32 operation."""
    w = np.ascontiguousarray(w, np.float32)
    mx = np.max(np.abs(w), axis=1)
    scale = np.where(mx == 0, np.float32(1.0), mx / np.float32(127.0)).astype(np.float32)
    inv = (np.float32(1.0) / scale).astype(np.float32)
    prod = (w * inv[:, None]).astype(np.float32)
    a = np.abs(prod).astype(np.float64)                    # exact: f32 values below 2^24
    q = np.sign(prod).astype(np.float64) * np.floor(a + 0.5)
    return np.clip(q, -127, 127).astype(np.int8), scale


def bf16_to_f32(raw: bytes) -> np.ndarray:
    u = np.frombuffer(raw, np.uint16).astype(np.uint32) << np.uint32(16)
    return u.view(np.float32)


# ------------------------------------------------------------ the library side
class ArtifactMeta(C.Structure):
    _fields_ = [("model_id", C.c_char * 64), ("format_version", C.c_uint32), ("vocab", C.c_uint32),
                ("hidden", C.c_uint32), ("inter", C.c_uint32), ("layers", C.c_uint32), ("n_q", C.c_uint32),
                ("n_kv", C.c_uint32), ("head_dim", C.c_uint32), ("max_pos", C.c_uint32), ("bos", C.c_uint32),
                ("eos", C.c_uint32), ("rope_theta", C.c_float), ("rms_norm_eps", C.c_float),
                ("tie_word_embeddings", C.c_uint32), ("tensor_count", C.c_uint32), ("file_bytes", C.c_uint64)]


class TensorInfo(C.Structure):
    _fields_ = [("name", C.c_char * 64), ("tensor_id", C.c_uint32), ("dtype", C.c_uint32), ("rank", C.c_uint32),
                ("shape", C.c_uint32 * 8), ("nbytes", C.c_uint64), ("data", C.c_void_p)]

    def array(self) -> np.ndarray:
        """The tensor's bytes in the mapped file as a numpy array (no copy)."""
        dt = {DT_F32: np.float32, DT_F16: np.float16, DT_BF16: np.uint16, DT_I8: np.int8}[self.dtype]
        buf = (C.c_uint8 * self.nbytes).from_address(self.data)
        return np.frombuffer(buf, dt).reshape([self.shape[i] for i in range(self.rank)])


class ArtifactError(ValueError):
    """A file the reader rejected; str() starts with the reference's error name."""


class Artifact:
    """An open artifact (zynfer_cu_artifact_open): validated, mapped read-only."""

    def __init__(self, path: str):
        from . import cuda
        self._lib = cuda.lib()
        h = C.c_void_p()
        rc = self._lib.zynfer_cu_artifact_open(str(path).encode(), C.byref(h))
        self.h = h
        if rc != cuda.OK:
            msg = self._lib.zynfer_cu_artifact_error(h).decode()
            self._lib.zynfer_cu_artifact_close(h)
            self.h = None
            raise ArtifactError(msg)

    def meta(self) -> ArtifactMeta:
        m = ArtifactMeta()
        if self._lib.zynfer_cu_artifact_meta(self.h, C.byref(m)):
            raise ArtifactError("meta")
        return m

    def tensors(self) -> list[TensorInfo]:
        out = []
        for i in range(self.meta().tensor_count):
            t = TensorInfo()
            self._lib.zynfer_cu_artifact_tensor(self.h, i, C.byref(t))
            out.append(t)
        return out

    def find_id(self, tensor_id: int) -> TensorInfo | None:
        t = TensorInfo()
        return t if self._lib.zynfer_cu_artifact_find_id(self.h, tensor_id, C.byref(t)) == 0 else None

    def find(self, name: str) -> TensorInfo | None:
        t = TensorInfo()
        return t if self._lib.zynfer_cu_artifact_find_name(self.h, name.encode(), C.byref(t)) == 0 else None

    def arch(self):
        """The model architecture (Meta.toArch, artifact.zig:101-121) as a cuda.Arch."""
        from . import cuda
        m = self.meta()
        return cuda.Arch(vocab=m.vocab, hidden=m.hidden, inter=m.inter, layers=m.layers, n_q=m.n_q, n_kv=m.n_kv,
                         head_dim=m.head_dim, max_pos=m.max_pos, eps=float(m.rms_norm_eps),
                         theta=float(m.rope_theta))

    def close(self):
        if self.h:
            self._lib.zynfer_cu_artifact_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def open_artifact(path: str) -> Artifact:
    return Artifact(path)


# ------------------------------------------------------------------- tools
def quantize(src: str, dst: str) -> dict:
    """Rewrite an artifact with every 2-D tensor (the linears and the tied
    embedding) as int8 + row scales (format version 2); vectors stay as they are."""
    out, n_q8 = [], 0
    with Artifact(src) as art:
        m = art.meta()
        meta = Meta(m.vocab, m.hidden, m.inter, m.layers, m.n_q, m.n_kv, m.head_dim, m.max_pos, m.bos, m.eos,
                    float(m.rope_theta), float(m.rms_norm_eps), bool(m.tie_word_embeddings),
                    m.model_id.decode())
        for t in art.tensors():
            name = t.name.decode()
            shape = [t.shape[i] for i in range(t.rank)]
            a = t.array()
            if t.rank == 2 and t.dtype in (DT_F32, DT_BF16):
                w = bf16_to_f32(a.tobytes()).reshape(shape) if t.dtype == DT_BF16 else np.asarray(a, np.float32)
                q, s = pack_row_q8(w)
                out.append(Tensor(name, DT_I8, shape, q.tobytes()))
                out.append(Tensor(name + ".scale", DT_F32, [shape[0]], s.tobytes()))
                n_q8 += 1
            else:
                out.append(Tensor(name, t.dtype, shape, a.tobytes()))
    blob = build(meta, out)
    with open(dst, "wb") as f:
        f.write(blob)
    return {"tensors": len(out), "int8": n_q8, "bytes": len(blob)}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    ins = sub.add_parser("inspect")
    ins.add_argument("path")
    qz = sub.add_parser("quantize")
    qz.add_argument("src")
    qz.add_argument("dst")
    args = ap.parse_args(argv)
    if args.cmd == "inspect":
        with Artifact(args.path) as art:
            m = art.meta()
            print(f"{m.model_id.decode()} v{m.format_version}: {m.tensor_count} tensors, {m.file_bytes} bytes, "
                  f"hidden {m.hidden}, layers {m.layers}, vocab {m.vocab}")
            for t in art.tensors():
                shape = "x".join(str(t.shape[i]) for i in range(t.rank))
                print(f"  {t.tensor_id:5d} {t.name.decode():48s} dtype {t.dtype} {shape}")
    else:
        print(quantize(args.src, args.dst))


if __name__ == "__main__":
    sys.exit(main())
