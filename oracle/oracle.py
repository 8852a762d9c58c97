"""ctypes binding of the oracle library (test infrastructure, the checker).

Follows the reference's CPU oracle (src/backends/cpu/ops.zig, src/model/qwen_*.zig)
through ``libzynfer_oracle.so``; see zynfer_oracle.h for the per-function
citations. Never used by the product path.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libzynfer_oracle.so")
_lib = None

F32P = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
I8P = np.ctypeslib.ndpointer(dtype=np.int8, flags="C_CONTIGUOUS")
U32P = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
SZ = C.c_size_t


def build() -> str:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


class ZoArch(C.Structure):
    _fields_ = [
        ("vocab", C.c_uint32), ("hidden", C.c_uint32), ("inter", C.c_uint32),
        ("layers", C.c_uint32), ("n_q", C.c_uint32), ("n_kv", C.c_uint32),
        ("head_dim", C.c_uint32), ("max_pos", C.c_uint32),
        ("eps", C.c_float), ("theta", C.c_float),
    ]


class ZoDiff(C.Structure):
    _fields_ = [
        ("max_abs", C.c_float), ("max_rel", C.c_float), ("rms", C.c_float),
        ("failing_index", C.c_size_t), ("expected", C.c_float), ("actual", C.c_float),
    ]


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        build()
    L = C.CDLL(_LIB_PATH)
    L.zo_add.argtypes = [F32P, F32P, F32P, SZ]
    L.zo_silu_scalar.argtypes = [C.c_float]
    L.zo_silu_scalar.restype = C.c_float
    L.zo_silu_mul.argtypes = [F32P, F32P, F32P, SZ]
    L.zo_rms_norm.argtypes = [F32P, F32P, F32P, SZ, SZ, C.c_float]
    L.zo_softmax.argtypes = [F32P, F32P, SZ, SZ]
    L.zo_matmul_f32.argtypes = [F32P, F32P, F32P, SZ, SZ, SZ, C.c_int]
    L.zo_matvec_f32.argtypes = [F32P, F32P, F32P, SZ, SZ]
    L.zo_pack_row_q8.argtypes = [F32P, SZ, SZ, I8P, F32P]
    L.zo_pack_tensor_q8.argtypes = [F32P, SZ, SZ, I8P, F32P]
    L.zo_matvec_q8.argtypes = [F32P, I8P, F32P, F32P, SZ, SZ, C.c_int, C.c_int]
    L.zo_matmul_q8.argtypes = [F32P, I8P, F32P, F32P, SZ, SZ, SZ, C.c_int]
    L.zo_rope.argtypes = [F32P, SZ, SZ, SZ, SZ, C.c_float]
    L.zo_attention_into.argtypes = [F32P, F32P, F32P, F32P, SZ, SZ, SZ, SZ, SZ, SZ, F32P, C.c_int]
    L.zo_attention_into.restype = C.c_int
    L.zo_tokens_heads_to_heads_tokens.argtypes = [F32P, F32P, SZ, SZ, SZ]
    L.zo_heads_tokens_to_tokens_heads.argtypes = [F32P, F32P, SZ, SZ, SZ]
    L.zo_embedding_gather.argtypes = [F32P, F32P, SZ, SZ, U32P, SZ]
    L.zo_embedding_gather.restype = C.c_int
    L.zo_bf16_to_f32.argtypes = [C.c_uint16]
    L.zo_bf16_to_f32.restype = C.c_float
    L.zo_f32_to_bf16_rne.argtypes = [C.c_float]
    L.zo_f32_to_bf16_rne.restype = C.c_uint16
    L.zo_diff_f32.argtypes = [F32P, F32P, SZ, C.POINTER(ZoDiff)]
    L.zo_expect_close.argtypes = [F32P, F32P, SZ, C.c_float, C.c_float]
    L.zo_expect_close.restype = C.c_int
    L.zo_top_k.argtypes = [F32P, SZ, SZ, U32P, F32P]
    L.zo_sample_row.argtypes = [F32P, SZ, C.c_float, C.c_uint32, C.c_float, C.c_uint64, C.c_uint32, C.c_uint32,
                                C.POINTER(C.c_uint32)]
    L.zo_sample_row.restype = C.c_int
    L.zo_synth_normal.argtypes = [F32P, SZ, C.c_uint64, C.c_uint64, C.c_float]
    L.zo_synth_tokens.argtypes = [U32P, SZ, C.c_uint64, C.c_uint64, C.c_uint32]
    L.zo_model_create.argtypes = [C.POINTER(ZoArch), C.c_int, C.c_int, C.c_int]
    L.zo_model_create.restype = C.c_void_p
    L.zo_model_create_synthetic.argtypes = [C.POINTER(ZoArch), C.c_int, C.c_int, C.c_uint64,
                                            C.c_float, C.c_float, C.c_int]
    L.zo_model_create_synthetic.restype = C.c_void_p
    L.zo_model_destroy.argtypes = [C.c_void_p]
    L.zo_model_set_tensor.argtypes = [C.c_void_p, C.c_char_p, F32P, SZ, SZ]
    L.zo_model_set_tensor.restype = C.c_int
    L.zo_model_get_q8.argtypes = [C.c_void_p, C.c_char_p, I8P, F32P, SZ, SZ]
    L.zo_model_get_q8.restype = C.c_int
    L.zo_model_set_threads.argtypes = [C.c_void_p, C.c_int]
    L.zo_session_create.argtypes = [C.c_void_p, SZ]
    L.zo_session_create.restype = C.c_void_p
    L.zo_session_destroy.argtypes = [C.c_void_p]
    L.zo_session_reset.argtypes = [C.c_void_p]
    L.zo_session_used.argtypes = [C.c_void_p]
    L.zo_session_used.restype = SZ
    L.zo_session_forward.argtypes = [C.c_void_p, U32P, SZ, C.c_void_p, C.c_void_p, C.c_void_p]
    L.zo_session_forward.restype = C.c_int
    L.zo_session_block.argtypes = [C.c_void_p, C.c_uint32, F32P, SZ, F32P]
    L.zo_session_block.restype = C.c_int
    L.zo_prefill_last_logits.argtypes = [C.c_void_p, U32P, SZ, F32P]
    L.zo_prefill_last_logits.restype = C.c_int
    L.zo_greedy_decode.argtypes = [C.c_void_p, C.c_uint32, SZ, C.c_void_p, U32P, C.c_void_p]
    L.zo_greedy_decode.restype = C.c_int
    L.zo_session_fill_kv.argtypes = [C.c_void_p, SZ, C.c_uint64]
    L.zo_session_fill_kv.restype = C.c_int
    L.zo_session_kv.argtypes = [C.c_void_p, C.c_uint32, C.c_int, F32P]
    L.zo_session_kv.restype = C.c_int
    _lib = L
    return L


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ----------------------------------------------------------------- ops
def rms_norm(x, w, eps=1e-6):
    x = f32(x)
    y = np.empty_like(x)
    cols = x.shape[-1]
    lib().zo_rms_norm(y, x, f32(w), x.size // cols, cols, eps)
    return y


def silu_mul(g, u):
    g, u = f32(g), f32(u)
    o = np.empty_like(g)
    lib().zo_silu_mul(o, g, u, g.size)
    return o


def softmax(x):
    x = f32(x)
    y = np.empty_like(x)
    lib().zo_softmax(y, x, x.size // x.shape[-1], x.shape[-1])
    return y


def matmul(a, b, threads=1):
    a, b = f32(a), f32(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.float32)
    lib().zo_matmul_f32(c, a, b, m, n, k, threads)
    return c


def matvec(a, x):
    a, x = f32(a), f32(x)
    y = np.empty(a.shape[0], np.float32)
    lib().zo_matvec_f32(y, a, x, a.shape[0], a.shape[1])
    return y


def pack_row_q8(w):
    w = f32(w)
    m, k = w.shape
    q = np.empty((m, k), np.int8)
    s = np.empty(m, np.float32)
    lib().zo_pack_row_q8(w, m, k, q, s)
    return q, s


def pack_tensor_q8(w):
    w = f32(w)
    m, k = w.shape
    q = np.empty((m, k), np.int8)
    s = np.empty(1, np.float32)
    lib().zo_pack_tensor_q8(w, m, k, q, s)
    return q, s


def matvec_q8(q, s, x, threads=1):
    q = np.ascontiguousarray(q, np.int8)
    m, k = q.shape
    y = np.empty(m, np.float32)
    s = f32(s)
    lib().zo_matvec_q8(y, q, s, f32(x), m, k, 1 if s.size == 1 and m > 1 else 0, threads)
    return y


def matmul_q8(q, s, b):
    q = np.ascontiguousarray(q, np.int8)
    b = f32(b)
    m, k = q.shape
    n = b.shape[1]
    c = np.empty((m, n), np.float32)
    s = f32(s)
    lib().zo_matmul_q8(c, q, s, b, m, n, k, 1 if s.size == 1 and m > 1 else 0)
    return c


def rope(x, pos0, theta):
    """x: [tokens, heads, d] (rotated copy returned)."""
    x = f32(x).copy()
    t, h, d = x.shape
    lib().zo_rope(x, t, h, d, pos0, theta)
    return x


def attention_into(q, k, v, kv_len, threads=1):
    """q [n_q, q_len, d]; k, v [n_kv, kv_stride, d] -> out [n_q, q_len, d]."""
    q, k, v = f32(q), f32(k), f32(v)
    n_q, q_len, d = q.shape
    n_kv, stride, _ = k.shape
    out = np.empty_like(q)
    scores = np.empty(max(threads, 1) * max(kv_len, 1), np.float32)
    rc = lib().zo_attention_into(out, q, k, v, n_q, q_len, d, n_kv, kv_len, stride, scores, threads)
    if rc:
        raise ValueError(f"attentionInto rejected the shapes (status {rc})")
    return out


def embedding_gather(table, ids):
    table = f32(table)
    ids = np.ascontiguousarray(ids, np.uint32)
    out = np.empty((ids.size, table.shape[1]), np.float32)
    rc = lib().zo_embedding_gather(out, table, table.shape[0], table.shape[1], ids, ids.size)
    if rc:
        raise ValueError("token id out of range")
    return out


def bf16_round(x):
    """f32 -> bf16 (RNE) -> f32 through the oracle's scalar conversion."""
    x = f32(x)
    L = lib()
    return np.array([L.zo_bf16_to_f32(L.zo_f32_to_bf16_rne(float(v))) for v in x.ravel()],
                    np.float32).reshape(x.shape)


def diff(expected, actual) -> ZoDiff:
    e, a = f32(expected).ravel(), f32(actual).ravel()
    d = ZoDiff()
    lib().zo_diff_f32(e, a, e.size, C.byref(d))
    return d


def expect_close(expected, actual, atol, rtol) -> bool:
    e, a = f32(expected).ravel(), f32(actual).ravel()
    return bool(lib().zo_expect_close(e, a, e.size, atol, rtol))


def top_k(logits, k):
    logits = f32(logits)
    ids = np.empty(k, np.uint32)
    vals = np.empty(k, np.float32)
    lib().zo_top_k(logits, logits.size, k, ids, vals)
    return ids, vals


def sample_row(logits, temperature, top_k, top_p, seed, slot, pos):
    """Extension: one sampled token id (zo_sample_row); inv_t = 1/temperature in f32."""
    logits = f32(logits)
    out = C.c_uint32()
    inv_t = float(np.float32(1.0) / np.float32(temperature))
    lib().zo_sample_row(logits, logits.size, inv_t, top_k, top_p, seed, slot, pos, C.byref(out))
    return int(out.value)


def synth_normal(n, seed, stream, std):
    out = np.empty(n, np.float32)
    lib().zo_synth_normal(out, n, seed, stream, std)
    return out


def synth_tokens(n, seed, stream, vocab):
    out = np.empty(n, np.uint32)
    lib().zo_synth_tokens(out, n, seed, stream, vocab)
    return out


# --------------------------------------------------------------- model
W_F32, W_BF16, W_Q8 = 0, 1, 2


@dataclass(frozen=True)
class Arch:
    """qwen3.zig:36-59."""
    vocab: int = 151936
    hidden: int = 1024
    inter: int = 3072
    layers: int = 28
    n_q: int = 16
    n_kv: int = 8
    head_dim: int = 128
    max_pos: int = 40960
    eps: float = 1e-6
    theta: float = 1_000_000.0

    def c(self) -> ZoArch:
        return ZoArch(self.vocab, self.hidden, self.inter, self.layers, self.n_q, self.n_kv,
                      self.head_dim, self.max_pos, self.eps, self.theta)


QWEN3_0_6B = Arch()  # qwen3.zig:19-34
STAGE11_MINI = Arch(vocab=8, hidden=16, inter=32, layers=1, n_q=2, n_kv=1, head_dim=8,
                    max_pos=32, eps=1e-6, theta=10_000.0)  # qwen3.zig:69-84


class Model:
    def __init__(self, arch: Arch, wkind: int, kv_bf16: bool = False, seed: int | None = None,
                 w_std: float = 0.02, norm_std: float = 0.0, threads: int = 1):
        self.arch = arch
        self.wkind = wkind
        self._arch_c = arch.c()
        L = lib()
        if seed is None:
            self.h = L.zo_model_create(C.byref(self._arch_c), wkind, int(kv_bf16), threads)
        else:
            self.h = L.zo_model_create_synthetic(C.byref(self._arch_c), wkind, int(kv_bf16), seed,
                                                 w_std, norm_std, threads)
        if not self.h:
            raise MemoryError("oracle model allocation failed")

    def set_tensor(self, name: str, data):
        data = f32(data)
        rows, cols = (data.shape[0], data.shape[1]) if data.ndim == 2 else (data.size, 1)
        rc = lib().zo_model_set_tensor(self.h, name.encode(), data, rows, cols)
        if rc:
            raise ValueError(f"set_tensor({name}) failed: {rc}")

    def get_q8(self, name: str, rows: int, cols: int):
        q = np.empty((rows, cols), np.int8)
        s = np.empty(rows, np.float32)
        rc = lib().zo_model_get_q8(self.h, name.encode(), q, s, rows, cols)
        if rc:
            raise ValueError(f"get_q8({name}) failed: {rc}")
        return q, s

    def set_threads(self, n: int):
        lib().zo_model_set_threads(self.h, n)

    def session(self, max_seq: int) -> "Session":
        return Session(self, max_seq)

    def close(self):
        if self.h:
            lib().zo_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Session:
    def __init__(self, model: Model, max_seq: int):
        self.model = model
        self.h = lib().zo_session_create(model.h, max_seq)
        if not self.h:
            raise ValueError("invalid max_seq")

    @property
    def used(self) -> int:
        return int(lib().zo_session_used(self.h))

    def reset(self):
        lib().zo_session_reset(self.h)

    def forward(self, ids, want_logits=True, dump=False):
        a = self.model.arch
        ids = np.ascontiguousarray(ids, np.uint32)
        logits = np.empty(a.vocab, np.float32) if want_logits else None
        layers = np.empty((a.layers, a.hidden), np.float32) if dump else None
        normed = np.empty(a.hidden, np.float32) if dump else None
        ptr = lambda x: None if x is None else x.ctypes.data_as(C.c_void_p)  # noqa: E731
        rc = lib().zo_session_forward(self.h, ids, ids.size, ptr(logits), ptr(layers), ptr(normed))
        if rc:
            raise ValueError(f"forward rejected (status {rc})")
        if dump:
            return logits, layers, normed
        return logits

    def block(self, layer: int, x):
        """One layer's forward on hidden states x [t, hidden] (qwen_block.zig:161-235)."""
        x = f32(x)
        out = np.empty_like(x)
        rc = lib().zo_session_block(self.h, layer, x, x.shape[0], out)
        if rc:
            raise ValueError(f"block forward rejected (status {rc})")
        return out

    def prefill_last_logits(self, ids):
        self.reset()
        return self.forward(ids)

    def greedy(self, first: int, n_steps: int, teacher=None, want_logits=False):
        a = self.model.arch
        out = np.empty(n_steps, np.uint32)
        logits = np.empty((n_steps, a.vocab), np.float32) if want_logits else None
        t = None if teacher is None else np.ascontiguousarray(teacher, np.uint32)
        rc = lib().zo_greedy_decode(self.h, first, n_steps,
                                    None if t is None else t.ctypes.data_as(C.c_void_p), out,
                                    None if logits is None else logits.ctypes.data_as(C.c_void_p))
        if rc:
            raise ValueError(f"greedy rejected (status {rc})")
        return (out, logits) if want_logits else out

    def fill_kv(self, n: int, seed: int):
        """Seeded stand-in cache of n positions (timing only)."""
        if lib().zo_session_fill_kv(self.h, n, seed):
            raise ValueError("n > max_seq")

    def kv(self, layer: int, which_v: bool):
        a = self.model.arch
        out = np.empty((a.n_kv, self.used, a.head_dim), np.float32)
        lib().zo_session_kv(self.h, layer, int(which_v), out)
        return out

    def close(self):
        if self.h:
            lib().zo_session_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
