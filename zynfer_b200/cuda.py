"""ctypes binding of libzynfer_cuda.so (include/zynfer_cuda.h).

The Python face of the `cuda` backend, shaped like the reference's Apple GPU
wrapper (src/backends/apple/gpu.zig:109-181: status -> error set, last_error
text) and its model session (src/model/qwen_forward.zig:21-160). It loads the
in-tree library and nothing else: there is no CPU path here.
"""
from __future__ import annotations

import atexit
import ctypes as C
import os
import weakref
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libzynfer_cuda.so")

OK, NO_DEVICE, OOM, INVALID, UNSUPPORTED, LAUNCH, TIMEOUT, INTERNAL = range(8)
W_Q8, W_BF16 = 0, 1
K_ATTN, K_LINEAR, K_LMHEAD, K_OTHER = range(4)


class CudaError(RuntimeError):
    status = INTERNAL


class NoDevice(CudaError):
    status = NO_DEVICE


class OutOfMemory(CudaError):
    status = OOM


class InvalidArgument(CudaError, ValueError):
    status = INVALID


class Unsupported(CudaError):
    status = UNSUPPORTED


class LaunchFailed(CudaError):
    status = LAUNCH


class DeviceTimeout(CudaError):
    status = TIMEOUT


class Internal(CudaError):
    status = INTERNAL


_ERRORS = {NO_DEVICE: NoDevice, OOM: OutOfMemory, INVALID: InvalidArgument, UNSUPPORTED: Unsupported,
           LAUNCH: LaunchFailed, TIMEOUT: DeviceTimeout, INTERNAL: Internal}


class Caps(C.Structure):
    _fields_ = [("device_name", C.c_char * 256), ("sm_major", C.c_int), ("sm_minor", C.c_int),
                ("sm_count", C.c_int), ("hbm_bytes", C.c_uint64), ("l2_bytes", C.c_uint64),
                ("max_smem_per_block", C.c_uint32), ("bulk_copy", C.c_int), ("tcgen05", C.c_int)]


class ModelDesc(C.Structure):
    _fields_ = [("vocab", C.c_uint32), ("hidden", C.c_uint32), ("inter", C.c_uint32),
                ("layers", C.c_uint32), ("n_q", C.c_uint32), ("n_kv", C.c_uint32),
                ("head_dim", C.c_uint32), ("max_pos", C.c_uint32), ("eps", C.c_float),
                ("theta", C.c_float), ("weights", C.c_uint32), ("max_batch", C.c_uint32),
                ("max_seqs", C.c_uint32), ("max_seq_len", C.c_uint32), ("kv_blocks", C.c_uint32),
                ("max_prefill", C.c_uint32), ("prefill_kv_f32", C.c_uint32)]


VP = C.c_void_p
U32 = C.c_uint32
U64 = C.c_uint64
_SIGS = {
    "zynfer_cu_create": (C.c_int, [C.c_int, C.POINTER(VP)]),
    "zynfer_cu_destroy": (None, [VP]),
    "zynfer_cu_caps": (C.c_int, [VP, C.POINTER(Caps)]),
    "zynfer_cu_last_error": (C.c_char_p, [VP]),
    "zynfer_cu_sync": (C.c_int, [VP]),
    "zynfer_cu_set_fail_at": (C.c_int, [VP, C.c_char_p]),
    "zynfer_cu_last_path": (C.c_char_p, [VP]),
    "zynfer_cu_build_info": (C.c_char_p, []),
    "zynfer_cu_model_init": (C.c_int, [VP, C.POINTER(ModelDesc)]),
    "zynfer_cu_upload_f32": (C.c_int, [VP, C.c_char_p, VP, U64, U64]),
    "zynfer_cu_upload_bf16": (C.c_int, [VP, C.c_char_p, VP, U64, U64]),
    "zynfer_cu_upload_q8": (C.c_int, [VP, C.c_char_p, VP, VP, U64, U64]),
    "zynfer_cu_fill_synthetic": (C.c_int, [VP, U64, C.c_float, C.c_float]),
    "zynfer_cu_download_q8": (C.c_int, [VP, C.c_char_p, VP, VP, U64, U64]),
    "zynfer_cu_seq_reset": (C.c_int, [VP, U32]),
    "zynfer_cu_seq_len": (C.c_int, [VP, U32, C.POINTER(U32)]),
    "zynfer_cu_kv_read": (C.c_int, [VP, U32, U32, C.c_int, VP]),
    "zynfer_cu_kv_fill_synthetic": (C.c_int, [VP, U32, U32, U64]),
    "zynfer_cu_seq_fork": (C.c_int, [VP, U32, U32, U32]),
    "zynfer_cu_extend": (C.c_int, [VP, U32, VP, U32, VP, VP]),
    "zynfer_cu_pool_stats": (C.c_int, [VP, C.POINTER(U32), C.POINTER(U32)]),
    "zynfer_cu_prefill": (C.c_int, [VP, U32, VP, U32, VP, VP]),
    "zynfer_cu_decode_step": (C.c_int, [VP, VP, VP, U32, VP, VP]),
    "zynfer_cu_generate": (C.c_int, [VP, VP, VP, U32, U32, VP, C.POINTER(C.c_float)]),
    "zynfer_cu_block_forward": (C.c_int, [VP, U32, U32, VP, U32, VP]),
    "zynfer_cu_linear": (C.c_int, [VP, C.c_int, VP, VP, VP, U32, U32, U32, VP]),
    "zynfer_cu_set_linear_path": (C.c_int, [VP, C.c_char_p]),
    "zynfer_cu_set_sampling": (C.c_int, [VP, C.c_float, U32, C.c_float, U64]),
    "zynfer_cu_sample": (C.c_int, [VP, VP, U32, U32, VP, VP, C.c_float, U32, C.c_float, U64, VP]),
    "zynfer_cu_set_decode_schedule": (C.c_int, [VP, C.c_char_p]),
    "zynfer_cu_phase_trace": (C.c_int, [VP, VP, C.c_int]),
    "zynfer_cu_linear_q8_static": (C.c_int, [VP, VP, VP, U32, U32, U32, VP, VP]),
    "zynfer_cu_linear_q8_static_status": (C.c_int, [C.c_int]),
    "zynfer_cu_attn_decode": (C.c_int, [VP, U32, VP, U32, VP, VP]),
    "zynfer_cu_rmsnorm_qk_rope": (C.c_int, [VP, VP, U32, VP, VP, U32, VP, VP]),
    "zynfer_cu_swiglu": (C.c_int, [VP, VP, VP, U64, VP]),
    "zynfer_cu_pack_q8": (C.c_int, [VP, VP, U32, U32, VP, VP]),
    "zynfer_cu_rmsnorm": (C.c_int, [VP, VP, VP, U32, U32, C.c_float, VP]),
    "zynfer_cu_set_timing": (C.c_int, [VP, C.c_int]),
    "zynfer_cu_kernel_time": (C.c_int, [VP, C.c_int, C.POINTER(U64), C.POINTER(C.c_double)]),
    "zynfer_cu_last_step_ns": (U64, [VP]),
    "zynfer_cu_step_launches": (C.c_int, [VP]),
    "zynfer_cu_io_bytes": (C.c_int, [VP, C.POINTER(U64), C.POINTER(U64), C.c_int]),
    "zynfer_cu_alloc_events": (C.c_int, [VP, C.POINTER(U64), C.POINTER(U64)]),
    "zynfer_cu_artifact_open": (C.c_int, [C.c_char_p, C.POINTER(VP)]),
    "zynfer_cu_artifact_close": (None, [VP]),
    "zynfer_cu_artifact_error": (C.c_char_p, [VP]),
    "zynfer_cu_artifact_meta": (C.c_int, [VP, VP]),
    "zynfer_cu_artifact_tensor": (C.c_int, [VP, U32, VP]),
    "zynfer_cu_artifact_find_id": (C.c_int, [VP, U32, VP]),
    "zynfer_cu_artifact_find_name": (C.c_int, [VP, C.c_char_p, VP]),
    "zynfer_cu_model_desc_from_artifact": (C.c_int, [VP, C.POINTER(ModelDesc)]),
    "zynfer_cu_load_artifact": (C.c_int, [VP, VP]),
}
EXPORTS = tuple(_SIGS)

_lib = None


def lib():
    """Load the in-tree library; fail loudly when it is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m zynfer_b200.build` "
                              "(the cuda backend has no fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def _ptr(a) -> C.c_void_p | None:
    if a is None:
        return None
    if isinstance(a, int):
        return C.c_void_p(a)
    if hasattr(a, "data_ptr"):  # torch tensor (device pointer)
        return C.c_void_p(a.data_ptr())
    return a.ctypes.data_as(C.c_void_p)


STATIC_MAX_ROWS, STATIC_MAX_K = 64, 4096


def linear_q8_static(w, scale, x, batch: int, m: int, k: int, y, stream=None):
    """zynfer_cu_linear_q8_static: the int8 linear that allocates nothing (no
    context; device pointers; scratch in a library-owned device array)."""
    if stream is not None and hasattr(stream, "cuda_stream"):  # a torch.cuda.Stream
        stream = int(stream.cuda_stream)
    rc = lib().zynfer_cu_linear_q8_static(_ptr(w), _ptr(scale), _ptr(x), batch, m, k, _ptr(y), _ptr(stream))
    if rc != OK:
        raise _ERRORS.get(rc, CudaError)(f"zynfer_cu_linear_q8_static failed with status {rc}")


def linear_q8_static_status(clear: bool = True) -> int:
    """zynfer_cu_linear_q8_static_status: the status its device error word
    holds (OK, or TIMEOUT when a bounded device wait ran out); call after
    synchronising the stream the calls ran on."""
    return int(lib().zynfer_cu_linear_q8_static_status(int(clear)))


def arm_static_wait_fault():
    """zynfer_cu_set_fail_at(NULL, "wait"): the next allocation-free linear
    call skips its first K stage, so its bounded device waits run out."""
    rc = lib().zynfer_cu_set_fail_at(None, b"wait")
    if rc != OK:
        raise _ERRORS.get(rc, CudaError)("zynfer_cu_set_fail_at(NULL, wait) failed")


@dataclass
class Arch:
    """src/model/qwen3.zig:19-34 (Qwen3-0.6B)."""
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


QWEN3_0_6B = Arch()


_LIVE: "weakref.WeakSet[Gpu]" = weakref.WeakSet()


@atexit.register
def _close_live_contexts():
    """Destroy contexts before interpreter teardown, while the CUDA runtime is still up."""
    for g in list(_LIVE):
        g.close()


class Gpu:
    """One context on one device (zynfer_cu_create / destroy). One model per context."""

    def __init__(self, device: int = 0):
        L = lib()
        h = VP()
        rc = L.zynfer_cu_create(device, C.byref(h))
        self.h = h
        if rc != OK:
            msg = L.zynfer_cu_last_error(h).decode() if h else "create failed"
            if h:
                L.zynfer_cu_destroy(h)
            self.h = None
            raise _ERRORS.get(rc, CudaError)(msg)
        _LIVE.add(self)

    def check(self, rc: int):
        if rc != OK:
            raise _ERRORS.get(rc, CudaError)(lib().zynfer_cu_last_error(self.h).decode())

    def caps(self) -> Caps:
        c = Caps()
        self.check(lib().zynfer_cu_caps(self.h, C.byref(c)))
        return c

    @property
    def last_error(self) -> str:
        return lib().zynfer_cu_last_error(self.h).decode()

    @property
    def last_path(self) -> str:
        return lib().zynfer_cu_last_path(self.h).decode()

    def sync(self):
        self.check(lib().zynfer_cu_sync(self.h))

    def set_fail_at(self, spec: str):
        self.check(lib().zynfer_cu_set_fail_at(self.h, spec.encode()))

    # op level (device pointers)
    def linear(self, wkind, w, scale, x, batch, m, k, y):
        self.check(lib().zynfer_cu_linear(self.h, wkind, _ptr(w), _ptr(scale), _ptr(x), batch, m, k, _ptr(y)))

    def set_linear_path(self, path: str):
        """"auto" | "gemv" | "mma" | "tcgen05" | "simt"."""
        self.check(lib().zynfer_cu_set_linear_path(self.h, path.encode()))

    def set_sampling(self, temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0, seed: int = 0):
        """Next-token rule of decode / generate / prefill: temperature 0 = greedy."""
        self.check(lib().zynfer_cu_set_sampling(self.h, temperature, top_k, top_p, seed))

    def sample(self, logits, rows: int, vocab: int, slots, positions, temperature: float, top_k: int = 0,
               top_p: float = 1.0, seed: int = 0):
        """The sampling rule on device logits [rows][vocab]; returns one id per row."""
        s = np.ascontiguousarray(slots, np.uint32)
        p = np.ascontiguousarray(positions, np.uint32)
        out = np.empty(rows, np.uint32)
        self.check(lib().zynfer_cu_sample(self.h, _ptr(logits), rows, vocab, _ptr(s), _ptr(p), temperature, top_k,
                                          top_p, seed, _ptr(out)))
        return out

    def phase_trace(self):
        """Phase timestamps (ns) of the last persistent decode step run with timing on."""
        n = lib().zynfer_cu_phase_trace(self.h, None, 0)
        out = np.zeros(max(n, 0), np.uint64)
        if n > 0:
            lib().zynfer_cu_phase_trace(self.h, _ptr(out), n)
        return out

    def set_decode_schedule(self, schedule: str):
        """"auto" | "kernels" | "persistent" (one cooperative kernel per decode step)."""
        self.check(lib().zynfer_cu_set_decode_schedule(self.h, schedule.encode()))

    def swiglu(self, gate, up, n, out):
        """siluMul (ops.zig:36-42) on device pointers."""
        self.check(lib().zynfer_cu_swiglu(self.h, _ptr(gate), _ptr(up), n, _ptr(out)))

    def alloc_events(self):
        """(device, host) allocation events since model init."""
        d, h = U64(), U64()
        self.check(lib().zynfer_cu_alloc_events(self.h, C.byref(d), C.byref(h)))
        return int(d.value), int(h.value)

    def pack_q8(self, w, rows, cols, q, scale):
        self.check(lib().zynfer_cu_pack_q8(self.h, _ptr(w), rows, cols, _ptr(q), _ptr(scale)))

    def rmsnorm(self, x, w, rows, cols, eps, y):
        self.check(lib().zynfer_cu_rmsnorm(self.h, _ptr(x), _ptr(w), rows, cols, eps, _ptr(y)))

    def set_timing(self, on: bool):
        self.check(lib().zynfer_cu_set_timing(self.h, int(on)))

    def kernel_time(self, cls: int):
        n = U64()
        ms = C.c_double()
        self.check(lib().zynfer_cu_kernel_time(self.h, cls, C.byref(n), C.byref(ms)))
        return int(n.value), float(ms.value)

    @property
    def step_launches(self) -> int:
        return int(lib().zynfer_cu_step_launches(self.h))

    def io_bytes(self, reset: bool = False):
        h2d, d2h = U64(), U64()
        self.check(lib().zynfer_cu_io_bytes(self.h, C.byref(h2d), C.byref(d2h), int(reset)))
        return int(h2d.value), int(d2h.value)

    @property
    def last_step_ns(self) -> int:
        return int(lib().zynfer_cu_last_step_ns(self.h))

    def close(self):
        if self.h:
            lib().zynfer_cu_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Model:
    """Weights + paged KV pool + sequences on one Gpu (qwen_forward.Session)."""

    def __init__(self, gpu: Gpu, arch: Arch = QWEN3_0_6B, weights: int = W_Q8, max_batch: int = 1,
                 max_seqs: int = 1, max_seq_len: int = 4096, kv_blocks: int = 0, max_prefill: int = 0,
                 prefill_kv_f32: bool = False):
        self.gpu = gpu
        self.arch = arch
        self.weights = weights
        self.desc = ModelDesc(arch.vocab, arch.hidden, arch.inter, arch.layers, arch.n_q, arch.n_kv,
                              arch.head_dim, arch.max_pos, arch.eps, arch.theta, weights, max_batch,
                              max_seqs, max_seq_len, kv_blocks, max_prefill, int(prefill_kv_f32))
        gpu.check(lib().zynfer_cu_model_init(gpu.h, C.byref(self.desc)))

    # weights
    def load_artifact(self, art):
        """Every tensor of an open `.zynfer` artifact (zynfer_b200.artifact.Artifact) to the device."""
        self.gpu.check(lib().zynfer_cu_load_artifact(self.gpu.h, art.h))

    def fill_synthetic(self, seed: int, w_std: float = 0.02, norm_std: float = 0.0):
        self.gpu.check(lib().zynfer_cu_fill_synthetic(self.gpu.h, seed, w_std, norm_std))

    def upload_f32(self, name: str, data):
        a = np.ascontiguousarray(data, np.float32)
        rows, cols = (a.shape[0], a.shape[1]) if a.ndim == 2 else (a.size, 1)
        self.gpu.check(lib().zynfer_cu_upload_f32(self.gpu.h, name.encode(), _ptr(a), rows, cols))

    def upload_bf16(self, name: str, bits):
        a = np.ascontiguousarray(bits, np.uint16)
        rows, cols = (a.shape[0], a.shape[1]) if a.ndim == 2 else (a.size, 1)
        self.gpu.check(lib().zynfer_cu_upload_bf16(self.gpu.h, name.encode(), _ptr(a), rows, cols))

    def upload_q8(self, name: str, q, scale):
        q = np.ascontiguousarray(q, np.int8)
        s = np.ascontiguousarray(scale, np.float32)
        self.gpu.check(lib().zynfer_cu_upload_q8(self.gpu.h, name.encode(), _ptr(q), _ptr(s), *q.shape))

    def download_q8(self, name: str, rows: int, cols: int):
        q = np.empty((rows, cols), np.int8)
        s = np.empty(rows, np.float32)
        self.gpu.check(lib().zynfer_cu_download_q8(self.gpu.h, name.encode(), _ptr(q), _ptr(s), rows, cols))
        return q, s

    # sequences
    def seq_reset(self, seq: int):
        self.gpu.check(lib().zynfer_cu_seq_reset(self.gpu.h, seq))

    def seq_len(self, seq: int) -> int:
        n = U32()
        self.gpu.check(lib().zynfer_cu_seq_len(self.gpu.h, seq, C.byref(n)))
        return int(n.value)

    def seq_fork(self, dst: int, src: int, n: int):
        """`dst` becomes the first n positions of `src` (whole blocks shared, the partial one copied)."""
        self.gpu.check(lib().zynfer_cu_seq_fork(self.gpu.h, dst, src, n))

    def extend(self, seq: int, tokens, want_logits: bool = True):
        """Append tokens to a sequence; the last token's logits and argmax."""
        t = np.ascontiguousarray(tokens, np.uint32)
        logits = np.empty(self.arch.vocab, np.float32) if want_logits else None
        am = np.zeros(1, np.uint32)
        self.gpu.check(lib().zynfer_cu_extend(self.gpu.h, seq, _ptr(t), t.size, _ptr(logits), _ptr(am)))
        return (logits, int(am[0])) if want_logits else int(am[0])

    def pool_stats(self):
        free, shared = U32(), U32()
        self.gpu.check(lib().zynfer_cu_pool_stats(self.gpu.h, C.byref(free), C.byref(shared)))
        return int(free.value), int(shared.value)

    def kv_fill_synthetic(self, seq: int, n: int, seed: int):
        """Reset `seq` and fill positions [0, n) of every layer with the seeded stand-in K/V."""
        self.gpu.check(lib().zynfer_cu_kv_fill_synthetic(self.gpu.h, seq, n, seed))

    def attn_decode(self, layer: int, seqs, qkv, out):
        """Decode attention of `layer` (device qkv [B][(n_q + 2 n_kv) d] -> out [B][n_q][d])."""
        s = np.ascontiguousarray(seqs, np.uint32)
        self.gpu.check(lib().zynfer_cu_attn_decode(self.gpu.h, layer, _ptr(s), s.size, _ptr(qkv), _ptr(out)))

    def rmsnorm_qk_rope(self, qkv, rows: int, q_norm, k_norm, pos0: int, q_out, k_out):
        """Per-head q/k RMSNorm + RoPE of `rows` tokens (device pointers, heads-major outputs)."""
        self.gpu.check(lib().zynfer_cu_rmsnorm_qk_rope(self.gpu.h, _ptr(qkv), rows, _ptr(q_norm), _ptr(k_norm),
                                                       pos0, _ptr(q_out), _ptr(k_out)))

    def kv(self, seq: int, layer: int, which_v: bool):
        a = self.arch
        out = np.empty((a.n_kv, self.seq_len(seq), a.head_dim), np.float32)
        self.gpu.check(lib().zynfer_cu_kv_read(self.gpu.h, seq, layer, int(which_v), _ptr(out)))
        return out

    # forward
    def prefill(self, seq: int, tokens, want_logits: bool = True):
        t = np.ascontiguousarray(tokens, np.uint32)
        logits = np.empty(self.arch.vocab, np.float32) if want_logits else None
        am = np.zeros(1, np.uint32)
        self.gpu.check(lib().zynfer_cu_prefill(self.gpu.h, seq, _ptr(t), t.size, _ptr(logits), _ptr(am)))
        return (logits, int(am[0])) if want_logits else int(am[0])

    def prefill_last_logits(self, seq: int, tokens):
        return self.prefill(seq, tokens, True)[0]

    def decode_step(self, seqs, tokens, want_logits: bool = False):
        s = np.ascontiguousarray(seqs, np.uint32)
        t = np.ascontiguousarray(tokens, np.uint32)
        am = np.zeros(s.size, np.uint32)
        logits = np.empty((s.size, self.arch.vocab), np.float32) if want_logits else None
        self.gpu.check(lib().zynfer_cu_decode_step(self.gpu.h, _ptr(s), _ptr(t), s.size, _ptr(am), _ptr(logits)))
        return (am, logits) if want_logits else am

    def generate(self, seqs, first, steps: int):
        s = np.ascontiguousarray(seqs, np.uint32)
        f = np.ascontiguousarray(first, np.uint32)
        out = np.empty((steps, s.size), np.uint32)
        ms = C.c_float()
        self.gpu.check(lib().zynfer_cu_generate(self.gpu.h, _ptr(s), _ptr(f), s.size, steps, _ptr(out), C.byref(ms)))
        return out, float(ms.value)

    def block_forward(self, layer: int, seq: int, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        self.gpu.check(lib().zynfer_cu_block_forward(self.gpu.h, layer, seq, _ptr(x), x.shape[0], _ptr(out)))
        return out
