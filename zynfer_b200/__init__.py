"""zynfer_b200: the B200-native `cuda` backend for the Zynfer Qwen3 runtime.

The product is the C-ABI library ``libzynfer_cuda.so`` (include/zynfer_cuda.h,
hand-written sm_100a kernels). This package holds its sources (``csrc/``),
the in-tree build (``build.py``), the backend switch mirrored from the
reference (``backend.py``) and the ctypes binding (``cuda.py``). There is no
CPU fallback: without the library or a B200, the `cuda` backend is
unavailable and says so.
"""
from .backend import (BackendKind, BackendUnavailable, UnknownBackend, default_kind,  # noqa: F401
                      is_backend_buildable, parse_backend_kind, require_backend)
