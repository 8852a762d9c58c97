"""Backend identity and the `--backend` / ZYNFER_BACKEND switch with `cuda` added.

Mirrors src/runtime/backend.zig:10-22 (BackendKind), :106-112
(parseBackendKind: unknown names fail), :114-124 (isBackendBuildable,
requireBackend: a kind that is not built fails, never falls back) and :126-130
(defaultKind). The `cuda` kind is buildable when libzynfer_cuda.so is present.
"""
from __future__ import annotations

import enum
import os


class UnknownBackend(ValueError):
    """parseBackendKind: error.UnknownBackend."""


class BackendUnavailable(RuntimeError):
    """requireBackend: error.BackendUnavailable."""


class BackendKind(enum.Enum):
    cpu = "cpu"
    apple = "apple"
    amd_hip = "amd-hip"
    cuda = "cuda"

    @property
    def display(self) -> str:  # BackendKind.name, backend.zig:15-21
        return self.value


def parse_backend_kind(text: str) -> BackendKind:
    """backend.zig:106-112 plus the `cuda` kind. Unknown names raise."""
    if text == "cpu":
        return BackendKind.cpu
    if text in ("apple", "metal"):
        return BackendKind.apple
    if text in ("amd", "hip", "amd-hip"):
        return BackendKind.amd_hip
    if text == "cuda":
        return BackendKind.cuda
    raise UnknownBackend(f"unknown backend: {text}")


def _cuda_library_present() -> bool:
    here = os.path.dirname(os.path.abspath(__file__))
    return os.path.exists(os.path.join(here, "libzynfer_cuda.so"))


def is_backend_buildable(kind: BackendKind) -> bool:
    """backend.zig:114-120. This package builds only the `cuda` backend; the
    reference's cpu backend is its Zig oracle, apple/amd-hip are not built here."""
    if kind is BackendKind.cuda:
        return _cuda_library_present()
    return False


def require_backend(kind: BackendKind) -> None:
    """backend.zig:122-124: no silent fallback."""
    if not is_backend_buildable(kind):
        raise BackendUnavailable(f"backend {kind.value} is not available in this build")


def default_kind() -> BackendKind:
    """backend.zig:126-130 with cuda first when it is built."""
    return BackendKind.cuda if _cuda_library_present() else BackendKind.cpu


def resolve_kind(flag: str | None = None) -> BackendKind:
    """main.zig:58-64,110-114,208-221: --backend, else ZYNFER_BACKEND, else default."""
    name = flag if flag is not None else os.environ.get("ZYNFER_BACKEND")
    if name is None:
        return default_kind()
    kind = parse_backend_kind(name)
    require_backend(kind)
    return kind
