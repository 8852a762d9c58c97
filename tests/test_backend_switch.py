"""The backend switch with `cuda` added (src/runtime/backend.zig:106-130,
tests/numerical/ops.zig:12-14, tests/integration/cli.zig:63-67): unknown names
still fail, unavailable kinds fail, nothing falls back. The reference's
"cuda is unknown" assertions are re-pointed at a name that is still unknown."""
import pytest

from zynfer_b200 import backend as B


def test_parse_accepts_cuda_and_aliases():  # backend.zig:158-163 (cuda now known)
    assert B.parse_backend_kind("cuda") is B.BackendKind.cuda
    assert B.parse_backend_kind("cpu") is B.BackendKind.cpu
    assert B.parse_backend_kind("metal") is B.BackendKind.apple
    assert B.parse_backend_kind("hip") is B.BackendKind.amd_hip


@pytest.mark.parametrize("name", ["bogus", "CUDA", "cuda12", "", "nvidia"])
def test_unknown_backend_does_not_fall_back(name):
    with pytest.raises(B.UnknownBackend):
        B.parse_backend_kind(name)


def test_unbuilt_kind_is_unavailable():  # backend.zig:122-124
    with pytest.raises(B.BackendUnavailable):
        B.require_backend(B.BackendKind.apple)


def test_cuda_buildable_when_library_present():
    from zynfer_b200 import build
    build.build()
    assert B.is_backend_buildable(B.BackendKind.cuda)
    B.require_backend(B.BackendKind.cuda)
    assert B.default_kind() is B.BackendKind.cuda


def test_resolve_kind_env(monkeypatch):  # main.zig:58-64,110-114
    monkeypatch.setenv("ZYNFER_BACKEND", "bogus")
    with pytest.raises(B.UnknownBackend):
        B.resolve_kind()
    assert B.resolve_kind("cuda") is B.BackendKind.cuda
