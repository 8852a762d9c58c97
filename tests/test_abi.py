"""The C-ABI library loads and exports every symbol include/zynfer_cuda.h
declares, and fails loudly (no fallback) where there is no B200. CPU-only."""
import ctypes as C
import os
import re
import subprocess

import pytest

from zynfer_b200 import cuda as zc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "zynfer_cuda.h")


def header_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(zynfer_cu_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def built():
    from zynfer_b200 import build
    build.build()
    return zc.lib()


def test_header_is_plain_c():
    # compiles as C99 (Zig @cImport, cgo and ctypes need a C header)
    res = subprocess.run(["gcc", "-std=c99", "-fsyntax-only", "-Wall", "-Werror", "-x", "c", HEADER],
                         capture_output=True, text=True)
    assert res.returncode == 0, res.stderr


def test_every_declared_symbol_is_exported(built):
    names = header_functions()
    assert len(names) >= 25
    nm = subprocess.run(["nm", "-D", "--defined-only", zc.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (zynfer_cu_\w+)", nm))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    extra = sorted(exported - set(names))
    assert not extra, f"exported but undeclared: {extra}"
    for n in names:
        assert getattr(built, n) is not None


def test_binding_covers_the_header():
    assert sorted(zc.EXPORTS) == header_functions()


def test_build_info(built):
    assert b"sm_100a" in built.zynfer_cu_build_info()


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_has_gpu(), reason="checks the no-device path")
def test_create_without_device_fails_loudly(built):
    h = C.c_void_p()
    rc = built.zynfer_cu_create(0, C.byref(h))
    assert rc == zc.NO_DEVICE
    assert b"no CUDA device" in built.zynfer_cu_last_error(h)
    built.zynfer_cu_destroy(h)
    with pytest.raises(zc.NoDevice):
        zc.Gpu(0)


def test_null_context_is_rejected(built):
    assert built.zynfer_cu_sync(None) == zc.INVALID
    assert built.zynfer_cu_model_init(None, None) == zc.INVALID
    assert built.zynfer_cu_last_error(None) == b"null context"
