"""The C-ABI library loads and exports every symbol include/*.h declares (no GPU needed)."""
import ctypes
import glob
import os
import re

import pytest

from drofell_for_revision_b200 import _capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    syms = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        syms |= set(re.findall(r"W4A16_API\s+[\w\s\*]+?\b(w4a16_\w+)\s*\(", text))
    return syms


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ["w4a16_create", "w4a16_destroy", "w4a16_dequant", "w4a16_gemm", "w4a16_gemm_t",
              "w4a16_workspace_size", "w4a16_last_error"]:
        assert s in syms


def test_library_exports_every_declared_symbol():
    lib = _capi.lib()
    for s in declared_symbols():
        assert hasattr(lib, s), s
    assert set(_capi.EXPORTED) <= declared_symbols()


def test_version_and_empty_error():
    lib = _capi.lib()
    assert lib.w4a16_version() == 101
    assert isinstance(lib.w4a16_last_error(), bytes)


def test_create_rejects_bad_arguments_without_touching_cuda():
    lib = _capi.lib()
    out = ctypes.c_void_p()
    # null packed pointers
    rc = lib.w4a16_create(None, None, None, None, 64, 64, 1, 0, None, ctypes.byref(out))
    assert rc == _capi.W4A16_ERR_INVALID
    assert b"null" in lib.w4a16_last_error()
    fake = ctypes.c_void_p(0x1000)
    # K not a multiple of 32
    rc = lib.w4a16_create(fake, fake, fake, None, 48, 64, 1, 0, None, ctypes.byref(out))
    assert rc == _capi.W4A16_ERR_INVALID
    # groups not dividing K
    rc = lib.w4a16_create(fake, fake, fake, None, 64, 64, 3, 0, None, ctypes.byref(out))
    assert rc == _capi.W4A16_ERR_INVALID
    # group size not a multiple of 8 (K=96, G=24 -> gs=4)
    rc = lib.w4a16_create(fake, fake, fake, None, 96, 64, 24, 0, None, ctypes.byref(out))
    assert rc == _capi.W4A16_ERR_UNSUPPORTED
    # misaligned qweight
    rc = lib.w4a16_create(ctypes.c_void_p(0x1004), fake, fake, None, 64, 64, 1, 0, None, ctypes.byref(out))
    assert rc == _capi.W4A16_ERR_INVALID
    assert out.value is None


def test_null_handle_is_rejected():
    lib = _capi.lib()
    assert lib.w4a16_gemm(None, None, 1, None, 0, None, 0, 0, None) == _capi.W4A16_ERR_INVALID
    assert lib.w4a16_dequant(None, None, 0, None) == _capi.W4A16_ERR_INVALID
    assert lib.w4a16_workspace_size(None, 4, 0, 0) == 0
    assert lib.w4a16_destroy(None) == 0


def test_every_compute_entry_point_rejects_null_handles_before_cuda():
    # argument checks come before any CUDA call, so they hold on a machine without a GPU
    lib = _capi.lib()
    INV = _capi.W4A16_ERR_INVALID
    assert lib.w4a16_gemm_t(None, None, 1, None, 0, None, 0, None) == INV
    assert lib.w4a16_gemm_static(None, None, 1, None, 0, 0, None) == INV
    assert lib.w4a16_gemm_gather(None, None, None, 1, None, 8, 0, 0, None, 0, None) == INV
    assert lib.w4a16_mlp_forward(None, None, None, None, 1e-6, None, 1, None, None, None, None, 0, None, 0,
                                 None) == INV
    assert lib.w4a16_qkv_forward(None, None, None, None, 1e-6, None, 1, None, None, None, None, 0, None, 0,
                                 None) == INV
    assert b"null" in lib.w4a16_last_error()


def test_handle_requires_cuda_tensors():
    import torch
    qw = torch.zeros((8, 64), dtype=torch.int32)
    qz = torch.zeros((1, 8), dtype=torch.int32)
    sc = torch.zeros((1, 64), dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        _capi.Handle(qw, qz, sc, None, 0)
