"""CPU-only checks of the host side: the C-ABI library loads and exports every
symbol include/tda_b200.h declares, and the Python mirror of the reference
interface validates its arguments the way the reference does -- without any
compute call (there is no GPU here)."""
import os
import re

import pytest
import torch

import tda_b200
from tda_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tda_b200.h")


def _declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tda_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = _declared_symbols()
    for name in ("tda_rect_fwd", "tda_diff_fwd", "tda_workspace_size", "tda_last_error", "tda_key_inv_norms"):
        assert name in syms


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    syms = _declared_symbols()
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing
    # the Python binding covers the whole header, too
    assert set(syms) == set(_lib.SIGNATURES)


def test_library_host_only_calls():
    lib = _lib.load()
    assert lib.tda_version() == 101
    # workspace: per key tensor a key table of 2 x 128 (padded rows) x 17/16
    # floats = 1088 B, rounded up to 256 B
    assert lib.tda_workspace_size(0, _lib.TDA_BF16, 2, 100, 64, 1) == 1280
    assert lib.tda_workspace_size(1, _lib.TDA_BF16, 2, 100, 64, 1) == 2560
    assert lib.tda_workspace_size(1, _lib.TDA_BF16, 2, 100, 64, 0) == 0
    # fp32 at head_dim 64: TF32 high / low copies of q, k (2 x 51200 B each), three
    # per-row coefficient arrays (1024 B each, seq padded to 128) and V^T high / low (65536 B each)
    assert lib.tda_workspace_size(0, _lib.TDA_F32, 2, 100, 64, 1) == 4 * 51200 + 3 * 1024 + 2 * 65536
    assert lib.tda_workspace_size(1, _lib.TDA_F32, 2, 100, 64, 0) == 8 * 51200 + 6 * 1024 + 2 * 65536
    # head_dim 128: copies of 2 x 100 x 128 floats (102400 B), V^T copies of 2 x 128 x 128 (131072 B)
    assert lib.tda_workspace_size(0, _lib.TDA_F32, 2, 100, 128, 1) == 4 * 102400 + 3 * 1024 + 2 * 131072
    assert lib.tda_workspace_size(0, _lib.TDA_F32, 2, 100, 32, 1) == 0


def test_library_rejects_bad_arguments_without_launching():
    lib = _lib.load()
    # NULL status word -> invalid (checked before any CUDA call)
    rc = lib.tda_rect_fwd(16, 16, 16, 16, _lib.TDA_BF16, _lib.TDA_BF16, 1, 128, 64, 1.0, 2.0, 0, None, 0, None, None)
    assert rc == _lib.TDA_ERR_INVALID
    assert b"status" in lib.tda_last_error()
    rc = lib.tda_rect_fwd(16, 16, 16, 16, _lib.TDA_BF16, _lib.TDA_BF16, 1, 128, 48, 1.0, 2.0, 0, None, 0, 16, None)
    assert rc == _lib.TDA_ERR_UNSUPPORTED
    rc = lib.tda_diff_fwd(16, 16, 16, 16, 16, 16, 7, 7, 1, 128, 64, 1.0, 0.5, 2.0, 1, None, 0, 16, None)
    assert rc == _lib.TDA_ERR_INVALID
    rc = lib.tda_diff_fwd(16, 16, 16, 16, 16, 16, _lib.TDA_BF16, _lib.TDA_BF16, 1, 128, 64, 1.0, 0.5, 2.0, 1,
                          None, 0, 16, None)
    assert rc == _lib.TDA_ERR_WORKSPACE
    rc = lib.tda_rect_fwd(16, 16, 16, 16, _lib.TDA_F32, _lib.TDA_F32, 0, 128, 64, 1.0, 2.0, 0, None, 0, 16, None)
    assert rc == _lib.TDA_ERR_INVALID
    rc = lib.tda_rect_fwd(17, 16, 16, 16, _lib.TDA_F32, _lib.TDA_F32, 1, 128, 64, 1.0, 2.0, 0, None, 0, 16, None)
    assert rc == _lib.TDA_ERR_INVALID  # misaligned pointer
    with pytest.raises(ValueError):
        _lib.check(_lib.TDA_ERR_INVALID)
    # fp16 runs on the tensor cores only with normalize (P bounded): refused before any launch
    rc = lib.tda_rect_fwd(16, 16, 16, 16, _lib.TDA_F16, _lib.TDA_F16, 1, 128, 64, 1.0, 2.0, 0, None, 0, 16, None)
    assert rc == _lib.TDA_ERR_UNSUPPORTED and b"fp16" in lib.tda_last_error()
    rc = lib.tda_diff_fwd(16, 16, 16, 16, 16, 16, _lib.TDA_F16, _lib.TDA_F16, 1, 128, 64, -4.0, 0.5, 12.0, 1,
                          None, 0, 16, None)
    assert rc == _lib.TDA_ERR_UNSUPPORTED  # (1 + 4 sqrt(2 ln 128 / 64))^12 > 16384
    assert lib.tda_workspace_size(1, _lib.TDA_F16, 2, 100, 64, 1) == lib.tda_workspace_size(1, _lib.TDA_BF16, 2, 100,
                                                                                            64, 1)
    # device-lambda entry point: NULL lambda and negative strides are rejected
    rc = lib.tda_diff_fwd_lambda(16, 16, 16, 16, 16, None, 16, _lib.TDA_BF16, _lib.TDA_BF16, 1, 2, 128, 64, 1.0,
                                 None, 0, 1, 2.0, 1, None, 0, 16, None)
    assert rc == _lib.TDA_ERR_INVALID
    rc = lib.tda_diff_fwd_lambda(16, 16, 16, 16, 16, None, 16, _lib.TDA_BF16, _lib.TDA_BF16, 1, 2, 128, 64, 1.0,
                                 16, -1, 1, 2.0, 1, None, 0, 16, None)
    assert rc == _lib.TDA_ERR_INVALID


def test_shape_mismatch_asserts_like_reference():
    q = torch.zeros(1, 2, 8, 64)
    k = torch.zeros(1, 2, 9, 64)
    with pytest.raises(AssertionError):
        tda_b200.threshold_rela_triton(q, k, q, torch.tensor(1.0))


def test_cpu_tensors_raise_no_fallback():
    q = torch.randn(1, 2, 8, 64)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        tda_b200.threshold_rela_triton(q, q, q, torch.tensor(1.0), 2.0)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        tda_b200.differential_threshold_rela_triton(q, q, q, q, q, torch.tensor(1.0), torch.tensor(0.5))


def test_reference_module_name_is_importable():
    from tda_b200 import triton_threshold_attention as tta
    assert tta.threshold_rela_triton is tda_b200.threshold_rela_triton
    assert tta.differential_threshold_rela_triton is tda_b200.differential_threshold_rela_triton
