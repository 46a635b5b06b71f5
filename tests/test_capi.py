"""The C-ABI library loads, exports every symbol include/pa_kernels.h declares,
and rejects invalid arguments with the documented status codes before any
device work (no GPU needed)."""
import ctypes
import os
import re

import pytest

from conftest import REPO


def _declared_symbols():
    hdr = open(os.path.join(REPO, "include", "pa_kernels.h")).read()
    hdr = re.sub(r"/\*.*?\*/", "", hdr, flags=re.S)
    return sorted(set(re.findall(r"\b(pa_[a-z0-9_]+)\s*\(", hdr)))


def test_header_and_binding_agree():
    import pa_capi
    assert sorted(pa_capi.EXPORTS) == _declared_symbols()


def test_library_exports_every_declared_symbol():
    import pa_capi
    lib = pa_capi.load()
    for name in _declared_symbols():
        assert hasattr(lib, name), name


def test_abi_version_and_status_strings():
    import pa_capi
    lib = pa_capi.load()
    assert lib.pa_abi_version() == 1
    for code in range(10):
        assert lib.pa_status_string(code)


def test_attention_argument_validation_without_gpu():
    import pa_capi
    lib = pa_capi.load()
    fwd = lib.pa_attn_fwd
    assert fwd(None, None, None, None, None, None, None, 0, None) == 8  # PA_ERR_NULL
    d = pa_capi.AttnDesc(1, 128, 1, 96, pa_capi.PA_BF16, 0.0)
    assert fwd(ctypes.byref(d), 16, 16, 16, 16, 16, None, 0, None) == 4  # head_dim 96
    d = pa_capi.AttnDesc(0, 128, 1, 64, pa_capi.PA_BF16, 0.0)
    assert fwd(ctypes.byref(d), 16, 16, 16, 16, 16, None, 0, None) == 1  # batch 0
    d = pa_capi.AttnDesc(1, 128, 1, 64, 7, 0.0)
    assert fwd(ctypes.byref(d), 16, 16, 16, 16, 16, None, 0, None) == 2  # dtype
    d = pa_capi.AttnDesc(1, 128, 1, 64, pa_capi.PA_BF16, 0.0)
    assert fwd(ctypes.byref(d), 16, 17, 16, 16, 16, None, 0, None) == 3  # misaligned k
    assert fwd(ctypes.byref(d), 16, 16, 16, 16, None, None, 0, None) == 8  # lse NULL
    assert lib.pa_attn_fwd_workspace_size(ctypes.byref(d)) == 0          # bf16: none
    d32 = pa_capi.AttnDesc(1, 128, 1, 32, pa_capi.PA_F32, 0.0)
    assert lib.pa_attn_fwd_workspace_size(ctypes.byref(d32)) >= 6 * 128 * 64 * 2
    assert fwd(ctypes.byref(d32), 16, 16, 16, 16, 16, None, 0, None) == 7  # f32 needs workspace
    d128 = pa_capi.AttnDesc(1, 128, 1, 128, pa_capi.PA_F32, 0.0)
    assert fwd(ctypes.byref(d128), 16, 16, 16, 16, 16, None, 0, None) == 4  # f32 d=128
    ws = lib.pa_attn_bwd_workspace_size(ctypes.byref(d))
    assert ws >= 128 * 64 * 4
    bwd = lib.pa_attn_bwd
    assert bwd(ctypes.byref(d), *([16] * 9), 0, None, 0, None) == 7   # no workspace
    assert bwd(ctypes.byref(d), *([16] * 9), 0, 256, ws - 1, None) == 7
    assert bwd(ctypes.byref(d), *([16] * 9), 0, 260, ws, None) == 3   # misaligned workspace


def test_layer_norm_and_matmul_validation_without_gpu():
    import pa_capi
    lib = pa_capi.load()
    assert lib.pa_layer_norm_fwd(None, None, None, None, None, None, 4, 8, 1e-5, None) == 8
    assert lib.pa_layer_norm_fwd(16, 16, 16, 16, 16, 16, 0, 8, 1e-5, None) == 1
    assert lib.pa_layer_norm_fwd(16, 16, 16, 16, 16, 16, 4, 6, 1e-5, None) == 4
    assert lib.pa_layer_norm_bwd(16, 16, 16, 16, 16, 16, 16, 16, 4, 8, None, 0, None) == 7
    # fused residual add: NULL sum, zero rows, N not a multiple of 4, misaligned r, sum aliasing x
    assert lib.pa_add_layer_norm_fwd(16, 16, None, 16, 16, 16, 16, 16, 4, 8, 1e-5, None) == 8
    assert lib.pa_add_layer_norm_fwd(16, 32, 48, 16, 16, 16, 16, 16, 0, 8, 1e-5, None) == 1
    assert lib.pa_add_layer_norm_fwd(16, 32, 48, 16, 16, 16, 16, 16, 4, 6, 1e-5, None) == 4
    assert lib.pa_add_layer_norm_fwd(16, 36, 48, 16, 16, 16, 16, 16, 4, 8, 1e-5, None) == 3
    assert lib.pa_add_layer_norm_fwd(16, 32, 16, 16, 16, 16, 16, 16, 4, 8, 1e-5, None) == 1
    # the same with the output's operand planes: planes NULL, r without sum, too few plane
    # bytes, planes not 256-byte aligned, N not a multiple of 4
    pl = lib.pa_layer_norm_fwd_planes
    need = lib.pa_linear_kept_size(4, 8)
    assert need > 0
    assert pl(16, None, None, 16, 16, 16, 16, 16, 4, 8, 1e-5, None, need, None) == 8
    assert pl(16, 32, None, 16, 16, 16, 16, 16, 4, 8, 1e-5, 256, need, None) == 8
    assert pl(16, None, None, 16, 16, 16, 16, 16, 4, 8, 1e-5, 256, need - 1, None) == 1
    assert pl(16, None, None, 16, 16, 16, 16, 16, 4, 8, 1e-5, 272, need, None) == 3
    assert pl(16, None, None, 16, 16, 16, 16, 16, 4, 6, 1e-5, 256, need, None) == 4
    assert lib.pa_matmul(16, 16, 16, 0, 4, 4, None, 0, None) == 1
    assert lib.pa_matmul_grad_x(None, 16, 16, 4, 4, 4, None, 0, None) == 8
    assert lib.pa_matmul_grad_w(16, 16, 16, 4, 4, 4, None, 0, None) == 7   # no workspace
    assert lib.pa_matmul_workspace_size(8192, 1536, 512) >= 4 * 8192 * 1536
    assert lib.pa_split_last_dim(16, None, 3, 4, 4, None) == 8
    arr = (ctypes.c_void_p * 9)(*([16] * 9))
    assert lib.pa_split_last_dim(16, arr, 9, 4, 4, None) == 1          # more than 8 parts
