"""CPU tests of the native boundary: the C-ABI library loads, exports every
function include/flashlite_b200.h declares, rejects invalid arguments before
touching a device, and the torch binding reproduces the reference's error
messages (thebigblender/FlashLite csrc/kernel_flash2.cu:741-764,
csrc/kernel_naive.cu:252-276). No kernel is launched here."""
import ctypes

import pytest
import torch

from flashlite_b200 import flash_attn_wmma as fa

FL_OK, FL_ERR_INVALID_ARGUMENT, FL_ERR_UNSUPPORTED = 0, 1, 2


def test_header_declares_expected_api(header_fns):
    for name in ("fl_flash2_fwd", "fl_naive_fwd", "fl_flash2_fwd_block", "fl_ring_finalize",
                 "fl_status_str", "fl_last_error", "fl_device_error", "fl_version",
                 "fl_flash2_fwd_ex", "fl_flash2_bwd", "fl_flash2_bwd_workspace_size",
                 "fl_selftest_bounded_wait"):
        assert name in header_fns


def test_library_exports_every_header_symbol(fl_lib, header_fns):
    for name in header_fns:
        assert hasattr(fl_lib, name), f"{name} declared in the header but not exported"


def test_status_strings(fl_lib):
    assert fl_lib.fl_status_str(0) == b"ok"
    for code in range(1, 7):
        assert fl_lib.fl_status_str(code) not in (b"", b"unknown status")
    assert fl_lib.fl_status_str(99) == b"unknown status"
    assert fl_lib.fl_version().count(b".") == 2


def test_null_pointer_rejected(fl_lib):
    st = fl_lib.fl_flash2_fwd(None, None, None, None, 1, 1, 128, 64, 0.0, 0, None)
    assert st == FL_ERR_INVALID_ARGUMENT
    assert b"null" in fl_lib.fl_last_error()


def test_head_dim_rejected_before_device(fl_lib):
    buf = ctypes.create_string_buffer(64)
    p = ctypes.addressof(buf)
    st = fl_lib.fl_flash2_fwd(p, p, p, p, 1, 1, 128, 128, 0.0, 0, None)
    assert st == FL_ERR_UNSUPPORTED
    assert b"head_dim == 64" in fl_lib.fl_last_error()


def test_negative_size_rejected(fl_lib):
    buf = ctypes.create_string_buffer(64)
    p = ctypes.addressof(buf)
    assert fl_lib.fl_naive_fwd(p, p, p, p, -1, 1, 128, 64, 0.0, 0, None) == FL_ERR_INVALID_ARGUMENT
    assert fl_lib.fl_naive_fwd(p, p, p, p, 1, 1, 128, 2048, 0.0, 0, None) == FL_ERR_UNSUPPORTED
    assert fl_lib.fl_ring_finalize(None, None, -5, None) == FL_ERR_INVALID_ARGUMENT


def test_empty_inputs_are_noops(fl_lib):
    buf = ctypes.create_string_buffer(64)
    p = ctypes.addressof(buf)
    assert fl_lib.fl_flash2_fwd(p, p, p, p, 0, 8, 128, 64, 0.0, 1, None) == FL_OK
    assert fl_lib.fl_flash2_fwd(p, p, p, p, 2, 8, 0, 64, 0.0, 0, None) == FL_OK
    assert fl_lib.fl_ring_finalize(None, None, 0, None) == FL_OK


def _qkv(dtype=torch.float16, shape=(1, 2, 128, 64)):
    return [torch.zeros(shape, dtype=dtype) for _ in range(3)]


def test_binding_rejects_cpu_tensors():
    q, k, v = _qkv()
    with pytest.raises(RuntimeError, match="All tensors must be on CUDA"):
        fa.forward_flash2(q, k, v)
    with pytest.raises(RuntimeError, match="Query tensor must be on CUDA"):
        fa.forward_naive(q, k, v)


def test_binding_signature_defaults():
    doc = fa.forward_flash2.__doc__
    assert "sm_scale" in doc and "is_causal" in doc and "out" in doc
    assert "= 0.0" in doc and "= False" in doc and "= None" in doc
    assert "sm_scale" in fa.forward_naive.__doc__


def test_package_refuses_to_import_without_native_code(tmp_path, monkeypatch):
    # the package has no pure-Python path: its public functions are the
    # binding's own builtins
    assert type(fa.forward_flash2).__name__ == "builtin_function_or_method"
    assert type(fa.forward_naive).__name__ == "builtin_function_or_method"


def test_backward_checks_before_device(fl_lib):
    # fl_flash2_bwd validates pointers, head_dim and the workspace size
    # before it looks for a device
    vp, i64, sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_size_t
    fl_lib.fl_flash2_bwd_workspace_size.argtypes = [i64, i64, i64, i64]
    fl_lib.fl_flash2_bwd_workspace_size.restype = sz
    fl_lib.fl_flash2_bwd.argtypes = [vp] * 10 + [sz, i64, i64, i64, i64, ctypes.c_float, ctypes.c_int, ctypes.c_int, vp]
    need = fl_lib.fl_flash2_bwd_workspace_size(2, 8, 1000, 64)
    # fp32 dQ accumulator + two per-row vectors padded to 128-row tiles
    assert need == (2 * 8 * 1000 * 64 + 2 * 2 * 8 * 1024) * 4
    assert fl_lib.fl_flash2_bwd_workspace_size(2, 8, 1000, 128) == 0
    buf = ctypes.create_string_buffer(4096)
    p = ctypes.addressof(buf)
    args = [p] * 10
    assert fl_lib.fl_flash2_bwd(*([None] * 10), 0, 1, 1, 128, 64, 0.0, 0, 0, None) == FL_ERR_INVALID_ARGUMENT
    assert fl_lib.fl_flash2_bwd(*args, 4096, 1, 1, 128, 128, 0.0, 0, 0, None) == FL_ERR_UNSUPPORTED
    assert b"head_dim == 64" in fl_lib.fl_last_error()
    assert fl_lib.fl_flash2_bwd(*args, 16, 1, 1, 128, 64, 0.0, 0, 0, None) == FL_ERR_INVALID_ARGUMENT
    assert b"workspace too small" in fl_lib.fl_last_error()
    assert fl_lib.fl_flash2_bwd(*args, 0, 0, 1, 128, 64, 0.0, 0, 0, None) == FL_OK  # empty batch


def test_backward_binding_rejects_cpu_tensors():
    q, k, v = _qkv()
    lse = torch.zeros(1, 2, 128)
    with pytest.raises(RuntimeError, match="All tensors must be on CUDA"):
        fa.backward_flash2(q, k, v, q, q, lse)
    assert "is_causal" in fa.backward_flash2.__doc__ and "sm_scale" in fa.backward_flash2.__doc__


def test_selftest_bounded_wait_rejects_bad_arguments(fl_lib):
    """Checked before any device work: a null result buffer, a zero limit and
    a limit above one second are refused."""
    buf = ctypes.create_string_buffer(64)
    p = ctypes.addressof(buf)
    assert fl_lib.fl_selftest_bounded_wait(1000, None, None) == FL_ERR_INVALID_ARGUMENT
    assert fl_lib.fl_selftest_bounded_wait(0, p, None) == FL_ERR_INVALID_ARGUMENT
    assert fl_lib.fl_selftest_bounded_wait(2_000_000_000, p, None) == FL_ERR_INVALID_ARGUMENT
    assert b"limit_ns" in fl_lib.fl_last_error()
