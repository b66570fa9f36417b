"""The C-ABI library loads without a GPU and exports exactly what
include/rmsnorm_tp_b200.h declares; argument checks run before any CUDA call."""
import ctypes
import os
import re

import pytest

from conftest import ROOT
from rmsnorm_tp_b200 import _lib

HEADER = os.path.join(ROOT, "include", "rmsnorm_tp_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b((?:rmsnorm)_\w+)\s*\(", text)))


def test_header_declares_functions():
    names = declared_functions()
    assert "rmsnorm_tp_forward" in names and "rmsnorm_tp_create" in names
    assert len(names) >= 20


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_the_header():
    assert sorted(_lib.SIGNATURES) == declared_functions()


def test_abi_version():
    assert _lib.LIB.rmsnorm_tp_abi_version() == 103


@pytest.mark.parametrize("rank,tp,nmax", [(2, 2, 16), (-1, 2, 16), (0, 0, 16), (0, 9, 16), (0, 2, 0)])
def test_create_rejects_bad_arguments_before_touching_cuda(rank, tp, nmax):
    out = ctypes.c_void_p()
    rc = _lib.LIB.rmsnorm_tp_create(rank, tp, nmax, 0, ctypes.byref(out))
    assert rc == _lib.ERR_INVALID
    assert out.value is None
    assert _lib.last_error().startswith("create:")


def test_null_communicator_is_an_error_not_a_crash():
    L = _lib.LIB
    assert L.rmsnorm_tp_forward(None, None, None, None, 1, 8, 8, 0, 1e-6, None) == _lib.ERR_INVALID
    assert L.rmsnorm_tp_finalize(None) == _lib.ERR_INVALID
    assert L.rmsnorm_tp_destroy(None) == _lib.OK
    assert L.rmsnorm_tp_open_peer(None, 1, b"x" * 128, 128) == _lib.ERR_INVALID
    assert L.rmsnorm_tp_set_timeout(None, 5) == _lib.ERR_INVALID
    code = ctypes.c_uint32()
    assert L.rmsnorm_tp_poll_error(None, ctypes.byref(code)) == _lib.ERR_INVALID


def test_local_forward_validates_shape_without_gpu():
    L = _lib.LIB
    assert L.rmsnorm_local_forward(None, None, None, 4, 8, 7, 1e-6, None) == _lib.ERR_INVALID  # dtype
    assert L.rmsnorm_local_forward(None, None, None, -1, 8, 0, 1e-6, None) == _lib.ERR_INVALID  # rows
    assert L.rmsnorm_local_forward(None, None, None, 4, 0, 0, 1e-6, None) == _lib.ERR_INVALID  # width
    assert L.rmsnorm_local_forward(None, None, None, 4, 8, 0, 1e-6, None) == _lib.ERR_INVALID  # NULL
    assert L.rmsnorm_local_forward(None, None, None, 0, 8, 0, 1e-6, None) == _lib.OK  # no rows: no launch


def test_residual_entry_points_validate_without_gpu():
    L = _lib.LIB
    out, x, w = 0x10000, 0x20000, 0x30000          # never dereferenced: every call fails first
    # NULL residual
    assert L.rmsnorm_local_forward_residual(out, None, x, w, 4, 8, 0, 1e-6, None) == _lib.ERR_INVALID
    assert L.rmsnorm_tp_forward_residual(None, out, None, x, w, 4, 8, 16, 0, 1e-6, None) == \
        _lib.ERR_INVALID
    # residual overlapping the output (4 rows x 8 fp32 = 128 bytes)
    assert L.rmsnorm_local_forward_residual(out, out, x, w, 4, 8, 0, 1e-6, None) == _lib.ERR_INVALID
    assert L.rmsnorm_local_forward_residual(out, out + 124, x, w, 4, 8, 0, 1e-6, None) == \
        _lib.ERR_INVALID
    assert "overlaps" in _lib.last_error()
    # adjacent is fine up to the launch, which needs a communicator / GPU: no rows -> no launch
    assert L.rmsnorm_local_forward_residual(out, out + 128, x, w, 0, 8, 0, 1e-6, None) == _lib.OK
    assert L.rmsnorm_tp_forward_emulated_residual(None, 2, None, None, None, None, 4, 8, 0, 1e-6,
                                                  None) == _lib.ERR_INVALID


def test_backward_entry_points_validate_without_gpu():
    L = _lib.LIB
    assert L.rmsnorm_tp_backward_workspace_bytes(0, 64) == 0
    assert L.rmsnorm_tp_backward_workspace_bytes(10, 64) == 10 * 64 * 4
    assert L.rmsnorm_tp_backward_workspace_bytes(100000, 64) == 296 * 64 * 4   # grid bound
    dx, dw, dy, x, w, ws = 0x10000, 0x20000, 0x30000, 0x40000, 0x50000, 0x60000
    need = L.rmsnorm_tp_backward_workspace_bytes(4, 8)
    # workspace too small
    assert L.rmsnorm_local_backward(dx, dw, dy, x, w, 4, 8, 0, 1e-6, ws, need - 1, None) == \
        _lib.ERR_INVALID
    # dx overlapping dy / x
    assert L.rmsnorm_local_backward(dy, dw, dy, x, w, 4, 8, 0, 1e-6, ws, need, None) == _lib.ERR_INVALID
    assert L.rmsnorm_local_backward(x + 8, dw, dy, x, w, 4, 8, 0, 1e-6, ws, need, None) == \
        _lib.ERR_INVALID
    # NULL dw, width above the shared-memory bound
    assert L.rmsnorm_local_backward(dx, None, dy, x, w, 4, 8, 0, 1e-6, ws, need, None) == \
        _lib.ERR_INVALID
    assert L.rmsnorm_local_backward(dx, dw, dy, x, w, 1, 53249, 0, 1e-6, ws, 1 << 20, None) == \
        _lib.ERR_INVALID
    assert L.rmsnorm_tp_backward(None, dx, dw, dy, x, w, 4, 8, 16, 0, 1e-6, ws, need, None) == \
        _lib.ERR_INVALID
    assert L.rmsnorm_tp_backward_emulated(None, 2, None, None, None, None, None, 4, 8, 0, 1e-6,
                                          None, need, None) == _lib.ERR_INVALID


def test_check_maps_codes_to_exceptions():
    with pytest.raises(_lib.RMSNormTPDeviceError):
        _lib.check(_lib.ERR_DEVICE, "x")
    with pytest.raises(_lib.RMSNormTPError) as e:
        _lib.check(_lib.ERR_INVALID, "x")
    assert e.value.code == _lib.ERR_INVALID and isinstance(e.value, RuntimeError)


def test_dependent_launch_switch_round_trips_and_rejects_other_values():
    L = _lib.LIB
    before = L.rmsnorm_tp_get_dependent_launch()
    assert before == 1                                  # on by default
    try:
        assert L.rmsnorm_tp_set_dependent_launch(0) == _lib.OK
        assert L.rmsnorm_tp_get_dependent_launch() == 0
        assert L.rmsnorm_tp_set_dependent_launch(2) == _lib.ERR_INVALID
        assert L.rmsnorm_tp_get_dependent_launch() == 0  # unchanged by the rejected call
        assert L.rmsnorm_tp_set_dependent_launch(1) == _lib.OK
        assert L.rmsnorm_tp_get_dependent_launch() == 1
    finally:
        L.rmsnorm_tp_set_dependent_launch(before)
