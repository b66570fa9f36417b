"""ctypes binding of the C-ABI library ``_C/librmsnorm_tp_b200.so``.

This is the stub a maintainer of the reference would add in place of its
pybind11 module ``rmsnorm_tp_cpp`` (reference csrc/bindings.cpp:150-197).
There is no fallback: if the library is missing, importing the package fails
with the command that builds it.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_C", "librmsnorm_tp_b200.so")

# enum rmsnorm_tp_dtype
F32, BF16, F16 = 0, 1, 2
# enum rmsnorm_tp_error
OK, ERR_INVALID, ERR_CUDA, ERR_STATE, ERR_ROWS, ERR_DEVICE, ERR_HANDLE = range(7)
# enum rmsnorm_tp_device_status
STATUS_OK, STATUS_TIMEOUT, STATUS_ABORTED, STATUS_LOAD_TIMEOUT = 0, 1, 2, 3
# kernel families (rmsnorm_tp_set_kernel_family)
FAMILY_AUTO, FAMILY_REGISTER, FAMILY_BULK, FAMILY_BATCH = 0, 1, 2, 3
# push encodings (rmsnorm_tp_set_push_mode)
PUSH_PACKED, PUSH_RELEASE = 0, 1

MAX_TP = 8
HANDLE_BYTES = 128

_c_void_p = ctypes.c_void_p
_i32 = ctypes.c_int
_i64 = ctypes.c_int64
_u32 = ctypes.c_uint32
_u64 = ctypes.c_uint64
_sz = ctypes.c_size_t


class StatusInfo(ctypes.Structure):
    """struct rmsnorm_tp_status_info"""

    _fields_ = [
        ("code", _u32),
        ("src_rank", _u32),
        ("row", _i64),
        ("expected_tag", _u32),
        ("seen_tag", _u32),
        ("generation", _u64),
        ("next_generation", _u64),
    ]


class PlanInfo(ctypes.Structure):
    """struct rmsnorm_tp_plan_info"""

    _fields_ = [
        ("variant", _i32),
        ("vec_per_lane", _i32),
        ("team_warps", _i32),
        ("rows_per_tile", _i32),
        ("block_threads", _i32),
        ("teams_per_cta", _i32),
        ("tiles", _i64),
        ("grid", _i32),
        ("depth", _i32),
    ]


# name -> (restype, argtypes); every symbol of include/rmsnorm_tp_b200.h
SIGNATURES = {
    "rmsnorm_tp_create": (_i32, [_i32, _i32, _i64, _i32, ctypes.POINTER(_c_void_p)]),
    "rmsnorm_tp_export_handle": (_i32, [_c_void_p, _c_void_p, _sz, ctypes.POINTER(_sz)]),
    "rmsnorm_tp_open_peer": (_i32, [_c_void_p, _i32, ctypes.c_char_p, _sz]),
    "rmsnorm_tp_attach_peer": (_i32, [_c_void_p, _i32, _c_void_p]),
    "rmsnorm_tp_mailbox": (_i32, [_c_void_p, ctypes.POINTER(_c_void_p), ctypes.POINTER(_sz)]),
    "rmsnorm_tp_finalize": (_i32, [_c_void_p]),
    "rmsnorm_tp_destroy": (_i32, [_c_void_p]),
    "rmsnorm_tp_forward": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i32, ctypes.c_float, _c_void_p],
    ),
    "rmsnorm_local_forward": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i32, ctypes.c_float, _c_void_p],
    ),
    "rmsnorm_tp_forward_residual": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i32,
         ctypes.c_float, _c_void_p],
    ),
    "rmsnorm_local_forward_residual": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i32, ctypes.c_float, _c_void_p],
    ),
    "rmsnorm_tp_set_timeout": (_i32, [_c_void_p, _u64]),
    "rmsnorm_tp_set_profile": (_i32, [_c_void_p, _c_void_p]),
    "rmsnorm_tp_poll_error": (_i32, [_c_void_p, ctypes.POINTER(_u32)]),
    "rmsnorm_tp_status": (_i32, [_c_void_p, ctypes.POINTER(StatusInfo)]),
    "rmsnorm_tp_reset": (_i32, [_c_void_p, _u64]),
    "rmsnorm_tp_get_generation": (_i32, [_c_void_p, ctypes.POINTER(_u64)]),
    "rmsnorm_tp_forward_emulated": (
        _i32,
        [
            ctypes.POINTER(_c_void_p), _i32, ctypes.POINTER(_c_void_p), ctypes.POINTER(_c_void_p),
            ctypes.POINTER(_c_void_p), _i64, _i64, _i32, ctypes.c_float, _c_void_p,
        ],
    ),
    "rmsnorm_tp_forward_emulated_residual": (
        _i32,
        [
            ctypes.POINTER(_c_void_p), _i32, ctypes.POINTER(_c_void_p), ctypes.POINTER(_c_void_p),
            ctypes.POINTER(_c_void_p), ctypes.POINTER(_c_void_p), _i64, _i64, _i32, ctypes.c_float,
            _c_void_p,
        ],
    ),
    "rmsnorm_tp_create_linear": (_i32, [_i32, _i32, _i64, _i64, _i32, ctypes.POINTER(_c_void_p)]),
    "rmsnorm_tp_linear_forward": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i32,
         ctypes.c_float, _c_void_p],
    ),
    "rmsnorm_tp_linear_forward_emulated": (
        _i32,
        [
            ctypes.POINTER(_c_void_p), _i32, ctypes.POINTER(_c_void_p), ctypes.POINTER(_c_void_p),
            ctypes.POINTER(_c_void_p), ctypes.POINTER(_c_void_p), ctypes.POINTER(_c_void_p), _i64,
            _i64, _i32, ctypes.c_float, _c_void_p,
        ],
    ),
    "rmsnorm_tp_backward_workspace_bytes": (_sz, [_i64, _i64]),
    "rmsnorm_tp_backward": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i32,
         ctypes.c_float, _c_void_p, _sz, _c_void_p],
    ),
    "rmsnorm_local_backward": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i32, ctypes.c_float,
         _c_void_p, _sz, _c_void_p],
    ),
    "rmsnorm_tp_backward_emulated": (
        _i32,
        [
            ctypes.POINTER(_c_void_p), _i32, ctypes.POINTER(_c_void_p), ctypes.POINTER(_c_void_p),
            ctypes.POINTER(_c_void_p), ctypes.POINTER(_c_void_p), ctypes.POINTER(_c_void_p), _i64,
            _i64, _i32, ctypes.c_float, ctypes.POINTER(_c_void_p), _sz, _c_void_p,
        ],
    ),
    "rmsnorm_tp_forward_group_static": (
        _i32,
        [
            _i32, ctypes.POINTER(_c_void_p), ctypes.POINTER(_c_void_p), ctypes.POINTER(_c_void_p),
            _i64, _i64, _i32, ctypes.c_float, _c_void_p,
        ],
    ),
    "rmsnorm_tp_forward_group_static_status": (_i32, [ctypes.POINTER(StatusInfo)]),
    "rmsnorm_tp_probe_roundtrip": (_i32, [_c_void_p, _i32, _i32, _c_void_p, _c_void_p]),
    "rmsnorm_tp_plan": (_i32, [_i64, _i64, _i32, _i32, _i32, _i32, ctypes.POINTER(PlanInfo)]),
    "rmsnorm_tp_set_kernel_family": (_i32, [_i32]),
    "rmsnorm_tp_get_kernel_family": (_i32, []),
    "rmsnorm_tp_set_push_mode": (_i32, [_i32]),
    "rmsnorm_tp_get_push_mode": (_i32, []),
    "rmsnorm_tp_set_dependent_launch": (_i32, [_i32]),
    "rmsnorm_tp_get_dependent_launch": (_i32, []),
    "rmsnorm_tp_plan_coverage": (_i32, [ctypes.POINTER(PlanInfo), _i64, ctypes.POINTER(ctypes.c_int32)]),
    "rmsnorm_tp_tag_of": (_u32, [_u64]),
    "rmsnorm_tp_buffer_of": (_u32, [_u64]),
    "rmsnorm_tp_last_error": (ctypes.c_char_p, []),
    "rmsnorm_tp_abi_version": (_i32, []),
}


class RMSNormTPError(RuntimeError):
    """A C-ABI call failed; ``code`` is the rmsnorm_tp_error value."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class RMSNormTPDeviceError(RMSNormTPError):
    """A launch recorded a device-side failure (a peer's partial sum never arrived)."""


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"rmsnorm_tp_b200: native library {LIB_PATH} is missing; build it with "
            "`python rmsnorm_tp_b200/build.py` (needs nvcc). There is no CPU fallback."
        )
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


LIB = _load()


def last_error() -> str:
    msg = LIB.rmsnorm_tp_last_error()
    return msg.decode("utf-8", "replace") if msg else ""


def check(rc: int, what: str) -> None:
    """Raise the matching exception for a nonzero status code."""
    if rc == OK:
        return
    msg = f"{what}: {last_error()}"
    if rc == ERR_DEVICE:
        raise RMSNormTPDeviceError(rc, msg)
    raise RMSNormTPError(rc, msg)
