"""B200-native fused tensor-parallel RMSNorm.

Drop-in for the reference package ``rmsnorm_tp`` (haowen-han/RmsnormTP):
``FusedTPRMSNorm(hidden_dim, eps, tp_group, num_max_rows).forward(x, weight)``
and ``destroy()``. The compute runs in the C-ABI library
``_C/librmsnorm_tp_b200.so`` (hand-written sm_100a kernels); importing this
package fails if that library has not been built.
"""
from ._lib import RMSNormTPDeviceError, RMSNormTPError
from .api import (
    EmulatedTPGroup,
    EmulatedTPLinearGroup,
    exchange_handles,
    FusedTPLinearRMSNorm,
    FusedTPRMSNorm,
    IpcHandle,
    TPCommBuffer,
    buffer_of,
    dtype_code,
    local_rmsnorm,
    local_rmsnorm_backward,
    plan,
    plan_coverage,
    profile_counters,
    profile_summary,
    PROFILE_COUNTERS,
    set_kernel_family,
    get_kernel_family,
    set_push_mode,
    get_push_mode,
    set_dependent_launch,
    get_dependent_launch,
    tag_of,
)

__all__ = [
    "FusedTPRMSNorm",
    "FusedTPLinearRMSNorm",
    "EmulatedTPLinearGroup",
    "TPCommBuffer",
    "IpcHandle",
    "EmulatedTPGroup",
    "exchange_handles",
    "local_rmsnorm",
    "local_rmsnorm_backward",
    "RMSNormTPError",
    "RMSNormTPDeviceError",
    "plan",
    "plan_coverage",
    "profile_counters",
    "profile_summary",
    "PROFILE_COUNTERS",
    "tag_of",
    "set_kernel_family",
    "get_kernel_family",
    "set_push_mode",
    "get_push_mode",
    "set_dependent_launch",
    "get_dependent_launch",
    "buffer_of",
    "dtype_code",
]
