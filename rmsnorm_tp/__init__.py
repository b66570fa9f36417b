"""Drop-in import name of the reference package (``from rmsnorm_tp import
FusedTPRMSNorm``); everything lives in ``rmsnorm_tp_b200``."""
from rmsnorm_tp_b200 import FusedTPRMSNorm, IpcHandle, TPCommBuffer  # noqa: F401

__all__ = ["FusedTPRMSNorm", "TPCommBuffer", "IpcHandle"]
