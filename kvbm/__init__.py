"""``kvbm`` import path for users of the reference package: the same module names
(``kvbm._core``, ``kvbm.kernels``, ``kvbm.vllm.connector``, ``kvbm.vllm.dim_probe``, ``kvbm.hub``)
and the same root names, backed by kvbm_b200."""

from kvbm_b200 import __version__  # noqa: F401
from kvbm_b200._core import (ConnectorLeader, ConnectorWorker, KvbmRequest, KvbmRuntime,  # noqa: F401
                             KvbmVllmConfig, SchedulerOutput, Tensor, is_available)

from . import kernels  # noqa: F401,E402  (the sm_100a kernels are part of this build, never a stub)

_CORE_AVAILABLE = True
_KERNELS_AVAILABLE = True

__all__ = ["__version__", "is_available", "KvbmRuntime", "KvbmVllmConfig", "ConnectorLeader", "ConnectorWorker",
           "KvbmRequest", "SchedulerOutput", "Tensor", "kernels", "_CORE_AVAILABLE", "_KERNELS_AVAILABLE"]
