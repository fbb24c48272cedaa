"""``kvbm`` import path for users of the reference package: the same module
names (``kvbm._core``, ``kvbm.vllm.connector``, ``kvbm.vllm.dim_probe``,
``kvbm.hub``) backed by kvbm_b200."""

from kvbm_b200 import __version__  # noqa: F401
from kvbm_b200._core import is_available  # noqa: F401
