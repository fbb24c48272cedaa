"""``kvbm._core`` names, implemented by :mod:`kvbm_b200._core`."""

from kvbm_b200._core import *  # noqa: F401,F403
from kvbm_b200._core import hub  # noqa: F401
from kvbm_b200 import kernels  # noqa: F401,E402
