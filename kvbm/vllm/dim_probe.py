"""``kvbm.vllm.dim_probe`` names, implemented by :mod:`kvbm_b200.connector.dim_probe`."""

from kvbm_b200.connector.dim_probe import *  # noqa: F401,F403
