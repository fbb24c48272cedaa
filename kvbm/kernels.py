"""``kvbm.kernels``: tensor-level block permutes and copies (sm_100a kernels of kvbm_b200)."""

from kvbm_b200.kernels import (block_to_operational, block_to_universal, operational_to_block,  # noqa: F401
                               universal_to_block)
