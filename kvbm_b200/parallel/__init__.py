"""kvbm_b200.parallel."""
