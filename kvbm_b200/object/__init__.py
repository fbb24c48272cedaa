"""kvbm_b200.object."""
