"""kvbm_b200.physical."""
