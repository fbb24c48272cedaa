"""kvbm_b200.common."""
