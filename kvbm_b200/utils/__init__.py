"""kvbm_b200.utils."""
