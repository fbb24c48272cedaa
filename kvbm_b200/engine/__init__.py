"""kvbm_b200.engine."""
