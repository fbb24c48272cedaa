"""kvbm_b200.ops."""
