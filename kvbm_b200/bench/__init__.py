"""kvbm_b200.bench."""
