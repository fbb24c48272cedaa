"""kvbm_b200.models."""
