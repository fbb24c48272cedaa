"""kvbm_b200.service."""
