"""kvbm_b200.hub."""
