"""kvbm_b200.logical."""
