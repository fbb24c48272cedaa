"""kvbm_b200.consolidator."""
