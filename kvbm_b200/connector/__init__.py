"""kvbm_b200.connector."""
