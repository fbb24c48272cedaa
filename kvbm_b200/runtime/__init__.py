"""kvbm_b200.runtime: control-plane messaging and runtime assembly."""
