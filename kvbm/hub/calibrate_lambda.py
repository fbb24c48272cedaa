"""``kvbm.hub.calibrate_lambda``: the engine side of a hub-triggered calibration sweep."""

from kvbm_b200.hub.calibrate_lambda import capture_calibration_defaults, make_calibrate_lambda  # noqa: F401
