"""``kvbm.hub``: prefill-router handler, completion event, hub client, engine attach and calibration."""

from kvbm_b200.hub.calibrate_lambda import capture_calibration_defaults, make_calibrate_lambda  # noqa: F401
from kvbm_b200.hub.client import CompletionEvent, HubClient, PrefillRouterHandler  # noqa: F401
from kvbm_b200.hub.detect import make_dispatch_lambda, try_wrap_engine  # noqa: F401
