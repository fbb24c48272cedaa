"""``kvbm.hub.detect``: attach a prefill-role vLLM engine to the hub's prefill router."""

from kvbm_b200.hub.detect import connector_settings, try_wrap_engine  # noqa: F401
