"""``kvbm.hub.dispatch_lambda``: routed prefills as engine.generate calls."""

from kvbm_b200.hub.detect import make_dispatch_lambda  # noqa: F401
