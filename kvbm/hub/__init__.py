"""``kvbm.hub``: prefill-router handler, completion event, hub client."""

from kvbm_b200.hub.client import CompletionEvent, HubClient, PrefillRouterHandler  # noqa: F401
from kvbm_b200.hub.detect import make_dispatch_lambda, try_wrap_engine  # noqa: F401
