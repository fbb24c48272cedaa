"""``kvbm.hub``: prefill-router handler, completion event, hub client."""

from kvbm_b200.hub.client import CompletionEvent, HubClient, PrefillRouterHandler  # noqa: F401
