"""The engine side of a calibration sweep.

:func:`make_calibrate_lambda` builds the callable a
:class:`~kvbm_b200.hub.client.PrefillRouterHandler` invokes when the hub asks
its prefill engine to calibrate: ``(resolved: dict, event) -> None``. It
schedules the sweep on the engine's event loop and returns at once; the
sweep sends one request at a time (optionally a small warm-up first), each
``isl`` tokens long with ``osl`` generated tokens (``ignore_eos``), records
the time to the first streamed output and the gap between later outputs, and
completes ``event`` with ``{"traces": [...]}`` (or fails it with the error).
The fitting happens in the handler (``hub.calibration.analyze``).

Every request's first token is a cache buster: a fresh id from
``buster_vocab`` (a counter seeded from the clock, so sweeps in one process
never repeat one), so neither the engine's prefix cache nor a G2 index hit
serves a calibration prompt. Body tokens come from ``body_vocab`` with the
sweep's seed.

:func:`capture_calibration_defaults` reads the engine's limits (context,
input and output caps, vocabulary size) for the handler to resolve requests
against.

Parity: python/kvbm/hub/calibrate_lambda.py (capture_calibration_defaults,
make_calibrate_lambda).
"""

from __future__ import annotations

import asyncio
import itertools
import random
import time
import uuid
from typing import Any, Callable


def capture_calibration_defaults(engine: Any, model_id: str) -> dict:
    """The engine's calibration limits as a plain dict (``CalibrationDefaults`` fields)."""
    cfg = getattr(engine, "model_config", None)
    if cfg is None:
        cfg = getattr(getattr(engine, "vllm_config", None), "model_config", None)
    if cfg is None:
        raise RuntimeError("capture_calibration_defaults: engine has no model_config / vllm_config")
    max_len = int(getattr(cfg, "max_model_len", 0) or getattr(cfg, "max_seq_len", 0) or 0)
    if max_len <= 0:
        raise RuntimeError("capture_calibration_defaults: could not read max_model_len from the engine")
    vocab = 0
    tok = getattr(engine, "tokenizer", None)
    if tok is not None:
        vocab = int(getattr(tok, "vocab_size", 0) or getattr(getattr(tok, "tokenizer", None), "vocab_size", 0) or 0)
    if vocab <= 0:  # engines started without a tokenizer: the model's own vocabulary
        hf = getattr(cfg, "hf_config", None)
        vocab = int(getattr(hf, "vocab_size", 0) or 0) or int(getattr(cfg, "get_vocab_size", lambda: 0)() or 0)
    if vocab <= 0:
        raise RuntimeError("capture_calibration_defaults: could not read the vocabulary size")
    return {"model_id": model_id, "max_seq_len": max_len,
            "max_input_len": int(getattr(cfg, "max_input_len", 0) or max_len),
            "max_output_len": int(getattr(cfg, "max_output_len", 0) or max_len),
            "vocab_size": vocab, "safe_vocab_lo": min(1000, max(1, vocab // 4))}


def _vllm_request(token_ids: list[int], osl: int):
    from vllm.inputs import TokensPrompt
    from vllm.sampling_params import SamplingParams

    return (TokensPrompt(prompt_token_ids=token_ids),
            SamplingParams(max_tokens=osl, min_tokens=osl, ignore_eos=True, temperature=0.0, detokenize=False))


def make_calibrate_lambda(engine: Any, loop: asyncio.AbstractEventLoop,
                          make_request: Callable[[list[int], int], tuple] | None = None) -> Callable[[dict, Any], None]:
    """``(resolved, event) -> None`` for a :class:`PrefillRouterHandler`; ``engine.generate(prompt,
    params, request_id)`` must be an async iterator of streamed outputs. ``make_request(token_ids,
    osl)`` builds (prompt, params) (vLLM's types by default)."""
    make_request = make_request or _vllm_request
    bust = itertools.count(time.time_ns())

    async def one(isl: int, osl: int, rng: random.Random, body: tuple[int, int], buster: tuple[int, int]) -> dict:
        if isl < 2:
            raise ValueError("isl must be >= 2 (a cache-buster token and a body)")
        first = buster[0] + next(bust) % max(1, buster[1] - buster[0])
        ids = [first] + [rng.randrange(body[0], body[1]) for _ in range(isl - 1)]
        prompt, params = make_request(ids, osl)
        t0 = time.monotonic_ns()
        ttft_us, prev, gaps = None, None, []
        async for _ in engine.generate(prompt, params, f"kvbm-calibrate-{uuid.uuid4().hex}"):
            now = (time.monotonic_ns() - t0) // 1000
            if ttft_us is None:
                ttft_us = now
            else:
                gaps.append(now - prev)
            prev = now
        if ttft_us is None:
            raise RuntimeError(f"the engine streamed no output for isl={isl}")
        return {"isl": isl, "osl": osl, "ttft_us": int(ttft_us), "itl_us": [int(g) for g in gaps],
                "first_token": int(first)}

    async def run(resolved: dict, event) -> None:
        try:
            rng = random.Random(int(resolved["seed"]))
            body = tuple(int(v) for v in resolved["body_vocab"])
            buster = tuple(int(v) for v in resolved["buster_vocab"])
            osl = int(resolved["osl"])
            if resolved.get("warmup", True):
                await one(min(128, max(2, min(resolved["seq"]))), min(16, osl), rng, body, buster)
            traces = [await one(int(isl), osl, rng, body, buster) for isl in resolved["seq"]]
            event.complete({"traces": traces})
        except BaseException as e:  # noqa: BLE001 - every failure reaches the waiting handler
            event.fail(repr(e))

    def calibrate(resolved: dict, event) -> None:
        asyncio.run_coroutine_threadsafe(run(resolved, event), loop)

    return calibrate
