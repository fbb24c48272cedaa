"""Prefill routing for conditional disaggregation: load-aware worker
selection, a tick-driven circuit breaker and TTFT/ITL calibration.

* :class:`Selector` picks, among prefill workers with free concurrency, the
  one with the lowest outstanding *net-new* prefill tokens (tokens the
  prefill must actually compute: prompt length minus the tokens the decode
  side already provides). A pick returns a charge that is released when the
  prefill finishes.
* :class:`CircuitBreaker` is a three-tier hysteresis state machine
  (calm -> warm -> hot) over fleet pressure (queued + in-flight net-new
  tokens per worker). It only narrows disaggregation (hot = decode should
  prefill locally) and is evaluated by a periodic tick, never by dispatch
  events (so it cannot latch in hot when traffic stops).
* :class:`Calibration` fits TTFT(ISL) as a quadratic and ITL as a linear
  function of context from measured samples (least squares), used to
  predict whether remote prefill pays off.

Parity: crates/kvbm-hub/src/features/prefill_router/{selection.rs,
breaker.rs, calibration.rs, dispatcher.rs, router.rs, protocol.rs
(targets / counters / calibrate routes)}.
"""

from __future__ import annotations

import enum
import threading
import time
from dataclasses import dataclass, field

import numpy as np


@dataclass
class WorkerSlot:
    instance_id: int
    max_inflight: int = 4
    inflight: int = 0
    load_net_new: int = 0
    dispatched: int = 0
    completed: int = 0
    detached: bool = False


class Charge:
    def __init__(self, sel: "Selector", slot: WorkerSlot, net_new: int):
        self.sel, self.slot, self.net_new = sel, slot, net_new
        self._done = False

    def release(self, ok: bool = True) -> None:
        if self._done:
            return
        self._done = True
        with self.sel._cv:
            self.slot.inflight -= 1
            self.slot.load_net_new -= self.net_new
            if ok:
                self.slot.completed += 1
            self.sel._cv.notify_all()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.release(ok=exc[0] is None)


class Selector:
    def __init__(self, max_inflight: int = 4, block_size: int = 16):
        self.max_inflight, self.block_size = max_inflight, block_size
        self._slots: dict[int, WorkerSlot] = {}
        self._cv = threading.Condition()

    @staticmethod
    def net_new_tokens(num_tokens: int, num_provided_tokens: int) -> int:
        return max(0, num_tokens - num_provided_tokens)

    def add_worker(self, instance_id: int, max_inflight: int | None = None) -> None:
        with self._cv:
            self._slots[instance_id] = WorkerSlot(instance_id, max_inflight or self.max_inflight)
            self._cv.notify_all()

    def remove_worker(self, instance_id: int) -> None:
        with self._cv:
            s = self._slots.pop(instance_id, None)
            if s is not None:
                s.detached = True

    def pick(self, num_tokens: int, num_provided_tokens: int = 0, timeout: float | None = None) -> Charge:
        net = self.net_new_tokens(num_tokens, num_provided_tokens)
        deadline = None if timeout is None else time.monotonic() + timeout
        with self._cv:
            while True:
                free = [s for s in self._slots.values() if s.inflight < s.max_inflight]
                if free:
                    s = min(free, key=lambda w: (w.load_net_new, w.inflight, w.instance_id))
                    s.inflight += 1
                    s.load_net_new += net
                    s.dispatched += 1
                    return Charge(self, s, net)
                rem = None if deadline is None else deadline - time.monotonic()
                if rem is not None and rem <= 0:
                    raise TimeoutError("no prefill worker has free capacity")
                self._cv.wait(rem)

    def targets(self) -> list[dict]:
        with self._cv:
            return [dict(vars(s)) | {"instance_id": str(s.instance_id)} for s in self._slots.values()]

    def pressure(self) -> float:
        with self._cv:
            n = max(1, len(self._slots))
            return sum(s.load_net_new for s in self._slots.values()) / n


class BreakerTier(enum.IntEnum):
    CALM = 0
    WARM = 1
    HOT = 2


@dataclass
class BreakerConfig:
    warm_enter: float = 32768.0   # net-new tokens per worker
    hot_enter: float = 131072.0
    warm_exit: float = 16384.0
    hot_exit: float = 65536.0
    interval_s: float = 0.25


class CircuitBreaker:
    def __init__(self, cfg: BreakerConfig | None = None):
        self.cfg = cfg or BreakerConfig()
        self.tier = BreakerTier.CALM
        self.epoch = 0

    def evaluate(self, pressure: float) -> BreakerTier:
        c, t = self.cfg, self.tier
        if t == BreakerTier.CALM and pressure >= c.warm_enter:
            t = BreakerTier.HOT if pressure >= c.hot_enter else BreakerTier.WARM
        elif t == BreakerTier.WARM:
            if pressure >= c.hot_enter:
                t = BreakerTier.HOT
            elif pressure < c.warm_exit:
                t = BreakerTier.CALM
        elif t == BreakerTier.HOT and pressure < c.hot_exit:
            t = BreakerTier.WARM if pressure >= c.warm_exit else BreakerTier.CALM
        if t != self.tier:
            self.tier = t
            self.epoch += 1
        return self.tier


class BreakerTicker:
    """Evaluates a breaker on a fixed interval from a selector's pressure."""

    def __init__(self, breaker: CircuitBreaker, selector: Selector, on_change=None):
        self.breaker, self.selector, self.on_change = breaker, selector, on_change
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True, name="kvbm-breaker")
        self._t.start()

    def _run(self):
        while not self._stop.wait(self.breaker.cfg.interval_s):
            before = self.breaker.epoch
            tier = self.breaker.evaluate(self.selector.pressure())
            if self.breaker.epoch != before and self.on_change:
                self.on_change(tier)

    def stop(self):
        self._stop.set()
        self._t.join(timeout=2)


@dataclass
class Calibration:
    ttft: list[tuple[float, float]] = field(default_factory=list)  # (isl tokens, seconds)
    itl: list[tuple[float, float]] = field(default_factory=list)   # (context tokens, seconds)

    def add_ttft(self, isl: int, seconds: float) -> None:
        self.ttft.append((float(isl), float(seconds)))

    def add_itl(self, ctx: int, seconds: float) -> None:
        self.itl.append((float(ctx), float(seconds)))

    def ttft_model(self) -> np.ndarray:
        """Coefficients (a, b, c) of ttft = a + b*isl + c*isl^2."""
        if len(self.ttft) < 3:
            raise ValueError("need >= 3 TTFT samples")
        x, y = np.array(self.ttft).T
        A = np.stack([np.ones_like(x), x, x * x], axis=1)
        return np.linalg.lstsq(A, y, rcond=None)[0]

    def itl_model(self) -> np.ndarray:
        if len(self.itl) < 2:
            raise ValueError("need >= 2 ITL samples")
        x, y = np.array(self.itl).T
        A = np.stack([np.ones_like(x), x], axis=1)
        return np.linalg.lstsq(A, y, rcond=None)[0]

    def predict_ttft(self, isl: int) -> float:
        a, b, c = self.ttft_model()
        return float(a + b * isl + c * isl * isl)

    def to_dict(self) -> dict:
        out = {"ttft_samples": len(self.ttft), "itl_samples": len(self.itl)}
        try:
            out["ttft_coeffs"] = [float(v) for v in self.ttft_model()]
        except ValueError:
            pass
        try:
            out["itl_coeffs"] = [float(v) for v in self.itl_model()]
        except ValueError:
            pass
        return out
