"""Prefill-worker calibration: what a sweep runs, and the performance model fitted to it.

A calibration sweep sends single-stream requests of increasing input length
(ISL) to one prefill engine and records each request's time to first token
and its inter-token latencies. From those traces:

* TTFT(ISL) is fitted as ``a + b*ISL + c*ISL^2`` (prefill attention is
  quadratic in the prompt length), in microseconds;
* ITL(position) is fitted as ``i + s*position`` (a decode step grows with
  the tokens in the KV cache), dropping each trace's first and last
  inter-token gap (prefill tail, shutdown);
* ``n_opt``, the prompt length where one more prompt token costs as much
  prefill time as one decode step (``b + 2*c*N = i``; ``i / b`` when the
  fit is linear), and ``n_att = i / s``, the context length at which the
  attention share of a decode step equals its fixed part.

:class:`CalibrationRequest` holds the caller's optional knobs;
:meth:`CalibrationRequest.resolve` fills them from the engine's
:class:`CalibrationDefaults` and clamps what the engine cannot run,
recording every clamp. The fits are ordinary least squares (numpy) with
the coefficient of determination reported beside each.

Parity: crates/kvbm-hub/src/features/prefill_router/calibration.rs
(CalibrationRequest / CalibrationDefaults / resolve / analyze; the default
knob values and the ``n_opt`` / ``n_att`` definitions are the reference's
documented ones so both hubs give comparable answers).
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, field

import numpy as np

CALIBRATE_HANDLER = "kvbm.prefill_router.calibrate"

DEFAULT_BODY_VOCAB = (1000, 2000)      # body tokens: a narrow id range
DEFAULT_BUSTER_VOCAB = (1000, 30000)   # first token of every request: unique per request (no cache hits)
DEFAULT_SEQ_LADDER = (1024, 2048, 4096, 8192, 16384, 32768, 65536, 131072)
DEFAULT_OSL = 64
DEFAULT_SEED = 0xC0FFEE
DEFAULT_MAX_ISL_FRACTION = 0.80


@dataclass
class CalibrationDefaults:
    """What the engine can run, captured from the live engine (see ``calibrate_lambda``)."""

    model_id: str = ""
    max_seq_len: int = 8192
    max_input_len: int = 8192
    max_output_len: int = 8192
    vocab_size: int = 32000
    safe_vocab_lo: int = 1000   # first id past special / added tokens

    @classmethod
    def from_dict(cls, d: dict | None) -> "CalibrationDefaults":
        if not d:
            return cls()
        return cls(**{k: d[k] for k in cls.__dataclass_fields__ if k in d})


@dataclass
class ResolvedCalibration:
    seq: list[int]
    osl: int
    seed: int
    max_isl_fraction: float
    warmup: bool
    body_vocab: tuple[int, int]
    buster_vocab: tuple[int, int]
    clamps: list[str] = field(default_factory=list)

    def to_dict(self) -> dict:
        d = asdict(self)
        d["body_vocab"], d["buster_vocab"] = list(self.body_vocab), list(self.buster_vocab)
        return d


def _clamp_vocab(label: str, rng, defaults: CalibrationDefaults, clamps: list[str]) -> tuple[int, int]:
    lo_raw, hi_raw = int(rng[0]), int(rng[1])
    safe_lo, safe_hi = int(defaults.safe_vocab_lo), int(defaults.vocab_size)
    if safe_hi <= safe_lo:
        raise ValueError(f"{label}: engine vocabulary is empty above id {safe_lo} (vocab_size {safe_hi})")
    lo = min(max(lo_raw, safe_lo), safe_hi - 1)
    hi = min(max(hi_raw, lo + 1), safe_hi)
    if (lo, hi) != (lo_raw, hi_raw):
        clamps.append(f"{label} clamped ({lo_raw}, {hi_raw}) -> ({lo}, {hi}) (vocab [{safe_lo}, {safe_hi}))")
    return lo, hi


@dataclass
class CalibrationRequest:
    """Caller knobs; None means the engine-derived default."""

    force: bool = False
    seq: list[int] | None = None
    osl: int | None = None
    seed: int | None = None
    max_isl_fraction: float | None = None
    warmup: bool | None = None
    body_vocab: tuple[int, int] | None = None
    buster_vocab: tuple[int, int] | None = None

    @classmethod
    def from_dict(cls, d: dict | None) -> "CalibrationRequest":
        d = dict(d or {})
        return cls(**{k: d[k] for k in cls.__dataclass_fields__ if k in d and d[k] is not None})

    def resolve(self, defaults: CalibrationDefaults) -> ResolvedCalibration:
        clamps: list[str] = []
        osl_raw = max(1, int(self.osl if self.osl is not None else DEFAULT_OSL))
        osl = min(osl_raw, max(1, int(defaults.max_output_len)))
        if osl != osl_raw:
            clamps.append(f"osl clamped {osl_raw} -> {osl} (max_output_len)")
        frac_raw = float(self.max_isl_fraction if self.max_isl_fraction is not None else DEFAULT_MAX_ISL_FRACTION)
        frac = min(max(frac_raw, 0.10), 0.95)
        if abs(frac - frac_raw) > 1e-12:
            clamps.append(f"max_isl_fraction clamped {frac_raw:.3f} -> {frac:.3f} (allowed range [0.10, 0.95])")
        cap = int(defaults.max_seq_len * frac)
        user = self.seq is not None
        seq: list[int] = []
        for isl in (self.seq if user else DEFAULT_SEQ_LADDER):
            isl = int(isl)
            if isl < 2:
                clamps.append(f"isl {isl} dropped (must be >= 2)")
            elif isl > defaults.max_input_len:
                clamps.append(f"isl {isl} dropped (exceeds max_input_len {defaults.max_input_len})")
            elif isl + osl > defaults.max_seq_len:
                clamps.append(f"isl {isl} dropped (isl+osl {isl + osl} > max_seq_len {defaults.max_seq_len})")
            elif not user and isl + osl > cap:
                # the soft cap only trims the default ladder; an explicit list obeys the hard caps alone
                clamps.append(f"isl {isl} dropped (isl+osl {isl + osl} > max_isl_fraction cap {cap})")
            else:
                seq.append(isl)
        if not seq:
            raise ValueError(f"no calibration input length fits (max_seq_len={defaults.max_seq_len}, "
                             f"max_input_len={defaults.max_input_len}, osl={osl})")
        if len(set(seq)) < 4:
            raise ValueError(f"{len(set(seq))} distinct input length(s) left; the quadratic TTFT fit needs >= 4 "
                             f"(widen seq or raise max_isl_fraction, now {frac:.2f}, max_seq_len="
                             f"{defaults.max_seq_len})")
        return ResolvedCalibration(
            seq=seq, osl=osl, seed=int(self.seed if self.seed is not None else DEFAULT_SEED), max_isl_fraction=frac,
            warmup=True if self.warmup is None else bool(self.warmup),
            body_vocab=_clamp_vocab("body_vocab", self.body_vocab or DEFAULT_BODY_VOCAB, defaults, clamps),
            buster_vocab=_clamp_vocab("buster_vocab", self.buster_vocab or DEFAULT_BUSTER_VOCAB, defaults, clamps),
            clamps=clamps)


def _lstsq(cols: list[np.ndarray], y: np.ndarray) -> tuple[np.ndarray, float]:
    """Least-squares coefficients of y on [1, *cols] and the fit's R^2."""
    A = np.stack([np.ones_like(y)] + cols, axis=1)
    coef, *_ = np.linalg.lstsq(A, y, rcond=None)
    resid = y - A @ coef
    ss_tot = float(((y - y.mean()) ** 2).sum())
    r2 = 1.0 - float((resid ** 2).sum()) / ss_tot if ss_tot > 0 else 1.0
    return coef, r2


def _nonneg_int(v: float) -> int:
    if not np.isfinite(v) or v <= 0:
        return 0
    return int(min(v, 2 ** 32 - 1))


def analyze(traces: list[dict]) -> dict:
    """Fit the performance model to sweep traces (each: isl, osl, ttft_us, itl_us, first_token)."""
    if not traces:
        raise ValueError("no traces to analyze")
    x = np.array([float(t["isl"]) for t in traces])
    y = np.array([float(t["ttft_us"]) for t in traces])
    if len(np.unique(x)) < 4:
        raise ValueError(f"need at least 4 distinct input lengths for the quadratic TTFT fit; got "
                         f"{len(np.unique(x))}")
    (a, b, c), r2_ttft = _lstsq([x, x * x], y)
    px: list[float] = []
    py: list[float] = []
    for t in traces:
        itl = list(t.get("itl_us") or [])
        if len(itl) <= 2:
            continue
        pos = float(t["isl"]) + 1.0
        for lat in itl[1:-1]:
            pos += 1.0
            px.append(pos)
            py.append(float(lat))
    if not px:
        raise ValueError("no inter-token latencies to fit (every trace had <= 2 after dropping the ends)")
    (i0, s), r2_itl = _lstsq([np.array(px)], np.array(py))
    if abs(c) > 1e-12:
        n_opt = _nonneg_int((i0 - b) / (2.0 * c))
    elif abs(b) > 1e-12:
        n_opt = _nonneg_int(i0 / b)
    else:
        n_opt = 0
    n_att = _nonneg_int(i0 / s) if s != 0 else 0
    return {
        "performance_model": {"t2ft_intercept": float(a), "t2ft_linear": float(b), "t2ft_quadratic": float(c),
                              "t2tl_intercept": float(i0), "t2tl_slope": float(s), "t2ft_fit_r2": float(r2_ttft),
                              "t2tl_fit_r2": float(r2_itl)},
        "n_opt": n_opt, "n_att": n_att, "traces": list(traces),
        "t2ft_scatter_data": {"x": x.tolist(), "y": y.tolist()},
        "t2tl_scatter_data": {"x": px, "y": py},
    }


def samples_from_traces(traces: list[dict]) -> tuple[list[tuple[int, float]], list[tuple[int, float]]]:
    """(isl, ttft seconds) and (context tokens, itl seconds) samples for the router's TTFT/ITL models."""
    ttft = [(int(t["isl"]), float(t["ttft_us"]) * 1e-6) for t in traces]
    itl = []
    for t in traces:
        lat = list(t.get("itl_us") or [])
        for k, v in enumerate(lat[1:-1], start=2):
            itl.append((int(t["isl"]) + k, float(v) * 1e-6))
    return ttft, itl
