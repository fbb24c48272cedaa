"""Prefill-worker calibration on CPU: request resolution and clamps, the fitted
performance model on synthetic traces, and a hub-triggered sweep through a
PrefillRouterHandler whose calibrate lambda drives a fake streaming engine."""

import asyncio
import threading
from types import SimpleNamespace

import numpy as np
import pytest

from kvbm_b200.hub.calibration import (DEFAULT_SEED, CalibrationDefaults, CalibrationRequest, analyze,
                                       samples_from_traces)


def _defaults_32k():
    return CalibrationDefaults(model_id="m", max_seq_len=32768, max_input_len=32768, max_output_len=1024,
                               vocab_size=32000, safe_vocab_lo=1000)


def test_resolve_defaults_trims_the_ladder_to_the_soft_cap():
    r = CalibrationRequest().resolve(_defaults_32k())
    # cap = 0.8 * 32768 = 26214: 16384 + 64 fits, 32768 + 64 does not
    assert r.seq == [1024, 2048, 4096, 8192, 16384]
    assert (r.osl, r.seed, r.warmup) == (64, DEFAULT_SEED, True)
    assert r.body_vocab == (1000, 2000) and r.buster_vocab == (1000, 30000)
    assert any("32768 dropped" in c for c in r.clamps)


def test_resolve_clamps_and_errors():
    d = _defaults_32k()
    r = CalibrationRequest(seq=[1, 512, 1024, 2048, 40000, 4096], osl=4096, max_isl_fraction=2.0,
                           buster_vocab=(0, 99999)).resolve(d)
    assert r.osl == 1024 and r.max_isl_fraction == 0.95
    assert r.seq == [512, 1024, 2048, 4096]  # explicit lists obey only the hard caps
    assert r.buster_vocab == (1000, 32000)
    assert any(c.startswith("osl clamped") for c in r.clamps) and any("isl 1 dropped" in c for c in r.clamps)
    with pytest.raises(ValueError, match="needs >= 4"):
        CalibrationRequest(seq=[512, 1024, 1024]).resolve(d)
    with pytest.raises(ValueError, match="no calibration input length"):
        CalibrationRequest(seq=[40000]).resolve(d)
    small = CalibrationDefaults(max_seq_len=3000, max_input_len=3000, max_output_len=3000)
    with pytest.raises(ValueError):
        CalibrationRequest().resolve(small)  # only 1024 and 2048 fit under the soft cap


def _synthetic_traces(a=2000.0, b=0.05, c=2e-6, i0=6000.0, s=0.01, osl=32, seq=(1024, 2048, 4096, 8192)):
    out = []
    for isl in seq:
        ttft = a + b * isl + c * isl * isl
        itl = [i0 + s * (isl + 1 + k) for k in range(1, osl)]  # gap k lands at position isl + 1 + k
        out.append({"isl": isl, "osl": osl, "ttft_us": int(round(ttft)), "itl_us": [int(round(v)) for v in itl],
                    "first_token": 1000 + isl})
    return out


def test_analyze_recovers_the_model():
    tr = _synthetic_traces()
    res = analyze(tr)
    pm = res["performance_model"]
    assert pm["t2ft_quadratic"] == pytest.approx(2e-6, rel=1e-2)
    assert pm["t2ft_linear"] == pytest.approx(0.05, abs=5e-3)
    assert pm["t2tl_intercept"] == pytest.approx(6000.0, rel=1e-3)
    assert pm["t2tl_slope"] == pytest.approx(0.01, rel=0.1)
    assert pm["t2ft_fit_r2"] > 0.999
    # n_opt solves b + 2cN = ITL intercept; n_att = intercept / slope
    assert res["n_opt"] == pytest.approx((6000.0 - 0.05) / (2 * 2e-6), rel=0.02)
    assert res["n_att"] == pytest.approx(6000.0 / 0.01, rel=0.1)
    assert len(res["t2tl_scatter_data"]["x"]) == 4 * (32 - 1 - 2)  # first and last gap of each trace dropped
    ttft, itl = samples_from_traces(tr)
    assert ttft[0] == (1024, pytest.approx(tr[0]["ttft_us"] * 1e-6))
    with pytest.raises(ValueError, match="4 distinct"):
        analyze(tr[:3])


def test_hub_triggers_a_sweep_through_the_prefill_worker(capsys):
    from kvbm_b200.hub.calibrate_lambda import capture_calibration_defaults, make_calibrate_lambda
    from kvbm_b200.hub.client import HubClient, PrefillRouterHandler
    from kvbm_b200.hub.server import HubServer
    from kvbm_b200.runtime.messenger import wait_until

    seen = []

    class FakeEngine:
        """Streams osl outputs; time to first output grows with the prompt, later gaps are fixed."""

        model_config = SimpleNamespace(max_model_len=9000, hf_config=SimpleNamespace(vocab_size=4096))

        async def generate(self, prompt, params, request_id):
            ids, osl = prompt
            seen.append(ids)
            await asyncio.sleep(1e-3 + 2e-7 * len(ids))
            for _ in range(osl):
                yield SimpleNamespace()
                await asyncio.sleep(5e-4)

    loop = asyncio.new_event_loop()
    t = threading.Thread(target=loop.run_forever, daemon=True)
    t.start()
    hub = HubServer(max_seq_len=4096, ttl=5.0).start()
    eng = FakeEngine()
    defaults = capture_calibration_defaults(eng, "fake")
    assert defaults["max_seq_len"] == 9000 and defaults["vocab_size"] == 4096
    gate = threading.Event()

    def dispatch(req, done):
        gate.wait(5.0)
        done.complete({"ok": True})

    handler = PrefillRouterHandler(hub.url, dispatch, calibrate_lambda=make_calibrate_lambda(
        eng, loop, make_request=lambda ids, osl: ((ids, osl), None)), calibration_defaults=defaults)
    client = HubClient(hub.url)
    try:
        assert wait_until(lambda: len(client.targets()) == 1, 5.0)
        req = {"seq": [256, 512, 1024, 2048], "osl": 6, "warmup": False}
        out = client.run_calibration(handler.instance_id, req, timeout=60)
        assert not out["from_cache"] and out["resolved"]["seq"] == [256, 512, 1024, 2048]
        assert [len(ids) for ids in seen] == [256, 512, 1024, 2048]
        firsts = [ids[0] for ids in seen]
        assert len(set(firsts)) == 4 and all(1000 <= f < 4096 for f in firsts)  # cache busters, all distinct
        assert all(1000 <= v < 2000 for ids in seen for v in ids[1:])           # body vocabulary
        pm = out["results"]["performance_model"]
        assert all(np.isfinite(v) for v in pm.values())  # wall-clock sleeps: only the shape is checked
        # the hub fed its router's TTFT model for this instance
        cal = client.router_counters()["calibration"][str(handler.instance_id)]
        assert cal["ttft_samples"] == 4 and "ttft_coeffs" in cal
        # a second ask is served from the worker's cache unless forced (here through kvbmctl)
        assert client.run_calibration(handler.instance_id, req, timeout=60)["from_cache"]
        import json

        from kvbm_b200.hub.kvbmctl import main as kvbmctl

        assert kvbmctl(["--hub", hub.url, "--json", "calibrate", "--instance-id", str(handler.instance_id),
                        "--seq", "256,512,1024,2048", "--osl", "6"]) == 0
        assert json.loads(capsys.readouterr().out)["from_cache"]
        assert kvbmctl(["--hub", hub.url, "calibrate", "--instance-id", str(handler.instance_id)]) == 0
        assert "TTFT(us)" in capsys.readouterr().out
        # while a prefill is in flight the worker refuses to calibrate (409 from the hub)
        th = threading.Thread(target=lambda: handler._on_dispatch({"payload": ""}), daemon=True)
        th.start()
        assert wait_until(lambda: handler.inflight == 1, 5.0)
        with pytest.raises(RuntimeError, match="409"):
            client.run_calibration(handler.instance_id, req, force=True, timeout=60)
        gate.set()
        th.join(5.0)
        # and a dispatch during a sweep is refused
        handler.calibrating = True
        with pytest.raises(RuntimeError, match="calibration_in_progress"):
            handler._on_dispatch({"payload": ""})
        handler.calibrating = False
    finally:
        handler.close()
        loop.call_soon_threadsafe(loop.stop)
        hub.stop()
