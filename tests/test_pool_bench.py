"""Config-1 plumbing: the native pool's hit rate and KV-event log equal an
independent pure-Python model of the same semantics (CPU)."""

from kvbm_b200.bench.pool_bench import PyLruPool, make_workload, run_native


def test_event_log_and_hit_rate_match_python_model():
    wl = make_workload(96, seed=3)
    nat = run_native(wl, 2048, "lru")
    model = PyLruPool(2048)
    hits = sum(max(0, model.process(h)) for h in wl)
    assert abs(nat["hit_rate"] - hits / sum(len(h) for h in wl)) < 1e-12
    assert model.events == [(k, h) for k, h in nat["events"]]
    assert any(k == "remove" for k, _ in nat["events"])  # the pool was under eviction pressure
    assert nat["hit_rate"] > 0.05  # shared prefixes were reused


def test_lineage_backend_runs_the_same_workload():
    wl = make_workload(64, seed=4)
    nat = run_native(wl, 2048, "lineage")
    assert 0.0 < nat["hit_rate"] < 1.0
