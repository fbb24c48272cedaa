"""CPU tests: audit-trace diff, pub/sub transports, shutdown cleanup of shared cache files."""

import json
import os
import signal
import subprocess
import sys
import textwrap
import time

import pytest

from kvbm_b200.engine.pubsub import PubSubEventSink, StubPubSub, ZmqPubSub, make_pubsub
from kvbm_b200.utils import audit_diff, disk_cleanup


def _log(path, events):
    with open(path, "w") as f:
        f.write("2026-01-01 INFO kvbm_audit not-json line\n")
        for e in events:
            f.write("2026-01-01 12:00:00 INFO kvbm_audit " + json.dumps(e) + "\n")


def test_audit_diff_sequences_multiset_and_normalize(tmp_path):
    a, b = tmp_path / "a.log", tmp_path / "b.log"
    _log(a, [{"event": "gnmt_pending", "request": "x1"}, {"event": "gnmt_matched", "request": "x1"},
             {"event": "transfer_session_opened", "session": "s"}])
    _log(b, [{"event": "gnmt_pending", "request": "y9"}, {"event": "gnmt_matched", "request": "y9"}])
    assert audit_diff.main([str(a), str(b)]) == 1
    assert audit_diff.main([str(a), str(b), "--normalize-request-ids", "--filter-prefixes", "transfer_"]) == 0
    _log(b, [{"event": "gnmt_matched", "request": "y9"}, {"event": "gnmt_pending", "request": "y9"}])
    args = [str(a), str(b), "--normalize-request-ids", "--filter-prefixes", "transfer_"]
    assert audit_diff.main(args) == 1 and audit_diff.main(args + ["--multiset"]) == 0
    # key=value records after a kvbm_audit: tag
    rec = audit_diff.parse_line('ts kvbm_audit: event="onboard_complete" request_id=r1 ok=true')
    assert rec == {"event": "onboard_complete", "request_id": "r1", "ok": "true"}
    assert audit_diff.main([str(a), str(tmp_path / "missing.log")]) == 2


def test_pubsub_stub_and_zmq_and_event_sink():
    s = StubPubSub()
    got = []
    s.subscribe("kvbm.events", lambda subj, p: got.append((subj, PubSubEventSink.decode(p))))
    PubSubEventSink(s)(7, [("create", [1, 2 << 100])])
    assert got == [("kvbm.events.7", (7, [("create", [1, 2 << 100])]))]

    a, b = ZmqPubSub(), make_pubsub("tcp://127.0.0.1:0")
    seen = []
    b.subscribe("kv.", lambda subj, p: seen.append((subj, p)))
    b.connect(a.endpoint)
    deadline = time.time() + 5
    while not seen and time.time() < deadline:  # PUB/SUB joins asynchronously
        a.publish("kv.x", b"hello")
        a.publish("other", b"nope")
        time.sleep(0.05)
    assert seen and all(x == ("kv.x", b"hello") for x in seen)
    a.close()
    b.close()


def test_disk_cleanup_unlinks_on_sigterm(tmp_path):
    f = tmp_path / "g2.shm"
    code = textwrap.dedent(f"""
        import os, sys, time
        sys.path.insert(0, {os.getcwd()!r})
        from kvbm_b200.utils import disk_cleanup
        open({str(f)!r}, "w").write("x")
        disk_cleanup.register({str(f)!r})
        print("ready", flush=True)
        time.sleep(30)
    """)
    p = subprocess.Popen([sys.executable, "-c", code], stdout=subprocess.PIPE, text=True)
    assert p.stdout.readline().strip() == "ready" and f.exists()
    p.send_signal(signal.SIGTERM)
    assert p.wait(10) == 128 + signal.SIGTERM
    assert not f.exists()
    g = tmp_path / "keep"
    g.write_text("y")
    disk_cleanup.register(str(g))
    disk_cleanup.deregister(str(g))
    assert str(g) not in disk_cleanup.registered() and g.exists()


def test_every_source_file_compiles():
    """Every Python file of the package, the import-alias package and the bench entry point is valid
    Python (a syntax error in a rarely imported module, e.g. a bench, would otherwise go unnoticed)."""
    import pathlib

    root = pathlib.Path(__file__).resolve().parents[1]
    files = sorted(list((root / "kvbm_b200").rglob("*.py")) + list((root / "kvbm").rglob("*.py"))
                   + [root / "bench.py", root / "__graft_entry__.py"])
    assert len(files) > 50
    for f in files:
        compile(f.read_text(), str(f), "exec")


def test_bench_entry_points_parse_their_arguments(monkeypatch, capsys):
    """Every bench module imports and answers --help on a machine without a GPU."""
    import pathlib
    import runpy
    import sys

    root = pathlib.Path(__file__).resolve().parents[1]
    mods = sorted(p.stem for p in (root / "kvbm_b200" / "bench").glob("*.py") if p.stem != "__init__")
    assert "connector_bench" in mods and "kvbench" in mods
    for m in mods:
        monkeypatch.setattr(sys, "argv", [m, "--help"])
        with pytest.raises(SystemExit) as e:
            runpy.run_module(f"kvbm_b200.bench.{m}", run_name="__main__")
        assert e.value.code in (0, None), m
        assert "usage" in capsys.readouterr().out, m


def test_kernels_api_validates_arguments_without_a_gpu():
    """``kvbm.kernels`` rejects bad layouts, backends and mismatched groups before touching a GPU."""
    import torch

    from kvbm import kernels

    with pytest.raises(ValueError, match="layout"):
        kernels.block_to_universal([[torch.zeros(1)]], [torch.zeros(1)], "XYZ")
    with pytest.raises(ValueError, match="groups"):
        kernels.block_to_universal([[torch.zeros(1)], [torch.zeros(1)]], [torch.zeros(1)], "NHD")
    with pytest.raises(ValueError, match="backend"):
        kernels.block_to_operational([[torch.zeros(1)]], [torch.zeros(1)], backend="dma")
    with pytest.raises(ValueError, match="CUDA"):
        kernels.block_to_operational([[torch.zeros(4)]], [torch.zeros(4)])
    with pytest.raises(TypeError):
        kernels.block_to_universal(torch.zeros(3), [torch.zeros(1)])
