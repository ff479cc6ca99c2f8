"""Failure detection on the host: gloo ranks where one rank stops, and corrupted persistent state.

No GPU is faulted, trapped or hung: a "crashed" rank is a process that stops beating (and exits); the survivors
detect it between rounds through the store, within the timeout.
"""

import datetime
import json
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    from eagle4_b200.parallel.health import Heartbeat, PeerFailure

    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=20))
    hb = Heartbeat(store, rank, world)
    res = {"detected": None}
    try:
        for step in range(1, 6):
            if rank == 1 and step == 3:
                res["stopped_at"] = step
                return  # the "crash": this rank never beats again
            hb.beat(step)
            hb.check(step, timeout=2.0)
    except PeerFailure as e:
        res["detected"] = (e.ranks, e.step)
    finally:
        out[rank] = res
        if rank == 0:
            import time
            time.sleep(0.5)


def test_heartbeat_detects_stopped_rank():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(3, _port(), out), nprocs=3, start_method="spawn", join=True)
        res = dict(out)
    assert res[1].get("stopped_at") == 3
    for r in (0, 2):
        assert res[r]["detected"] == ([1], 3), res[r]


def test_corrupt_live_cost_cache_is_remeasured(tmp_path):
    from eagle4_b200.core.live_costs import CostKey, LiveCosts

    key = CostKey("NVIDIA B200", 1, "m", "d", "eagle4_b200", "bfloat16")
    path = os.path.join(tmp_path, f"{key.digest}.json")
    with open(path, "w") as f:
        f.write("{not json")
    live = LiveCosts(lambda b: [1, 8], key=key, draft_shape=(4, 12))
    assert live.load(path) is False  # refused, costs are measured again
    with open(path, "w") as f:
        json.dump({"version": -1}, f)
    assert live.load(path) is False


def test_cost_tables_of_another_setup_are_refused(tmp_path):
    from eagle4_b200.core.live_costs import CostKey, check_key, write_key

    write_key(str(tmp_path), CostKey("NVIDIA H100", 1, "m", "d", "eagle4_b200", "bfloat16"))
    with pytest.raises(ValueError):
        check_key(str(tmp_path), CostKey("NVIDIA B200", 1, "m", "d", "eagle4_b200", "bfloat16"))


def test_unsupported_gpu_is_refused(monkeypatch):
    import torch

    from eagle4_b200.utils import arch

    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(torch.cuda, "current_device", lambda: 0)
    monkeypatch.setattr(torch.cuda, "get_device_capability", lambda d=None: (9, 0))
    monkeypatch.setattr(torch.cuda, "get_device_name", lambda d=None: "NVIDIA H100")
    with pytest.raises(arch.UnsupportedDevice, match="sm_90"):
        arch.require_sm100()
    monkeypatch.setattr(torch.cuda, "get_device_capability", lambda d=None: (10, 0))
    arch.require_sm100()


def test_engine_beats_and_stops_on_a_late_peer():
    """The serving loop beats and checks its heartbeat every ``heartbeat_every`` rounds, before the round's
    collectives, and a late peer ends generation with PeerFailure naming it."""
    import torch

    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.parallel.health import PeerFailure

    class FakeHeartbeat:
        def __init__(self, fail_at=None):
            self.beats, self.checks, self.fail_at = [], [], fail_at

        def beat(self, step):
            self.beats.append(step)

        def check(self, step, timeout):
            self.checks.append(step)
            if self.fail_at is not None and step >= self.fail_at:
                raise PeerFailure([1], step)

    llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_len=256)
    eng = llm.engine
    eng.heartbeat, eng.heartbeat_every = FakeHeartbeat(), 4
    p = torch.randint(0, 4096, (1, 16), generator=torch.Generator().manual_seed(0))
    llm.generate(p, 20, speculative=False)
    assert eng.heartbeat.beats == eng.heartbeat.checks == list(range(1, len(eng.heartbeat.beats) + 1))
    assert len(eng.heartbeat.beats) >= 4
    eng.heartbeat = FakeHeartbeat(fail_at=eng._rounds_served // 4 + 2)
    try:
        llm.generate(p, 40, speculative=False)
        raise AssertionError("a late peer must stop the loop")
    except PeerFailure as e:
        assert e.ranks == [1]


def test_batches_above_the_verify_limit_decode_natively():
    import torch

    from eagle4_b200.api import LLM, TreeSpec

    llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_len=256, max_batch=2,
                        config='{"mode": "static", "max_verify_batch_size": 1}')
    p = torch.randint(0, 4096, (2, 16), generator=torch.Generator().manual_seed(1))
    rec = []
    llm.engine.recorder = type("R", (), {"record": lambda self, **kw: rec.append(kw["kind"])})()
    out = llm.generate(p, 12)
    assert set(rec) == {"native"}
    assert torch.equal(out, llm.generate(p, 12, speculative=False))
    rec.clear()
    llm.generate(p[:1], 12)  # one request is within the limit: it speculates
    assert "tree" in rec
