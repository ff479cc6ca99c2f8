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
