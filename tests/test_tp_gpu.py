"""Tensor parallelism on 2 GPUs: the fused peer-memory collectives against the NCCL baseline and one GPU.

Runs as two spawned NCCL ranks (skipped with fewer than two GPUs). NVLS is off (``NCCL_NVLS_ENABLE=0``) and the
fused kernels use plain peer stores and loads, no multicast. Every wait in the fused kernels is bounded and the
process group has a short timeout, so a broken rank ends the test with an error instead of a hang.
"""

import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    res = {}
    try:
        from eagle4_b200.api import LLM, TreeSpec
        from eagle4_b200.models.target import RowBatch
        from eagle4_b200.ops import native
        from eagle4_b200.parallel.tp import TensorParallel

        dev = torch.device("cuda", rank)
        tree = TreeSpec(4, 2, 8)
        fused = TensorParallel(backend="fused", max_rows=256, max_cols=4096, device=dev)
        base = TensorParallel(backend="torch", device=dev)
        models = {"fused": LLM.synthetic("tiny", device=dev, tree=tree, max_len=512, tp=fused),
                  "nccl": LLM.synthetic("tiny", device=dev, tree=tree, max_len=512, tp=base),
                  "one": LLM.synthetic("tiny", device=dev, tree=tree, max_len=512)}
        g = torch.Generator().manual_seed(0)
        prompt = torch.randint(0, 4096, (200,), generator=g)
        hid = {}
        for name, m in models.items():
            eng = m.engine
            n = prompt.shape[0]
            pos = torch.arange(n, device=dev)
            slots = eng._slots(torch.tensor(0, device=dev), pos)
            z = torch.zeros(n, dtype=torch.int32, device=dev)
            rb = RowBatch(ids=prompt.to(dev), pos=pos, req=z, write_slot=slots, ctx_start=z, ctx_len=(pos + 1).int(),
                          extra=torch.zeros(n, 1, dtype=torch.int32, device=dev), n_extra=z, parent=(pos - 1).int(),
                          state_slot=z, scan=True)
            h, _ = m.target.forward(rb, eng.tcache)
            ids, _ = m.target.greedy(h)
            hid[name] = (h.float(), ids)
        res["fused_vs_nccl"] = (hid["fused"][0] - hid["nccl"][0]).abs().max().item()
        res["fused_vs_one"] = (hid["fused"][0] - hid["one"][0]).abs().max().item()
        res["scale"] = hid["one"][0].abs().max().item()
        res["tok_agree"] = (hid["fused"][1] == hid["nccl"][1]).float().mean().item()
        spec = models["fused"].generate(prompt[None], 24)
        plain = models["fused"].generate(prompt[None], 24, speculative=False)
        res["spec_eq_plain"] = bool(torch.equal(spec, plain))
        gathered = [None] * world
        dist.all_gather_object(gathered, spec.tolist())
        res["ranks_agree"] = all(x == gathered[0] for x in gathered)
        native.check_errors(dev)
        res["ok"] = True
        for m in models.values():
            m.engine.graphs.clear()
        torch.cuda.synchronize()
        fused.close()
    except Exception as e:  # noqa: BLE001 - reported to the parent
        res["error"] = repr(e)
    finally:
        out[rank] = res
        dist.destroy_process_group()


def test_fused_tp_matches_nccl_and_one_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(2, _port(), out), nprocs=2, start_method="spawn", join=True)
        res = dict(out)
    for r in range(2):
        assert res[r].get("ok"), res[r]
        assert res[r]["fused_vs_nccl"] <= 0.02 * res[r]["scale"], res[r]
        assert res[r]["fused_vs_one"] <= 0.05 * res[r]["scale"], res[r]
        assert res[r]["tok_agree"] >= 0.95 and res[r]["spec_eq_plain"] and res[r]["ranks_agree"], res[r]
