"""Tensor-parallel serving on CPU ranks (gloo): rank 0's batcher leads, rank 1 follows its scheduler commands
(runtime/lockstep.py). Every request's tokens must equal its tokens generated alone on the same tensor-parallel
engine, a refused request must be refused on both ranks without breaking the lockstep, idle beats must keep the
follower waiting, and stop must end the follower."""

import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, speculative, out, batch_prefill=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(1)
    try:
        from eagle4_b200.api import LLM, TreeSpec
        from eagle4_b200.parallel.tp import TensorParallel
        from eagle4_b200.runtime.lockstep import Lockstep, follow
        from eagle4_b200.runtime.scheduler import RequestParams
        from eagle4_b200.serve import Batcher

        tp = TensorParallel(backend="torch")
        llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_batch=2,
                            max_len=256, tp=tp)
        g = torch.Generator().manual_seed(3)
        prompts = [torch.randint(1, 4096, (int(torch.randint(5, 30, (1,), generator=g)),), generator=g)
                   for _ in range(4)]
        lens = [6, 3, 9, 4]
        alone = [llm.generate([p], n, speculative=False)[0].tolist() for p, n in zip(prompts, lens)]
        ls = Lockstep(timeout_s=30.0, beat_s=0.2)
        if rank == 0:
            b = Batcher(llm.engine, speculative=speculative, lockstep=ls, batch_prefill=batch_prefill)
            futs = [b.submit(p.tolist(), RequestParams(max_new_tokens=n)) for p, n in zip(prompts, lens)]
            bad = b.submit([1] * 300, RequestParams(max_new_tokens=4))
            got = [f.result(timeout=600).output for f in futs]
            try:
                bad.result(timeout=60)
                refused = False
            except ValueError:
                refused = True
            sent = ls.sent
            time.sleep(1.0)  # idle: beats only
            beats = ls.sent - sent
            b.close(timeout=60)
            out[rank] = {"got": got, "alone": alone, "refused": refused, "beats": beats,
                         "failed": b.failed is not None}
        else:
            rounds = follow(llm.engine, ls, speculative=speculative, batch_prefill=batch_prefill)
            out[rank] = {"rounds": rounds, "alone": alone}
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("speculative", [True, False])
def test_tensor_parallel_serving_in_lockstep(speculative):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(2, _port(), speculative, out), nprocs=2, start_method="spawn", join=True)
        res = dict(out)
    lead, follower = res[0], res[1]
    assert lead["got"] == lead["alone"] and lead["alone"] == follower["alone"]
    assert lead["refused"] and not lead["failed"]
    assert 2 <= lead["beats"] <= 10
    assert follower["rounds"] > 0


def test_tensor_parallel_serving_with_batched_prefill():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(2, _port(), True, out, True), nprocs=2, start_method="spawn", join=True)
        res = dict(out)
    assert res[0]["got"] == res[0]["alone"] and res[0]["refused"]
