"""Tensor parallelism on CPU: gloo ranks run the sharded model through the ``torch`` collective backend.

Checks that TP=2 (and a mixed TP=4 on a widened tiny model) reproduces the single-process forward, that every rank
holds the same greedy tokens, and that speculative output equals plain decode under TP.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from eagle4_b200.models import configs
from eagle4_b200.parallel import sharding


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(1)
    try:
        from eagle4_b200.api import LLM, TreeSpec
        from eagle4_b200.models.target import RowBatch
        from eagle4_b200.parallel.tp import TensorParallel

        tp = TensorParallel(backend="torch")
        llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_len=256, tp=tp)
        ref = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_len=256)
        g = torch.Generator().manual_seed(0)
        prompt = torch.randint(0, 4096, (24,), generator=g)
        outs = {}
        for name, m in (("tp", llm), ("ref", ref)):
            eng = m.engine
            n = prompt.shape[0]
            eng.pages.reserve(0, n + 1)  # map real KV pages (an unmapped row writes every position to the trash page)
            pos = torch.arange(n)
            slots = eng._slots(torch.tensor(0), pos)
            rb = RowBatch(ids=prompt, pos=pos, req=torch.zeros(n, dtype=torch.int32), write_slot=slots,
                          ctx_start=torch.zeros(n, dtype=torch.int32), ctx_len=(pos + 1).int(),
                          extra=torch.zeros(n, 1, dtype=torch.int32), n_extra=torch.zeros(n, dtype=torch.int32),
                          parent=(pos - 1).int(), state_slot=torch.zeros(n, dtype=torch.int32), scan=True)
            h, _ = m.target.forward(rb, eng.tcache)
            outs[name] = (h, m.target.greedy(h)[0])
        err = (outs["tp"][0] - outs["ref"][0]).abs().max().item()
        same_tokens = bool(torch.equal(outs["tp"][1], outs["ref"][1]))
        spec = llm.generate(prompt[None], 12)
        plain = llm.generate(prompt[None], 12, speculative=False)
        gathered = [None] * world
        dist.all_gather_object(gathered, spec.tolist())
        out[rank] = {"err": err, "same_tokens": same_tokens, "spec_eq_plain": bool(torch.equal(spec, plain)),
                     "ranks_agree": all(x == gathered[0] for x in gathered)}
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_tp_matches_single_process(world):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(world, _port(), out), nprocs=world, start_method="spawn", join=True)
        res = dict(out)
    for r in range(world):
        assert res[r]["err"] < 1e-4, res[r]
        assert res[r]["same_tokens"] and res[r]["spec_eq_plain"] and res[r]["ranks_agree"], res[r]


def _sampled_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(1)
    try:
        from eagle4_b200.api import LLM, TreeSpec
        from eagle4_b200.parallel.tp import TensorParallel

        tp = TensorParallel(backend="torch")
        kw = dict(device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_len=256, temperature=0.9,
                  sample_seed=11, max_batch=2)
        llm = LLM.synthetic("tiny", tp=tp, **kw)
        ref = LLM.synthetic("tiny", **kw)
        g = torch.Generator().manual_seed(3)
        prompts = [torch.randint(0, 4096, (20,), generator=g), torch.randint(0, 4096, (33,), generator=g)]
        got = llm.generate(prompts, 10).tolist()
        want = ref.generate(prompts, 10).tolist()
        gathered = [None] * world
        dist.all_gather_object(gathered, got)
        out[rank] = {"equal": got == want, "ranks_agree": all(x == gathered[0] for x in gathered), "got": got,
                     "want": want}
    finally:
        dist.destroy_process_group()


def test_vocab_parallel_sampling_equals_one_process():
    """Sampled speculative decoding at TP2 (the accept exchanges row statistics, candidate probabilities and residual
    masses instead of the full logits) gives the single-process sampled tokens for the same seed."""
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_sampled_worker, args=(2, _port(), out), nprocs=2, start_method="spawn", join=True)
        res = dict(out)
    for r in range(2):
        assert res[r]["ranks_agree"], res[r]
        assert res[r]["equal"], (res[r]["got"], res[r]["want"])


def test_shard_layouts_cover_the_weights():
    from eagle4_b200.models import weights

    cfg = configs.tiny_hybrid()
    w = weights.init_target(cfg, seed=0)
    parts = [sharding.shard_target(cfg, w, 2, r) for r in range(2)]
    # column-parallel shards partition the rows; row-parallel shards the columns
    for key in ("l0.in_proj", "l3.qkv", "l0.gate_up"):
        rows = sum(p[1][key].shape[0] for p in parts)
        assert rows == w[key].shape[0] or key == "l3.qkv"
    for key in ("l0.out_proj", "l3.o_proj", "l0.down"):
        torch.testing.assert_close(torch.cat([p[1][key] for p in parts], dim=1), w[key])
    lo0, hi0 = sharding.vocab_range(248320, 8, 0)
    lo7, hi7 = sharding.vocab_range(248320, 8, 7)
    assert lo0 == 0 and hi0 % 128 == 0 and hi7 == 248320 and (hi7 - lo7) % 128 == 0
    assert sharding.kv_layout(24, 4, 8, 5) == (1, 2)
    q = configs.qwen38_27b()
    loc = sharding.local_target_config(q, 8, 0)
    assert (loc.num_heads, loc.num_kv_heads, loc.gdn_k_heads, loc.gdn_v_heads) == (3, 1, 2, 6)
    with pytest.raises(ValueError):
        sharding.local_target_config(q, 3, 0)


def _mamba_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(1)
    try:
        from eagle4_b200.api import LLM, TreeSpec
        from eagle4_b200.parallel.tp import TensorParallel

        kw = dict(device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_len=256, max_batch=2)
        llm = LLM.synthetic("tiny-mamba", tp=TensorParallel(backend="torch"), **kw)
        ref = LLM.synthetic("tiny-mamba", **kw)
        g = torch.Generator().manual_seed(5)
        prompts = [torch.randint(0, 4096, (18,), generator=g), torch.randint(0, 4096, (27,), generator=g)]
        spec = llm.generate(prompts, 10).tolist()
        plain = llm.generate(prompts, 10, speculative=False).tolist()
        out[rank] = {"spec": spec, "plain": plain, "one": ref.generate(prompts, 10, speculative=False).tolist()}
    finally:
        dist.destroy_process_group()


def test_mamba_hybrid_under_tensor_parallelism():
    """A Nemotron-H-style Mamba2 hybrid at TP2 (heads, groups and their norm weights sharded): speculative == plain,
    and both equal the single-process greedy tokens."""
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_mamba_worker, args=(2, _port(), out), nprocs=2, start_method="spawn", join=True)
        res = dict(out)
    for r in range(2):
        assert res[r]["spec"] == res[r]["plain"] == res[r]["one"]
