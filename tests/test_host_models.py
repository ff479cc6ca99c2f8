"""The host-facing draft model classes and the candidate-logits path (CPU).

* ``DraftModel.forward_rows`` with a host's attention equals the engine's own forward over its paged draft KV;
* vLLM's ``LlamaForCausalLMEagle4``: config checks over vLLM's extra keys, row forwards, candidates, full rows;
* the candidate-logits processor: shard candidates (padding rows never chosen, global ids), the merge over ranks
  (checked in float64 against its definition, and over a real two-rank gloo group), the ``-inf``-filled row whose
  softmax is the candidates' softmax, and SGLang's ``LogitsProcessor`` built on a stand-in SGLang module;
* TokenSpeed's ``LlamaForCausalLMEagle4``: the exit's sampled rows and the candidate top-k, one rank and two
  vocabulary-sharded ranks.
"""

import dataclasses
import os
import socket
import sys
import types

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from eagle4_b200.models import configs, weights
from eagle4_b200.models.draft import DraftCache, DraftModel
from eagle4_b200.plugins import candidate_logits as cl

V = 4096


def _draft(seed=3, **kw):
    tc = configs.tiny_hybrid()
    dc = dataclasses.replace(configs.tiny_draft(tc, draft_vocab=V), **kw)
    return dc, weights.init_draft(dc, seed=seed)


def _causal(q, k, v):
    """Each row attends to rows 0..itself (GQA), float64 softmax."""
    t, hq, d = q.shape
    grp = hq // k.shape[1]
    s = torch.einsum("thd,shd->ths", q.double(), k.double().repeat_interleave(grp, 1)) * d ** -0.5
    s = s.masked_fill(torch.ones(t, t, dtype=torch.bool).triu(1)[:, None, :], float("-inf"))
    return torch.einsum("ths,shd->thd", torch.softmax(s, -1), v.double().repeat_interleave(grp, 1)).to(q.dtype)


def _rows(dc, t=7, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randint(0, V, (t,), generator=g), torch.arange(5, 5 + t),
            torch.randn(t, dc.hidden_size, generator=g))


@pytest.mark.parametrize("kw", [{}, {"attn_norm": True}, {"use_rope": False}])
def test_forward_rows_with_host_attention_equals_the_engine_forward(kw):
    dc, w = _draft(**kw)
    m = DraftModel(dc, w)
    ids, pos, hidden = _rows(dc)
    t = ids.shape[0]
    cache = DraftCache.allocate(dc, torch.arange(1, dtype=torch.int32).view(1, 1), 16, "cpu", torch.float32)
    extra = torch.arange(t, dtype=torch.int32).expand(t, t).contiguous()  # row r: slots 0..r (itself last)
    zero = torch.zeros(t, dtype=torch.int32)
    want = m.forward(ids, hidden, pos, zero, torch.arange(t, dtype=torch.int32), zero, zero, extra,
                     torch.arange(1, t + 1, dtype=torch.int32), cache)
    seen = {}

    def attend(q, k, v):
        seen.update(q=q.shape, k=k.shape, v=v.shape)
        return _causal(q, k, v)

    got = m.forward_rows(ids, pos, hidden, attend)
    assert seen == {"q": (t, dc.num_heads, dc.head_dim), "k": (t, dc.num_kv_heads, dc.head_dim),
                    "v": (t, dc.num_kv_heads, dc.head_dim)}
    for a, b in zip(got, want):
        assert torch.allclose(a, b, rtol=1e-5, atol=1e-5)


def test_vllm_config_check_drops_vllm_keys_and_refuses_unbuilt_structures():
    from eagle4_b200.plugins.vllm.models import LlamaForCausalLMEagle4, check_supported

    dc, _ = _draft()
    hf = dict(dc.to_hf(), eagle_aux_hidden_state_layer_ids=[0, 2, 3], target_layer_count=4)
    assert "target_layer_count" not in check_supported(hf)
    model = LlamaForCausalLMEagle4(config=types.SimpleNamespace(**hf))
    assert model.aux_layer_ids == (0, 2, 3) and model.cfg.hidden_size == dc.hidden_size
    with pytest.raises(NotImplementedError):
        check_supported(dict(hf, enable_moe=True, moe_architecture="sparse_swiglu"))
    with pytest.raises(ValueError):
        check_supported(dict(hf, some_new_structure=True))
    vllm_config = types.SimpleNamespace(speculative_config=types.SimpleNamespace(
        draft_model_config=types.SimpleNamespace(hf_config=hf)))
    assert LlamaForCausalLMEagle4(vllm_config=vllm_config).cfg == model.cfg


def test_vllm_model_rows_candidates_and_full_rows():
    from eagle4_b200.plugins.vllm.models import LlamaForCausalLMEagle4

    dc, w = _draft()
    model = LlamaForCausalLMEagle4(config=dc.to_hf())
    model.load_weights(weights.draft_state_dict(dc, w).items(), embed=w["embed"])
    own = DraftModel(dc, weights.draft_from_state_dict(dc, weights.draft_state_dict(dc, w), embed=w["embed"]))
    ids, pos, hidden = _rows(dc)
    aux = torch.randn(ids.shape[0], dc.num_aux * dc.target_hidden_size)
    assert torch.equal(model.combine_hidden_states(aux), own.project(aux))
    normed, nxt = model.forward_rows(ids, pos, hidden, _causal)
    w_normed, _ = own.forward_rows(ids, pos, hidden, _causal)
    assert torch.equal(normed, w_normed)
    probs, tok = model.compute_candidates(normed, 4)
    p2, t2 = own.candidates(normed, 4)
    assert torch.equal(tok, t2) and torch.equal(probs, p2)
    full = model.compute_logits(normed)
    assert full.shape == (ids.shape[0], V) and full.dtype == torch.float32
    assert int(torch.isfinite(full).sum(-1).min()) == dc.num_candidates
    top = torch.topk(torch.softmax(full, -1), 4)
    assert torch.equal(top.indices, tok) and torch.allclose(top.values, probs, atol=1e-6)


def test_vllm_speculator_takes_the_model_class():
    from eagle4_b200.plugins.vllm.adapter import HarnessSpeculator
    from eagle4_b200.plugins.vllm.models import LlamaForCausalLMEagle4

    dc, w = _draft()
    model = LlamaForCausalLMEagle4(config=dc.to_hf())
    with pytest.raises(RuntimeError):
        HarnessSpeculator().load_model(model, max_reqs=2, max_len=128, tree=(4, 2, 8))
    model.load_weights(weights.draft_state_dict(dc, w).items(), embed=w["embed"])
    spec = HarnessSpeculator()
    spec.load_model(model, max_reqs=2, max_len=128, tree=(4, 2, 8))
    assert spec.drafter.engine.draft is model.draft


def _shard_def(h, down, scores, lm_head, c, shards):
    """The merge's definition in float64: each shard's top ``c`` by low-rank score, then the top ``c`` of their
    union by exact logit."""
    per = -(-scores.shape[0] // shards)
    pool = []
    for r in range(shards):
        lo, hi = r * per, min((r + 1) * per, scores.shape[0])
        s = (h.double() @ down.double().T) @ scores[lo:hi].double().T
        pool.append(torch.topk(s, c, dim=-1).indices + lo)
    ids = torch.cat(pool, -1)
    exact = torch.einsum("th,tch->tc", h.double(), lm_head.double()[ids])
    top, pick = torch.topk(exact, c, dim=-1)
    return torch.gather(ids, -1, pick), top


def test_shard_candidates_and_merge_match_their_definition():
    dc, w = _draft()
    h = torch.randn(5, dc.hidden_size, generator=torch.Generator().manual_seed(4))
    c, shards, per = dc.num_candidates, 2, V // 2
    parts = [cl.shard_candidates(h, w["lr_down"], w["lr_scores"][r * per:(r + 1) * per],
                                 w["lm_head"][r * per:(r + 1) * per], num_candidates=c, vocab_start=r * per)
             for r in range(shards)]
    for r, p in enumerate(parts):
        inside = (p.token_ids >= r * per) & (p.token_ids < (r + 1) * per)
        assert p.token_ids.dtype == torch.int64 and bool(inside.all())
    fake_gather = iter([torch.cat([p.logits for p in parts], -1), torch.cat([p.token_ids for p in parts], -1)])
    merged = cl.merge_candidates(parts[0], c, lambda x: next(fake_gather))
    want_ids, want_logits = _shard_def(h, w["lr_down"], w["lr_scores"], w["lm_head"], c, shards)
    order = torch.argsort(merged.token_ids, -1)
    w_order = torch.argsort(want_ids, -1)
    assert torch.equal(torch.gather(merged.token_ids, -1, order), torch.gather(want_ids, -1, w_order))
    assert torch.allclose(torch.gather(merged.logits, -1, order).double(), torch.gather(want_logits, -1, w_order),
                          atol=1e-4)
    # one rank: returned as is
    one = cl.merge_candidates(parts[1], c)
    assert one.token_ids is parts[1].token_ids


def test_padding_rows_of_a_shard_are_never_candidates():
    dc, w = _draft()
    h = torch.randn(3, dc.hidden_size, generator=torch.Generator().manual_seed(8))
    scores = w["lr_scores"][:1000].clone()
    scores[900:] = 1e4  # padding rows with huge scores
    got = cl.shard_candidates(h, w["lr_down"], scores, w["lm_head"][:1000], num_candidates=16, vocab_start=2000,
                              vocab_rows=900)
    assert bool((got.token_ids < 2900).all()) and bool((got.token_ids >= 2000).all())
    with pytest.raises(ValueError):
        cl.shard_candidates(h, w["lr_down"], scores, w["lm_head"][:1000], num_candidates=901, vocab_rows=900)


def test_scatter_to_vocab_softmax_is_the_candidates_softmax():
    g = torch.Generator().manual_seed(2)
    logits = torch.randn(4, 8, generator=g)
    ids = torch.stack([torch.randperm(100, generator=g)[:8] for _ in range(4)])
    full = cl.scatter_to_vocab(cl.Candidates(logits, ids), 100)
    assert torch.isinf(full).sum() == 4 * 92
    assert torch.allclose(torch.gather(torch.softmax(full, -1), -1, ids), torch.softmax(logits, -1))


def test_candidate_logits_processor_on_a_stand_in_sglang(monkeypatch):
    class LogitsProcessor:
        def __init__(self, config):
            self.vocab_size = config.vocab_size
            self.logit_scale = None
            self.final_logit_softcapping = None

        def _copy_logits_to_buffer(self, logits, logits_metadata, use_buffer=True):
            return ("copied", logits, logits_metadata)

    mod = types.ModuleType("sglang.srt.layers.logits_processor")
    mod.LogitsProcessor = LogitsProcessor
    for name in ("sglang", "sglang.srt", "sglang.srt.layers"):
        monkeypatch.setitem(sys.modules, name, types.ModuleType(name))
    monkeypatch.setitem(sys.modules, "sglang.srt.layers.logits_processor", mod)
    cand = cl.Candidates(torch.tensor([[1.0, 2.0]]), torch.tensor([[3, 7]]))
    proc = cl.candidate_logits_processor(types.SimpleNamespace(vocab_size=10), lambda h: cand)
    tag, logits, meta = proc._get_logits(torch.zeros(1, 4), None, "meta")
    assert tag == "copied" and meta == "meta" and logits[0, 3] == 1.0 and logits[0, 7] == 2.0
    assert int(torch.isinf(logits).sum()) == 8
    with pytest.raises(NotImplementedError):
        proc._get_logits(torch.zeros(1, 4), None, "meta", embedding_bias=torch.zeros(10))


def test_tokenspeed_exit_and_candidate_topk_one_rank():
    from eagle4_b200.plugins.tokenspeed.models import CandidateRows, LlamaForCausalLMEagle4

    dc, w = _draft()
    model = LlamaForCausalLMEagle4(dc.to_hf())
    model.load_weights(weights.draft_state_dict(dc, w).items(), embed=w["embed"])
    normed = torch.randn(6, dc.hidden_size, generator=torch.Generator().manual_seed(5))
    nxt = normed * 2
    ctx = types.SimpleNamespace(gather_ids=torch.tensor([1, 4]), logits_rows_selected=False, input_logprob_rows=None,
                                query_shard=None)
    out = model.exit_logits(None, normed, (nxt,), ctx)
    assert isinstance(out, CandidateRows) and out.next_token_logits.shape == (2, 0)
    assert torch.equal(out.normed, normed[[1, 4]]) and torch.equal(out.hidden_states, nxt[[1, 4]])
    # rows already one per request stay as they are
    same = model.exit_logits(None, normed[:2], (nxt[:2],), ctx)
    assert torch.equal(same.normed, normed[:2])
    with pytest.raises(NotImplementedError):
        model.exit_logits(None, normed, (nxt,), types.SimpleNamespace(input_logprob_rows=[0], query_shard=None))
    probs, ids = model.candidate_topk(out.normed, 4)
    p2, i2 = DraftModel(dc, w).candidates(out.normed, 4)
    assert torch.equal(ids, i2) and torch.allclose(probs, p2)
    full = model.full_logits(out.normed)
    assert torch.equal(torch.topk(full, 4).indices, i2)
    with pytest.raises(NotImplementedError):
        LlamaForCausalLMEagle4(dataclasses.replace(dc, low_rank=None).to_hf())


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from eagle4_b200.plugins.tokenspeed.models import LlamaForCausalLMEagle4

        dc, w = _draft()
        mapping = types.SimpleNamespace(lm_head=types.SimpleNamespace(tp_rank=rank, tp_size=world))
        model = LlamaForCausalLMEagle4(dc.to_hf(), mapping)
        model.load_weights(weights.draft_state_dict(dc, w).items(), embed=w["embed"],
                           all_gather=cl.group_all_gather())
        normed = torch.randn(5, dc.hidden_size, generator=torch.Generator().manual_seed(6))
        cand, (probs, ids) = model.candidate_head(normed, 4)
        want_ids, want_logits = _shard_def(normed, w["lr_down"], w["lr_scores"], w["lm_head"], dc.num_candidates,
                                           world)
        got = torch.sort(cand.token_ids, -1).values
        out[rank] = {"ids_ok": bool(torch.equal(got, torch.sort(want_ids, -1).values)),
                     "ids": ids.tolist(), "probs": probs.tolist(),
                     "rows": (model.vocab_start, model.vocab_rows)}
    finally:
        dist.destroy_process_group()


def test_tokenspeed_candidate_head_over_two_vocab_shards():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_tp_worker, args=(2, _port(), out), nprocs=2, start_method="spawn", join=True)
        res = dict(out)
    assert res[0]["ids_ok"] and res[1]["ids_ok"]
    assert res[0]["ids"] == res[1]["ids"] and res[0]["probs"] == res[1]["probs"]
    assert res[0]["rows"] == (0, V // 2) and res[1]["rows"] == (V // 2, V // 2)


def test_sglang_model_shares_the_embedding_and_answers_the_worker():
    from eagle4_b200.plugins.sglang.models.llama_eagle4 import LlamaForCausalLMEagle4

    dc, w = _draft()
    model = LlamaForCausalLMEagle4(dc.to_hf())
    embed = w["embed"].clone()
    model.set_embed_and_head(embed, torch.zeros(1))  # the head argument is not taken
    model.load_weights(weights.draft_state_dict(dc, w).items())
    assert model.draft.w["embed"] is embed and model.draft.w["lm_head"].shape[0] == V
    assert model.get_hot_token_id() is None
    assert model.get_attention_sliding_window_size() == (dc.sliding_window - 1 if dc.sliding_window else None)
    normed = torch.randn(4, dc.hidden_size, generator=torch.Generator().manual_seed(9))
    probs, ids = model.candidate_topk(normed, 3)
    p2, i2 = DraftModel(dc, w).candidates(normed, 3)
    assert torch.equal(ids, i2) and torch.allclose(probs, p2)
    cand = model.proposal_candidates(normed)
    assert cand.logits.shape == (4, dc.num_candidates) and cand.token_ids.dtype == torch.int64
    full = cl.scatter_to_vocab(cand, V)
    assert torch.equal(torch.topk(full, 3).indices, i2)
