"""Full rounds through the engine adapters with fake hosts. The host is a target-only engine (it prefills with aux
capture and verifies externally drafted rows, as SGLang / vLLM / TokenSpeed do with their own models); the adapter
drafts with plugins.host_round.HostDrafter and takes the accepted path. The emitted tokens must equal the engine's
own generation: plain greedy for greedy rounds, and, with the round counter shared as in one process, the sampled
engine's tokens for sampled rounds."""

from types import SimpleNamespace

import pytest
import torch

from eagle4_b200.api import LLM, TreeSpec
from eagle4_b200.runtime.engine import Engine

TREE = TreeSpec(4, 2, 8)


def _setup(bs, temperature=0.0, name="tiny"):
    llm = LLM.synthetic(name, device="cpu", dtype=torch.float32, tree=TREE, max_batch=bs, max_len=256,
                        temperature=temperature, sample_seed=5)
    host = Engine(llm.target, None, max_reqs=bs, max_len=256, steps=TREE.steps, top_k=TREE.top_k,
                  verify_tokens=TREE.draft_tokens, temperature=temperature, seed=5)
    g = torch.Generator().manual_seed(bs + 17)
    prompts = [torch.randint(1, 4096, (int(torch.randint(6, 40, (1,), generator=g)),), generator=g) for _ in range(bs)]
    return llm, host, prompts


def _drafter(llm, bs, temperature=0.0):
    from eagle4_b200.plugins.host_round import HostDrafter

    return HostDrafter(llm.draft, max_reqs=bs, max_len=256, steps=TREE.steps, top_k=TREE.top_k,
                       verify_tokens=TREE.draft_tokens, temperature=temperature, seed=5)


def _host_verify(host, bs, tokens, prow, accept):
    w = tokens.shape[1]
    tk, acc, cnt, bonus, aux = host._verify_forward(bs, w, tokens[:, 1:] if w > 1 else None, prow, None,
                                                    accept=accept)
    host.L[:bs] += cnt.long()
    host.root[:bs] = bonus
    return tk, acc, cnt, bonus, aux


@pytest.mark.parametrize("bs", [1, 3])
def test_sglang_draft_worker_rounds_equal_plain_greedy(bs):
    from eagle4_b200.plugins.sglang.adapter import HarnessDraftWorker, HarnessWorker

    llm, host, prompts = _setup(bs)
    n_new = 12
    want = llm.generate(prompts, n_new, speculative=False).tolist()
    worker = HarnessDraftWorker.for_drafter(_drafter(llm, bs))
    reqs = [SimpleNamespace(rid=f"r{b}", origin_input_ids=p.tolist()) for b, p in enumerate(prompts)]
    batch = SimpleNamespace(reqs=reqs)
    firsts, auxes = [], []
    for b, p in enumerate(prompts):
        first, aux = host.prefill(b, p)
        firsts.append(int(first[0]))
        auxes.append(aux)
    worker.forward_draft_extend(batch, torch.cat(auxes), torch.tensor(firsts))
    outs = [[f] for f in firsts]
    rounds = 0
    while min(len(o) for o in outs) < n_new:
        spec = worker.draft_round(batch)
        assert spec["draft_tokens"].shape == spec["parent_rows"].shape == (bs, spec["width"])
        tk, acc, cnt, bonus, aux = _host_verify(host, bs, spec["draft_tokens"], spec["parent_rows"], lambda out, t:
                                                HarnessWorker.accept_step(None, host.target.greedy(out)[0], t,
                                                                          spec["parent_rows"]))
        for o, e in zip(outs, worker.finish_round(spec, acc, cnt, bonus, aux)):
            o.extend(e)
        rounds += 1
    assert [o[:n_new] for o in outs] == want
    assert rounds < n_new * bs + 2


def test_vllm_speculator_rounds_with_logits_and_release():
    from eagle4_b200.plugins.vllm.adapter import HarnessSpeculator

    bs = 3
    llm, host, prompts = _setup(bs)
    want = llm.generate(prompts, 10, speculative=False).tolist()
    spec = HarnessSpeculator.__new__(HarnessSpeculator)
    spec.load_model(llm.draft, max_reqs=bs, max_len=256, tree=(TREE.steps, TREE.top_k, TREE.draft_tokens))
    rids = [10, 11, 12]
    outs = {}
    for b, (rid, p) in enumerate(zip(rids, prompts)):
        first, aux = host.prefill(b, p)
        spec.prefill_request(rid, p, aux, int(first[0]))
        outs[rid] = [int(first[0])]
    limits = {10: 10, 11: 4, 12: 10}  # request 11 finishes early and leaves the batch
    live = list(rids)
    while live:
        tokens, prow = spec.propose_tree(live)
        assert torch.equal(spec.prepare_verify_inputs(prow, torch.zeros(len(live), dtype=torch.long))[0][:, 0],
                           torch.zeros(len(live), dtype=torch.long))
        # the host's rejection sampler is the adapter's TreeAccept on the verify logits; the aux rows are known
        # after the forward, so the accepted path goes to the drafter afterwards
        tk, acc, cnt, bonus, aux = host._verify_forward(len(live), tokens.shape[1],
                                                        tokens[:, 1:] if tokens.shape[1] > 1 else None, prow, None,
                                                        accept=lambda out, t: _logit_accept(spec, out, t, prow, host))
        host.L[:len(live)] += cnt.long()
        host.root[:len(live)] = bonus
        emitted = spec.drafter.accept(live, tk, acc, cnt, bonus, aux)
        for rid, e in zip(live, emitted):
            outs[rid].extend(e)
        done = [r for r in live if len(outs[r]) >= limits[r]]
        for r in done:
            spec.finish_request(r)
            b = live.index(r)
            # the host compacts its own rows the same way (last row into the hole)
            last = len(live) - 1
            for t in (host.L, host.root, host.slot):
                t[b] = t[last]
            live[b] = live[last]
            live.pop()
    for b, rid in enumerate(rids):
        assert outs[rid][:limits[rid]] == want[b][:limits[rid]]


def _logit_accept(spec, out, tokens, prow, host):
    return spec.make_rejection_sampler()(host.target.logits(out), tokens, prow)


def test_vllm_sampled_tree_accept_equals_the_sampled_engine():
    from eagle4_b200.plugins.vllm.adapter import HarnessSpeculator

    bs, temp = 2, 0.8
    llm, host, prompts = _setup(bs, temperature=temp)
    want = llm.generate(prompts, 10).tolist()  # sampled speculative engine, seed 5
    spec = HarnessSpeculator.__new__(HarnessSpeculator)
    spec.load_model(llm.draft, max_reqs=bs, max_len=256, tree=(TREE.steps, TREE.top_k, TREE.draft_tokens),
                    temperature=temp, seed=5)
    spec.drafter.engine.round_ctr = host.round_ctr  # one process, one round counter (as in the engine)
    outs = []
    for b, p in enumerate(prompts):
        first, aux = host.prefill(b, p)
        spec.prefill_request(b, p, aux, int(first[0]))
        outs.append([int(first[0])])
    while min(len(o) for o in outs) < 10:
        tokens, prow = spec.propose_tree([0, 1])
        tk, acc, cnt, bonus, aux = host._verify_forward(bs, tokens.shape[1],
                                                        tokens[:, 1:] if tokens.shape[1] > 1 else None, prow, None,
                                                        accept=lambda out, t: _logit_accept(spec, out, t, prow, host))
        host.L[:bs] += cnt.long()
        host.root[:bs] = bonus
        for o, e in zip(outs, spec.drafter.accept([0, 1], tk, acc, cnt, bonus, aux)):
            o.extend(e)
    assert [o[:10] for o in outs] == want


def test_tokenspeed_drafter_rounds_equal_plain_greedy():
    from eagle4_b200.plugins.tokenspeed.adapter import HarnessDrafter

    bs = 2
    llm, host, prompts = _setup(bs, name="tiny-moe")  # a latent-MoE / attn_norm draft through the host path
    want = llm.generate(prompts, 9, speculative=False).tolist()
    d = HarnessDrafter.__new__(HarnessDrafter)
    d.attach(_drafter(llm, bs))
    outs = []
    for b, p in enumerate(prompts):
        first, aux = host.prefill(b, p)
        d.prefill_request(b, p, aux, int(first[0]))
        outs.append([int(first[0])])
    while min(len(o) for o in outs) < 9:
        tokens, prow = d.draft_round([0, 1])
        holder = {}

        def accept(out, t):
            from eagle4_b200.plugins.common import accept_greedy_rows

            holder["ids"], _ = host.target.greedy(out)
            return accept_greedy_rows(holder["ids"], t, prow)

        tk, acc, cnt, bonus, aux = _host_verify(host, bs, tokens, prow, accept)
        _, _, _, emitted = d.accept_round([0, 1], tk, holder["ids"], prow, aux)
        for o, e in zip(outs, emitted):
            o.extend(e)
    assert [o[:9] for o in outs] == want
