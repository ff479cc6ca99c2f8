"""A Hugging Face Nemotron-H checkpoint through ``api.from_pretrained`` (CPU, reference ops): the logits of a prompt
must match Hugging Face's own model on the same weights. This covers the checkpoint names (``backbone.`` or
``model.`` trunk), the Mamba2 in_proj layout, the conv bias, the gated norm's per-channel weight and its
gate-before-norm order, NoPE attention, and the config reader (``layers_block_type`` or ``hybrid_override_pattern``).
The ops that take the new options are compared with their definitions as well."""

import json
import os

import pytest
import torch

from eagle4_b200.models.configs import TargetConfig
from eagle4_b200.ops import reference as ref

transformers = pytest.importorskip("transformers")


def _hf_model(seed=0):
    from transformers import NemotronHConfig, NemotronHForCausalLM

    torch.manual_seed(seed)
    cfg = NemotronHConfig(vocab_size=512, hidden_size=128, hybrid_override_pattern="M*MM", num_attention_heads=4,
                          num_key_value_heads=2, head_dim=32, intermediate_size=256, mamba_num_heads=8,
                          mamba_head_dim=16, ssm_state_size=16, n_groups=2, conv_kernel=4, use_conv_bias=True,
                          layer_norm_epsilon=1e-5, chunk_size=16, time_step_min=1e-6)
    model = NemotronHForCausalLM(cfg).eval()
    with torch.no_grad():  # move every weight off its identity / constant init so each mapping matters
        for name, p in model.named_parameters():
            p.add_(torch.randn_like(p) * (0.05 if "norm" in name or "bias" in name or name.endswith("D") else 0.01))
    return cfg, model


def _save(tmp_path, cfg, model, prefix):
    from safetensors.torch import save_file

    sd = {k.replace("model.", prefix, 1) if k.startswith("model.") else k: v.contiguous()
          for k, v in model.state_dict().items()}
    save_file(sd, os.path.join(tmp_path, "model.safetensors"))
    with open(os.path.join(tmp_path, "config.json"), "w") as f:
        json.dump(cfg.to_dict(), f, default=float)


@pytest.mark.parametrize("prefix", ["backbone.", "model."])
def test_nemotron_h_checkpoint_logits_match_hugging_face(tmp_path, prefix):
    from eagle4_b200.api import from_pretrained

    cfg, model = _hf_model()
    _save(str(tmp_path), cfg, model, prefix)
    llm = from_pretrained(str(tmp_path), device="cpu", dtype=torch.float32, max_len=64)
    assert llm.target.cfg.mamba_gate_first and [m for m, _ in llm.target.cfg.layers] == ["mamba", "attn", "mamba",
                                                                                          "mamba"]
    ids = torch.randint(0, 512, (11,), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        want = model(ids[None]).logits[0].double()
    got = _prefill_logits(llm, ids)
    assert torch.allclose(got, want, atol=1e-4 * want.abs().max().item(), rtol=1e-4), (got - want).abs().max()
    assert torch.equal(got.argmax(-1), want.argmax(-1))


def test_config_reader_takes_block_lists_and_refuses_moe_blocks():
    base = {"model_type": "nemotron_h", "hidden_size": 64, "vocab_size": 100, "intermediate_size": 128,
            "num_attention_heads": 2, "num_key_value_heads": 1, "head_dim": 32, "mamba_num_heads": 4,
            "mamba_head_dim": 16, "ssm_state_size": 16, "n_groups": 1}
    a = TargetConfig.from_hf(dict(base, hybrid_override_pattern="M-*"))
    b = TargetConfig.from_hf(dict(base, layers_block_type=["mamba", "mlp", "attention"]))
    assert a.layers == b.layers == [("mamba", None), (None, "relu2"), ("attn", None)]
    assert a.mamba_gate_first  # Hugging Face's order unless the config says otherwise
    assert TargetConfig.from_hf(a.to_hf()) == a
    with pytest.raises(NotImplementedError):
        TargetConfig.from_hf(dict(base, layers_block_type=["mamba", "moe"]))


def test_conv_bias_and_gate_first_norm_match_their_definitions():
    g = torch.Generator().manual_seed(3)
    x, cs = torch.randn(5, 6, generator=g), torch.randn(1, 6, 3, generator=g)
    w, bias = torch.randn(6, 4, generator=g), torch.randn(6, generator=g)
    parent = torch.tensor([-1, 0, 1, 1, 3])
    slot = torch.zeros(5, dtype=torch.int32)
    plain = ref.causal_conv_tree(x, cs, slot, parent, w)
    biased = ref.causal_conv_tree(x, cs, slot, parent, w, bias)
    win = torch.cat([cs[0], x[0:1].t()], 1)  # row 0: the committed window, then the row itself
    assert torch.allclose(biased[0], torch.nn.functional.silu((w * win).sum(1) + bias), atol=1e-6)
    assert not torch.allclose(plain, biased)
    o, z = torch.randn(4, 2, 8, generator=g), torch.randn(4, 16, generator=g)
    wn = torch.randn(16, generator=g)
    got = ref.gated_rmsnorm(o, z, wn, 1e-5, gate_first=True)
    y = o.reshape(4, 16) * torch.nn.functional.silu(z)
    yg = y.view(4, 2, 8)
    want = (yg * torch.rsqrt(yg.square().mean(-1, keepdim=True) + 1e-5)).reshape(4, 16) * wn
    assert torch.allclose(got, want, atol=1e-6)
    shared = ref.gated_rmsnorm(o, z, wn[:8], 1e-5)
    want_shared = (o * torch.rsqrt(o.square().mean(-1, keepdim=True) + 1e-5) * wn[:8]).reshape(4, 16) * \
        torch.nn.functional.silu(z)
    assert torch.allclose(shared, want_shared, atol=1e-6)


def _prefill_logits(llm, ids):
    from eagle4_b200.models.target import RowBatch

    eng = llm.engine
    n = ids.shape[0]
    eng.pages.reserve(0, n + 1)
    pos = torch.arange(n)
    rb = RowBatch(ids=ids, pos=pos, req=torch.zeros(n, dtype=torch.int32), write_slot=eng._slots(torch.tensor(0), pos),
                  ctx_start=torch.zeros(n, dtype=torch.int32), ctx_len=(pos + 1).int(),
                  extra=torch.zeros(n, 1, dtype=torch.int32), n_extra=torch.zeros(n, dtype=torch.int32),
                  parent=(pos - 1).int(), state_slot=torch.zeros(n, dtype=torch.int32), scan=True)
    h, _ = llm.target.forward(rb, eng.tcache)
    return llm.target.logits(h).double()


def _tp_worker(rank, world, port, path, out):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(1)
    try:
        from eagle4_b200.api import from_pretrained
        from eagle4_b200.parallel.tp import TensorParallel

        llm = from_pretrained(path, device="cpu", dtype=torch.float32, max_len=64, tp=TensorParallel(backend="torch"))
        ids = torch.randint(0, 512, (11,), generator=torch.Generator().manual_seed(1))
        out[rank] = _prefill_logits(llm, ids).tolist()
    finally:
        dist.destroy_process_group()


def test_nemotron_h_checkpoint_sharded_over_two_ranks(tmp_path):
    """The conv bias and the per-group norm weights are sharded with their heads and groups."""
    import socket

    import torch.multiprocessing as mp

    cfg, model = _hf_model(seed=4)
    _save(str(tmp_path), cfg, model, "backbone.")
    ids = torch.randint(0, 512, (11,), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        want = model(ids[None]).logits[0].double()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_tp_worker, args=(2, port, str(tmp_path), out), nprocs=2, start_method="spawn", join=True)
        res = dict(out)
    for r in range(2):
        got = torch.tensor(res[r], dtype=torch.float64)
        assert torch.allclose(got, want, atol=1e-4 * want.abs().max().item(), rtol=1e-4), (r, (got - want).abs().max())
