"""Hugging Face Qwen3.5 and Llama checkpoints through ``api.from_pretrained`` (CPU, reference ops): the logits of a
prompt must match Hugging Face's own model on the same weights (GDN layers with their gated norm, gated attention with
q/k norms and partial rotary, the zero-centred RMSNorm offset, SwiGLU; Llama's full rotary attention)."""

import json
import os

import pytest
import torch

pytest.importorskip("transformers")


def _perturb(model, scale=0.02):
    with torch.no_grad():  # move every weight off its identity / constant init so each mapping matters
        for name, p in model.named_parameters():
            p.add_(torch.randn_like(p) * (0.05 if "norm" in name or "bias" in name else scale))


def _save(path, cfg, model):
    from safetensors.torch import save_file

    save_file({k: v.contiguous() for k, v in model.state_dict().items()}, os.path.join(path, "model.safetensors"))
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg.to_dict(), f, default=float)


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


def _check(tmp_path, cfg, model):
    from eagle4_b200.api import from_pretrained

    _save(str(tmp_path), cfg, model)
    llm = from_pretrained(str(tmp_path), device="cpu", dtype=torch.float32, max_len=64)
    ids = torch.randint(0, cfg.vocab_size, (13,), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        want = model(ids[None]).logits[0].double()
    got = _prefill_logits(llm, ids)
    assert torch.allclose(got, want, atol=1e-4 * want.abs().max().item(), rtol=1e-4), (got - want).abs().max()
    assert torch.equal(got.argmax(-1), want.argmax(-1))
    return llm


def test_qwen3_5_checkpoint_logits_match_hugging_face(tmp_path):
    from transformers import Qwen3_5ForCausalLM, Qwen3_5TextConfig

    torch.manual_seed(0)
    cfg = Qwen3_5TextConfig(vocab_size=512, hidden_size=128, num_hidden_layers=4,
                            layer_types=["linear_attention"] * 3 + ["full_attention"], num_attention_heads=4,
                            num_key_value_heads=2, head_dim=32, intermediate_size=256, linear_num_key_heads=2,
                            linear_num_value_heads=4, linear_key_head_dim=16, linear_value_head_dim=16,
                            linear_conv_kernel_dim=4)
    model = Qwen3_5ForCausalLM(cfg).eval()
    _perturb(model)
    llm = _check(tmp_path, cfg, model)
    assert [m for m, _ in llm.target.cfg.layers] == ["gdn", "gdn", "gdn", "attn"]
    assert llm.target.cfg.rotary_dim == 8  # partial rotary 0.25 of head_dim 32


def test_llama_checkpoint_logits_match_hugging_face(tmp_path):
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(1)
    cfg = LlamaConfig(vocab_size=512, hidden_size=128, num_hidden_layers=3, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=32, intermediate_size=256, rope_theta=500000.0)
    model = LlamaForCausalLM(cfg).eval()
    _perturb(model)
    _check(tmp_path, cfg, model)


def test_eagle3_draft_without_aux_ids_takes_the_target_default_and_decodes_greedily(tmp_path):
    """An EAGLE-3 draft whose config names no aux layers (with a reduced draft vocabulary and ``d2t``) over a Llama
    checkpoint: the aux layers are 2, L // 2, L - 3 of the target, and speculative output equals plain greedy."""
    import dataclasses

    from transformers import LlamaConfig, LlamaForCausalLM

    from eagle4_b200.api import TreeSpec, from_pretrained
    from eagle4_b200.models import configs, weights

    torch.manual_seed(2)
    cfg = LlamaConfig(vocab_size=512, hidden_size=128, num_hidden_layers=8, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=32, intermediate_size=256)
    model = LlamaForCausalLM(cfg).eval()
    _perturb(model)
    target_dir, draft_dir = tmp_path / "t", tmp_path / "d"
    target_dir.mkdir()
    _save(str(target_dir), cfg, model)
    tcfg = configs.TargetConfig.from_hf(cfg.to_dict())
    dcfg = dataclasses.replace(configs.eagle3_llama_draft(tcfg), draft_vocab_size=128)
    dw = weights.init_draft(dcfg, seed=5)
    weights.save_draft(str(draft_dir), dcfg, dw)
    hf = json.loads((draft_dir / "config.json").read_text())
    hf.pop("eagle_config", None)
    (draft_dir / "config.json").write_text(json.dumps(hf))
    llm = from_pretrained(str(target_dir), str(draft_dir), device="cpu", dtype=torch.float32, max_len=128,
                          tree=TreeSpec(4, 2, 8))
    assert llm.draft.cfg.aux_layer_ids == (2, 4, 5) and llm.draft.cfg.family == "eagle3"
    prompt = torch.randint(0, 512, (1, 12), generator=torch.Generator().manual_seed(3))
    spec = llm.generate(prompt, 10)
    plain = llm.generate(prompt, 10, speculative=False)
    assert torch.equal(spec, plain)
    with torch.no_grad():
        ids = prompt[0].tolist()
        for _ in range(10):
            ids.append(int(model(torch.tensor([ids])).logits[0, -1].argmax()))
    assert plain[0].tolist() == ids[12:]


def _hf_target(kind):
    if kind == "qwen3_5":
        from transformers import Qwen3_5ForCausalLM, Qwen3_5TextConfig

        cfg = Qwen3_5TextConfig(vocab_size=512, hidden_size=128, num_hidden_layers=4,
                                layer_types=["linear_attention"] * 3 + ["full_attention"], num_attention_heads=4,
                                num_key_value_heads=2, head_dim=32, intermediate_size=256, linear_num_key_heads=2,
                                linear_num_value_heads=4, linear_key_head_dim=16, linear_value_head_dim=16,
                                linear_conv_kernel_dim=4)
        return cfg, Qwen3_5ForCausalLM(cfg).eval()
    from transformers import NemotronHConfig, NemotronHForCausalLM

    cfg = NemotronHConfig(vocab_size=512, hidden_size=128, hybrid_override_pattern="M*MM", num_attention_heads=4,
                          num_key_value_heads=2, head_dim=32, intermediate_size=256, mamba_num_heads=8,
                          mamba_head_dim=16, ssm_state_size=16, n_groups=2, conv_kernel=4, use_conv_bias=True,
                          layer_norm_epsilon=1e-5, chunk_size=16, time_step_min=1e-6)
    return cfg, NemotronHForCausalLM(cfg).eval()


@pytest.mark.parametrize("kind", ["qwen3_5", "nemotron_h"])
def test_eagle4_draft_over_a_checkpoint_target_decodes_plain_greedy(tmp_path, kind):
    """An EAGLE-4 draft checkpoint (low-rank candidate head) over a Hugging Face target: speculative output equals
    plain greedy decoding, which equals Hugging Face's own greedy decoding."""
    import dataclasses

    from eagle4_b200.api import TreeSpec, from_pretrained
    from eagle4_b200.models import configs, weights

    torch.manual_seed(4)
    cfg, model = _hf_target(kind)
    _perturb(model)
    target_dir, draft_dir = tmp_path / "t", tmp_path / "d"
    target_dir.mkdir()
    _save(str(target_dir), cfg, model)
    tcfg = configs.TargetConfig.from_hf(json.loads((target_dir / "config.json").read_text()))
    dcfg = dataclasses.replace(configs.tiny_draft(tcfg, draft_vocab=512), aux_layer_ids=(0, 1, 2))
    weights.save_draft(str(draft_dir), dcfg, weights.init_draft(dcfg, seed=6))
    llm = from_pretrained(str(target_dir), str(draft_dir), device="cpu", dtype=torch.float32, max_len=128,
                          tree=TreeSpec(4, 2, 8))
    prompt = torch.randint(0, 512, (1, 9), generator=torch.Generator().manual_seed(5))
    spec = llm.generate(prompt, 8)
    plain = llm.generate(prompt, 8, speculative=False)
    assert torch.equal(spec, plain)
    with torch.no_grad():
        ids = prompt[0].tolist()
        for _ in range(8):
            ids.append(int(model(torch.tensor([ids])).logits[0, -1].argmax()))
    assert plain[0].tolist() == ids[9:]


def test_dense_qwen3_checkpoint_logits_match_hugging_face(tmp_path):
    from transformers import Qwen3Config, Qwen3ForCausalLM

    torch.manual_seed(6)
    cfg = Qwen3Config(vocab_size=512, hidden_size=128, num_hidden_layers=3, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=32, intermediate_size=256)
    model = Qwen3ForCausalLM(cfg).eval()
    _perturb(model)
    llm = _check(tmp_path, cfg, model)
    assert llm.target.cfg.family == "qwen3" and llm.target.cfg.qk_norm and not llm.target.cfg.norm_offset


def test_moe_targets_are_refused():
    from eagle4_b200.models.configs import TargetConfig

    with pytest.raises(NotImplementedError, match="mixture-of-experts"):
        TargetConfig.from_hf({"model_type": "qwen3_moe", "num_experts": 64})
    with pytest.raises(NotImplementedError, match="mixture-of-experts"):
        TargetConfig.from_hf({"model_type": "qwen3_next", "num_experts": 512})
