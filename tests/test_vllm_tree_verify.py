"""vLLM's GDN / Mamba2 spec rows under tree verify (plugins/vllm/tree_verify.py), on CPU with stand-in spec rows.

vLLM keeps the state a step resumes from in ``state_indices[b, num_accepted - 1]`` and the conv window at column
``num_accepted - 1`` of ``conv_state[state_indices[b, 0]]`` (either conv layout). A tree round through the extension,
its commit of the accepted path and a following round must give the outputs of plain decoding of the same tokens:
here the plain outputs are computed from the round's inputs with chain parents from the original state."""

import types

import pytest
import torch

from eagle4_b200.ops import reference as ref
from eagle4_b200.plugins.common import GdnShape
from eagle4_b200.plugins.vllm import tree_verify as tv

KW, SPEC = 4, 4
PARENTS = torch.tensor([[-1, 0, 0, 1, 2], [-1, 0, 1, 1, 2]])
QSL = torch.tensor([0, 5, 9])  # request 1 verifies a 4-row prefix of its staged tree
STATE_INDICES = torch.tensor([[3, 4, 5, 6, 7], [8, 9, 10, 11, 2]], dtype=torch.int32)
PATHS = [[0, 2, 4], [0, 1]]  # accepted rows (local), root first


def _pool(slots, *shape, gen):
    """A state pool whose slots are not contiguous (vLLM keeps them inside a larger page)."""
    return (torch.randn(slots, 2, *shape, generator=gen) * 0.3)[:, 0]


def _conv_pool(slots, channels, dim_first, gen):
    full = torch.randn(slots, channels, KW - 1 + SPEC, generator=gen)
    return full if dim_first else full.transpose(1, 2).contiguous()


def _window(conv_state, slot, start, channels):
    if conv_state.shape[1] == channels:
        return conv_state[slot, :, start:start + KW - 1].clone()
    return conv_state[slot, start:start + KW - 1, :].t().clone()


def _chain_outputs(kind, shape, params, state0, window0, x, gate, steps):
    """Plain decoding of rows ``steps`` (in order) from one request's state and window; float64 reference ops."""
    xs = x[steps]
    parent = torch.arange(len(steps)) - 1
    slot = torch.zeros(len(steps), dtype=torch.int32)
    conv = ref.causal_conv_tree(xs, window0[None], slot, parent, params["weight"], params.get("bias"))
    if kind == "gdn":
        a, b = gate[0][steps], gate[1][steps]
        g, beta = ref.gdn_gates(a, b, params["A_log"], params["dt_bias"])
        return ref.gdn_tree(conv, g, beta, state0[None].clone(), slot, parent, shape, False).reshape(len(steps), -1)
    dt = gate[steps]
    y = ref.mamba_tree(conv, dt, params["A_log"], params["dt_bias"], params["D"], state0[None].clone(), slot, parent,
                       shape, False)
    return y.reshape(len(steps), -1)


def _rows(kind, shape, params, pools, x, gate, num_accepted, qsl, state_indices, tokens):
    out = torch.zeros(tokens, shape.gdn_value_dim if kind == "gdn" else shape.mamba_inner)
    common = dict(conv_state=pools["conv"], conv_weight=params["weight"][:, None, :], conv_bias=params.get("bias"),
                  activation="silu", state_indices=state_indices, num_accepted_tokens=num_accepted,
                  query_start_loc=qsl, ssm_state=pools["ssm"], out=out, layer_name="l0")
    if kind == "gdn":
        return types.SimpleNamespace(mixed_qkv=x, a=gate[0], b=gate[1], A_log=params["A_log"],
                                     dt_bias=params["dt_bias"], num_k_heads=shape.gdn_k_heads,
                                     head_k_dim=shape.gdn_k_dim, num_v_heads=shape.gdn_v_heads,
                                     head_v_dim=shape.gdn_v_dim, **common)
    return types.SimpleNamespace(hidden_states_B_C=x, dt=gate, A=-params["A_log"].exp(), D=params["D"],
                                 dt_bias=params["dt_bias"], num_heads=shape.mamba_heads, head_dim=shape.mamba_head_dim,
                                 n_groups=shape.mamba_groups, ssm_state_size=shape.mamba_state, **common)


def _setup(kind, dim_first, seed=0):
    g = torch.Generator().manual_seed(seed)
    if kind == "gdn":
        shape = GdnShape(2, 4, 16, 16, KW)
        channels = shape.gdn_conv_dim
        params = {"A_log": torch.randn(4, generator=g) * 0.5, "dt_bias": torch.randn(4, generator=g) * 0.5,
                  "weight": torch.randn(channels, KW, generator=g) * 0.5}
        pools = {"ssm": _pool(12, 4, 16, 16, gen=g), "conv": _conv_pool(12, channels, dim_first, g)}
        gate_of = lambda n: (torch.randn(n, 4, generator=g), torch.randn(n, 4, generator=g))  # noqa: E731
    else:
        shape = tv.MambaShape(4, 8, 16, 2, KW)
        channels = shape.mamba_inner + 2 * 2 * 16
        params = {"A_log": torch.randn(4, generator=g) * 0.5, "dt_bias": torch.randn(4, generator=g) * 0.5,
                  "D": torch.randn(4, generator=g), "weight": torch.randn(channels, KW, generator=g) * 0.5,
                  "bias": torch.randn(channels, generator=g) * 0.5}  # Nemotron-H's Mamba2 conv has a bias
        pools = {"ssm": _pool(12, 4, 8, 16, gen=g), "conv": _conv_pool(12, channels, dim_first, g)}
        gate_of = lambda n: torch.randn(n, 4, generator=g)  # noqa: E731
    return shape, channels, params, pools, gate_of, g


def _forward(ext, kind, rows):
    (ext.forward_spec_rows if kind == "gdn" else ext.forward_mamba2_spec_rows)(rows)
    return rows.out


def _cat_gate(kind, a, b):
    return (torch.cat([a[0], b[0]]), torch.cat([a[1], b[1]])) if kind == "gdn" else torch.cat([a, b])


@pytest.mark.parametrize("kind,dim_first", [("gdn", True), ("gdn", False), ("mamba2", True), ("mamba2", False)])
def test_tree_round_commit_and_next_round_equal_plain_decoding(kind, dim_first):
    shape, channels, params, pools, gate_of, g = _setup(kind, dim_first)
    num_accepted = torch.tensor([2, 1], dtype=torch.int32)
    starts = [int(a) - 1 for a in num_accepted]
    state0 = [pools["ssm"][int(STATE_INDICES[b, starts[b]])].clone() for b in range(2)]
    window0 = [_window(pools["conv"], int(STATE_INDICES[b, 0]), starts[b], channels) for b in range(2)]
    x1 = torch.randn(9, channels, generator=g)
    gate1 = gate_of(9)
    ext = tv.TreeVerify()
    tv.stage_tree(PARENTS)
    out1 = _forward(ext, kind, _rows(kind, shape, params, pools, x1, gate1, num_accepted, QSL, STATE_INDICES, 9))
    # every row's output is plain decoding of its root-to-row path
    for b in range(2):
        lo, hi = int(QSL[b]), int(QSL[b + 1])
        for r in range(lo, hi):
            path, cur = [], r - lo
            while cur >= 0:
                path.append(cur + lo)
                cur = int(PARENTS[b, cur])
            want = _chain_outputs(kind, shape, params, state0[b], window0[b], x1, gate1, path[::-1])[-1]
            assert torch.allclose(out1[r], want, atol=1e-5, rtol=1e-5), (b, r)
    accepted = torch.tensor([[0, 2, 4, -1, -1], [0, 1, -1, -1, -1]])
    counts = torch.tensor([3, 2])
    assert tv.commit_accepted(accepted, counts) == 1
    # next round: one chain row per request, read back from where vLLM resumes
    x2 = torch.randn(2, channels, generator=g)
    gate2 = gate_of(2)
    tv.stage_tree(None)
    out2 = _forward(ext, kind, _rows(kind, shape, params, pools, x2, gate2, counts.int(), torch.tensor([0, 1, 2]),
                                     STATE_INDICES, 2))
    x_all = torch.cat([x1, x2])
    gate_all = _cat_gate(kind, gate1, gate2)
    for b in range(2):
        steps = [int(QSL[b]) + p for p in PATHS[b]] + [9 + b]
        want = _chain_outputs(kind, shape, params, state0[b], window0[b], x_all, gate_all, steps)[-1]
        assert torch.allclose(out2[b], want, atol=1e-5, rtol=1e-5), b


def test_padded_requests_and_unstaged_chains():
    shape, channels, params, pools, gate_of, g = _setup("gdn", True, seed=1)
    before = pools["ssm"].clone()
    state_indices = torch.tensor([[3, 4, 5], [tv.NULL_BLOCK_ID, 0, 0]], dtype=torch.int32)
    x = torch.randn(6, channels, generator=g)
    gate = gate_of(6)
    ext = tv.TreeVerify()
    tv.stage_tree(None)  # chains: row i's parent is row i - 1
    rows = _rows("gdn", shape, params, pools, x, gate, torch.tensor([1, 0], dtype=torch.int32),
                 torch.tensor([0, 3, 6]), state_indices, 6)
    out = _forward(ext, "gdn", rows)
    window = _window(pools["conv"], 3, 0, channels)
    want = _chain_outputs("gdn", shape, params, before[3], window, x, gate, [0, 1, 2])
    assert torch.allclose(out[:3], want, atol=1e-5, rtol=1e-5)
    tv.commit_accepted(torch.tensor([[0, 1, -1], [0, -1, -1]]), torch.tensor([2, 1]))
    assert torch.equal(pools["ssm"][0], before[0])  # the padded request's null slot is never written
    assert not torch.equal(pools["ssm"][4], before[4])


def test_staged_tree_must_cover_the_rows_and_layers_are_checked():
    shape, channels, params, pools, gate_of, g = _setup("gdn", True, seed=2)
    tv.stage_tree(torch.tensor([[-1, 0]]))
    rows = _rows("gdn", shape, params, pools, torch.randn(3, channels, generator=g), gate_of(3),
                 torch.tensor([1], dtype=torch.int32), torch.tensor([0, 3]), STATE_INDICES[:1], 3)
    with pytest.raises(RuntimeError):
        tv.TreeVerify().forward_spec_rows(rows)

    class QwenGatedDeltaNetAttention:
        pass

    class KimiGatedDeltaNetAttention:
        pass

    tv.check_tree_verifiable([QwenGatedDeltaNetAttention()])
    with pytest.raises(RuntimeError, match="KimiGatedDeltaNetAttention"):
        tv.check_tree_verifiable([QwenGatedDeltaNetAttention(), KimiGatedDeltaNetAttention()])
    chain = types.SimpleNamespace(speculative_config=types.SimpleNamespace(method_config={"intensity": "chain_intensity"}))
    tree = types.SimpleNamespace(speculative_config=types.SimpleNamespace(method_config={}))
    assert tv.create_extension(chain) is None
    assert isinstance(tv.create_extension(tree), tv.TreeVerify)
