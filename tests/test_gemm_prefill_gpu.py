"""Prefill GEMM launches (whole (weight tile, 256-token chunk) units, no split tiles) against an fp32 product and the
regular stream-K launches, for every epilogue a prefill uses, including the folded norm and a partial last chunk."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _operands(T, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(T, K, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g, device="cuda") * K ** -0.5).to(torch.bfloat16)
    r = torch.randn(T, N, generator=g, device="cuda").to(torch.bfloat16)
    return x, w, r


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max()).item()


@pytest.mark.parametrize("T,N,K", [(1024, 5120, 6144), (700, 16480, 5120), (256, 34816, 5120), (1500, 4096, 2048)])
def test_prefill_units_match_fp32_and_the_regular_path(T, N, K):
    from eagle4_b200.ops import native

    x, w, r = _operands(T, N, K, T + N)
    ref = x.float() @ w.float().t()
    with native.prefill_gemms():
        plain = native.linear(x, w)
        resid = native.linear_residual(x, w, r)
        relu2 = native.linear_relu2(x, w)
    assert _rel(plain, ref) < 1e-2
    assert _rel(resid, ref + r.float()) < 1e-2
    assert _rel(relu2, torch.relu(ref) ** 2) < 2e-2
    assert _rel(plain, native.linear(x, w)) < 1e-2  # the regular launches: same products, another K split
    native.check_errors()


def test_prefill_units_swiglu_with_folded_norm():
    from eagle4_b200 import ops
    from eagle4_b200.ops import native

    T, F, K = 600, 4096, 5120
    x, _, _ = _operands(T, 2 * F, K, 7)
    g = torch.Generator(device="cuda").manual_seed(8)
    gate = (torch.randn(F, K, generator=g, device="cuda") * K ** -0.5).to(torch.bfloat16)
    up = (torch.randn(F, K, generator=g, device="cuda") * K ** -0.5).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(K, generator=g, device="cuda")).to(torch.bfloat16)
    from eagle4_b200.models.weights import interleave_gate_up

    wgu = ops.fold_norm_weight(interleave_gate_up(gate, up), nw, False)
    xn = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6) * nw.float()
    ref = torch.nn.functional.silu(xn @ gate.float().t()) * (xn @ up.float().t())
    with native.prefill_gemms():
        got = native.linear_swiglu(x, wgu, 1e-6)
    assert _rel(got, ref) < 2e-2
    assert _rel(got, native.linear_swiglu(x, wgu, 1e-6)) < 1e-2
    native.check_errors()


def test_prefill_mode_falls_back_below_one_unit_per_sm():
    """Few units (small N, one chunk): the launch keeps the regular partition, bit-identical to it."""
    from eagle4_b200.ops import native

    x, w, _ = _operands(100, 1024, 2048, 3)
    with native.prefill_gemms():
        a = native.linear(x, w)
    assert torch.equal(a, native.linear(x, w))
