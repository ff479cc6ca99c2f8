"""A peer-memory wait that nothing satisfies ends after its one-second limit with an error status, and the context
stays usable (the bounded waits of the fused collectives, exercised without faulting or hanging the GPU)."""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu

K_ERR_TIMEOUT_PEER = 5


def test_fused_allreduce_without_a_peer_times_out_and_reports():
    """The fused GEMM + all-reduce told that a second rank exists whose partials never arrive (both ranks' areas are
    this GPU's own buffer, and nothing writes rank 1's flags): each wait ends after one second, the kernel records
    the peer time-out, counts the missing partial as zero, and the context stays usable."""
    from eagle4_b200.ops import native
    from eagle4_b200.parallel import tp as tpm

    C = native._C
    dev = torch.device("cuda")
    n, k, rows, ldp = 256, 256, 2, 256
    part_bytes = 2 * tpm.MAX_RANKS * tpm.TP_ROWS * ldp * 2
    gath_bytes = 2 * tpm.TP_ROWS * ldp * 2
    base = C.sym_alloc(tpm._PART + part_bytes + gath_bytes, torch.cuda.current_device())  # zeroed: no flag set
    try:
        err = native.error_word(dev)
        err.zero_()
        x = torch.randn(rows, k, device=dev).to(torch.bfloat16)
        w = (torch.randn(n, k, device=dev) * 0.05).to(torch.bfloat16)
        res = torch.randn(rows, n, device=dev).to(torch.bfloat16)
        h = torch.empty_like(res)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        C.gemm_allreduce(x, w, res, h, [base + tpm._PART] * 2, [base + tpm._PART + part_bytes] * 2,
                         [base + tpm._FLAGS] * 2, base + tpm._CTRL_GEMM, ldp, 0, 1 << 30)
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        assert int(err.item()) == K_ERR_TIMEOUT_PEER
        err.zero_()
        assert 0.5 < waited < 20.0
        want = res.float() + x.float() @ w.float().t()  # rank 1's missing partial counted as zero
        torch.testing.assert_close(h.float(), want, atol=0.05, rtol=0.02)
        # the context still works
        y = native.linear(x, w)
        torch.cuda.synchronize()
        assert torch.isfinite(y.float()).all()
    finally:
        torch.cuda.synchronize()
        C.sym_free(base)
