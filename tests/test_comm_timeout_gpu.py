"""A peer-memory wait that nothing satisfies ends after its one-second limit with an error status, and the context
stays usable (the bounded waits of the fused collectives, exercised without faulting or hanging the GPU)."""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu

K_ERR_TIMEOUT_PEER = 5


def test_reduce_without_partials_times_out_and_reports():
    from eagle4_b200.ops import native

    C = native._C
    dev = torch.device("cuda")
    n, rows = 1024, 2
    slot = rows * n
    base = C.sym_alloc(4096 + 2 * slot * 8, torch.cuda.current_device())  # zeroed: no pair carries this tag
    try:
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        res = torch.randn(rows, n, device=dev).to(torch.bfloat16)
        h = torch.empty_like(res)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        C.tp_reduce(base + 4096, 1, slot, res, None, 1e-6, False, h, None, base, err)
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        assert int(err.item()) == K_ERR_TIMEOUT_PEER
        assert 0.5 < waited < 10.0
        torch.testing.assert_close(h.float(), res.float())  # missing partials counted as zero
        # the context still works
        x = torch.randn(4, 256, device=dev).to(torch.bfloat16)
        w = torch.randn(256, 256, device=dev).to(torch.bfloat16)
        y = native.linear(x, w)
        torch.cuda.synchronize()
        assert torch.isfinite(y.float()).all()
    finally:
        torch.cuda.synchronize()
        C.sym_free(base)
