"""The allocation-free GEMM entry point, called through its exported C symbol.

``e4_gemm_bf16_noalloc`` serves callers that cannot allocate device memory (hosts that only lend pre-allocated
buffers, fixed memory budgets, plain C programs without a device allocator): it runs the library's GEMM with its
workspace in a fixed device array. This checks it against the regular entry point on two calls in a row (the second
call reuses the array the first one left behind). The file sorts last so a stop-at-first-failure run has already run
every other test.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from eagle4_b200.ops.build import load

    mod = load()
    lib = ctypes.CDLL(mod.__file__)
    fn = lib.e4_gemm_bf16_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return fn


def _call(fn, x, w, y):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), y.data_ptr(), y.stride(0), x.shape[0], w.shape[0],
              x.shape[1], stream)


def test_noalloc_gemm_matches_regular_entry_point():
    from eagle4_b200.ops import native

    fn = _lib()
    g = torch.Generator(device="cuda").manual_seed(7)
    for T, N, K in ((16, 5120, 6144), (3, 16480, 5120)):  # two calls in a row, different shapes
        x = (torch.randn(T, K, generator=g, device="cuda")).to(torch.bfloat16)
        w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        y = torch.empty(T, N, dtype=torch.bfloat16, device="cuda")
        assert _call(fn, x, w, y) == 0
        want = native.linear(x, w)
        torch.cuda.synchronize()
        err = (y.float() - want.float()).abs().max().item()
        assert err <= 2e-2 * want.float().abs().max().item()


def test_noalloc_gemm_rejects_oversize():
    fn = _lib()
    x = torch.zeros(33, 256, dtype=torch.bfloat16, device="cuda")  # more tokens than the fixed workspace holds
    w = torch.zeros(256, 256, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(33, 256, dtype=torch.bfloat16, device="cuda")
    assert _call(fn, x, w, y) == 1
