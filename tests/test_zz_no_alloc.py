"""The allocation-free GEMM entry point, called through its exported C symbols (declared in ``csrc/e4_noalloc.h``).

``e4_gemm_bf16_noalloc`` is for callers that may not allocate device memory: a host that lends the library only
buffers it allocated itself, a deployment inside a fixed memory budget, a C program with no device allocator. It runs
the library's GEMM with its workspace in a fixed device array. These tests check it on two calls in a row (the second
call finds the array as the first one left it): bitwise against the regular entry point (same kernel, grid and
stream-K cut points), within tolerance against an fp32 product, with device memory in use unchanged across the call
and the kernel's error word zero. The file sorts last, so a stop-at-first-failure run has already run every other
test.
"""

import ctypes
import gc

import pytest
import torch

pytestmark = pytest.mark.gpu

OK, BAD_ARGS = 0, 1


def _lib():
    from eagle4_b200.ops.build import load

    lib = ctypes.CDLL(load().__file__)
    fn = lib.e4_gemm_bf16_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    status = lib.e4_gemm_noalloc_status
    status.restype = ctypes.c_int
    status.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]
    return fn, status


def _call(fn, x, w, y):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), y.data_ptr(), y.stride(0), x.shape[0], w.shape[0],
              x.shape[1], stream)


def _kernel_error(status) -> int:
    word = ctypes.c_int(-1)
    assert status(ctypes.byref(word), torch.cuda.current_stream().cuda_stream) == OK
    return word.value


def test_noalloc_gemm_matches_regular_entry_point():
    from eagle4_b200.ops import native

    fn, status = _lib()
    g = torch.Generator(device="cuda").manual_seed(7)
    cases = [(16, 5120, 6144), (3, 16480, 5120), (32, 1000, 768)]  # calls in a row, different shapes
    operands = []
    for T, N, K in cases:
        x = torch.randn(T, K, generator=g, device="cuda").to(torch.bfloat16)
        w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        y = torch.full((T, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        operands.append((x, w, y, native.linear(x, w)))
    # first call on this device: looks up the array's address (set-up); later calls must allocate nothing
    x, w, y, _ = operands[0]
    assert _call(fn, x, w, y) == OK
    torch.cuda.synchronize()
    want_err = []
    # garbage of earlier tests must not be collected (and freed) between the two readings
    gc.collect()
    gc.disable()
    try:
        for x, w, y, want in operands:
            y.fill_(float("nan"))
            torch.cuda.synchronize()
            torch_before = torch.cuda.memory_allocated()
            free_before, _ = torch.cuda.mem_get_info()
            assert _call(fn, x, w, y) == OK
            torch.cuda.synchronize()
            assert torch.cuda.memory_allocated() == torch_before
            assert torch.cuda.mem_get_info()[0] == free_before
            want_err.append((x, w, y, want, _kernel_error(status)))
    finally:
        gc.enable()
    for x, w, y, want, err_word in want_err:
        assert err_word == 0
        assert torch.equal(y, want), "the allocation-free path must give the regular path's bits"
        ref = x.float() @ w.float().t()
        err = (y.float() - ref).abs().max().item()
        assert err <= 1e-2 * ref.abs().max().item() + 1e-3


def test_noalloc_gemm_rejects_oversize():
    fn, _ = _lib()
    x = torch.zeros(33, 256, dtype=torch.bfloat16, device="cuda")  # more tokens than the fixed workspace holds
    w = torch.zeros(256, 256, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(33, 256, dtype=torch.bfloat16, device="cuda")
    assert _call(fn, x, w, y) == BAD_ARGS
    wide = torch.zeros(128 * 4096 + 1, 64, dtype=torch.bfloat16, device="cuda")  # more weight tiles than it counts
    assert _call(fn, x[:1, :64].contiguous(), wide, torch.empty(1, wide.shape[0], dtype=torch.bfloat16,
                                                               device="cuda")) == BAD_ARGS
