// Allocation-free GEMM entry point of the eagle4_b200 library. This has no counterpart in the reference.
//
// Who needs it: callers that are not allowed to allocate device memory. An inference host may lend this library only
// buffers it allocated itself and forbid allocation while it serves; some deployments run inside a fixed memory
// budget that must not grow; a plain C program may link the library without any device allocator at all. The
// library's regular GEMM takes its stream-K workspace (partial tiles, arrival counters, error word) from
// allocator-backed buffers. These functions run the same kernel with that workspace in one fixed array in device
// memory instead, and call no cudaMalloc, cudaFree or allocating library routine.
//
// Limits (calls outside them return E4_NOALLOC_BAD_ARGS and launch nothing):
//   * T <= E4_NOALLOC_MAX_TOKENS tokens per call;
//   * N <= 128 * E4_NOALLOC_MAX_TILES weight rows;
//   * x and w 16-byte aligned, with row strides (ldx, ldw) that are multiples of 8 elements.
// The array holds E4_NOALLOC_SCRATCH_BYTES (about 5.3 MB) on every GPU that loads the library, until the process
// exits.
//
// Set-up: the first call on a device, with that device current, looks up the array's device address and sets the
// kernel's shared-memory limit. Make that first call before any stream capture.
//
// Sharing: every call uses the one array. Each call clears the counters and the error word it needs before its
// kernel starts, so two calls that overlap on the GPU (different streams, or different host threads on one device)
// race on the array; the caller must serialise them.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

enum {
  E4_NOALLOC_OK = 0,
  E4_NOALLOC_BAD_ARGS = 1,   // shape, stride or alignment outside the limits above
  E4_NOALLOC_CUDA_ERROR = 2, // a CUDA runtime call failed (set-up, launch or copy)
  E4_NOALLOC_MAX_TOKENS = 32,
  E4_NOALLOC_MAX_TILES = 4096,
};

// Bytes of the fixed device array.
#define E4_NOALLOC_SCRATCH_BYTES (2ull * 160 * 32 * 128 * 4 + 4096 * 4 + 256)

// Y[T, N] = X[T, K] . W[N, K]^T on ``stream`` (a cudaStream_t; 0 for the legacy stream). bf16 operands and output,
// fp32 accumulation, row-major with leading dimensions in elements. Returns E4_NOALLOC_OK once the kernel is queued.
// The kernel's own failures (a bounded wait that ran out) are reported by e4_gemm_noalloc_status.
int e4_gemm_bf16_noalloc(const void* x, int ldx, const void* w, int ldw, void* y, int ldy, int T, int N, int K,
                         void* stream);

// Copies the error word of the last call queued on ``stream`` into ``*kernel_error`` after waiting for ``stream``:
// 0 when the kernel finished normally, else the library's error code (1-3: a pipeline wait ran out). Returns
// E4_NOALLOC_OK, or E4_NOALLOC_CUDA_ERROR if the copy failed. Allocates nothing.
int e4_gemm_noalloc_status(int* kernel_error, void* stream);

#ifdef __cplusplus
}
#endif
