// Tensor-parallel communication over NVLink peer memory: symmetric buffers shared through CUDA IPC, the reduce that
// completes a row-parallel GEMM (partial sums + residual + the next RMSNorm), and the greedy head's cross-rank
// (max, argmax) exchange.
//
// Each rank owns one buffer of the same layout; peers map it with cudaIpcOpenMemHandle, so a kernel stores into
// (or loads from) another GPU's buffer through a plain pointer. A "channel" is a set of words in the buffer:
//   arrive[2][kMaxRanks]   arrival counters per (parity, source rank); peers add to them with release semantics
//   done                   CTAs of the local reduce that passed the wait (the last one resets the counters)
//   calls                  local call counter; its low bit is the parity the next call uses
// Consecutive calls alternate parity, so a rank may run one call ahead of a slower peer without overwriting data the
// peer still reads: a rank cannot start call n + 2 before every rank has signalled call n + 1, which each does only
// after finishing call n. Every wait is bounded (2 s) and records kErrTimeoutPeer instead of spinning forever.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace e4 {
namespace comm {

constexpr int kMaxRanks = 8;

struct Channel {
  unsigned* arrive;  // local [2][kMaxRanks]
  unsigned* done;
  unsigned* calls;
};

E4_DEV unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
E4_DEV void red_release_sys(unsigned* p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Threads [0, world) wait until arrive[parity][t] >= expect; false after the time limit.
E4_DEV bool wait_arrivals(const Channel& ch, unsigned parity, int world, unsigned expect) {
  bool ok = true;
  if (threadIdx.x < world) {
    const unsigned* a = ch.arrive + parity * kMaxRanks + threadIdx.x;
    if (ld_acquire_sys(a) < expect) {
      const uint64_t t0 = globaltimer();
      while (ld_acquire_sys(a) < expect) {
        if (globaltimer() - t0 > kWaitLimitNs) { ok = false; break; }
      }
    }
  }
  return __syncthreads_and(ok);
}

// One CTA per row: h = residual + sum over ranks (rank order) of the fp32 partials; x = rmsnorm(h) (optional).
__global__ void __launch_bounds__(256) reduce_residual_norm_kernel(
    const float* __restrict__ recv, int world, long slot_stride, int N, const __nv_bfloat16* __restrict__ residual,
    int ldr, const __nv_bfloat16* __restrict__ norm_w, float eps, int offset, __nv_bfloat16* __restrict__ out_h,
    __nv_bfloat16* __restrict__ out_x, Channel ch, unsigned expect, int* err) {
  pdl_wait();
  const unsigned calls = *reinterpret_cast<volatile unsigned*>(ch.calls);
  const unsigned parity = calls & 1u;
  if (!wait_arrivals(ch, parity, world, expect) && threadIdx.x == 0) record_error(err, kErrTimeoutPeer);
  pdl_trigger();
  const int row = blockIdx.x;
  __shared__ float red[32];
  // each thread owns 4-element groups c = threadIdx.x + i * 256 (N % 4 == 0, N <= 8192)
  constexpr int kMax = 8;
  float4 acc[kMax];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMax; ++i) {
    const int c = threadIdx.x + i * 256;
    if (c * 4 >= N) break;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < world; ++r) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(
          recv + (size_t(parity) * world + r) * size_t(slot_stride) + size_t(row) * N) + c);
      s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
    }
    const __nv_bfloat162* rp = reinterpret_cast<const __nv_bfloat162*>(residual + size_t(row) * ldr) + 2 * c;
    const float2 r0 = __bfloat1622float2(rp[0]), r1 = __bfloat1622float2(rp[1]);
    // the residual stream is bf16: round h once, and normalise the rounded values
    const __nv_bfloat162 h0 = __floats2bfloat162_rn(s.x + r0.x, s.y + r0.y);
    const __nv_bfloat162 h1 = __floats2bfloat162_rn(s.z + r1.x, s.w + r1.y);
    __nv_bfloat162* hp = reinterpret_cast<__nv_bfloat162*>(out_h + size_t(row) * N) + 2 * c;
    hp[0] = h0;
    hp[1] = h1;
    const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
    acc[i] = make_float4(f0.x, f0.y, f1.x, f1.y);
    ss = fmaf(f0.x, f0.x, ss); ss = fmaf(f0.y, f0.y, ss); ss = fmaf(f1.x, f1.x, ss); ss = fmaf(f1.y, f1.y, ss);
  }
  if (norm_w != nullptr) {
    float tot = warp_sum(ss);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = tot;
    __syncthreads();
    tot = 0.f;
    for (int i = 0; i < 8; ++i) tot += red[i];
    const float rs = rsqrtf(tot / N + eps);
#pragma unroll
    for (int i = 0; i < kMax; ++i) {
      const int c = threadIdx.x + i * 256;
      if (c * 4 >= N) break;
      const __nv_bfloat162* wp = reinterpret_cast<const __nv_bfloat162*>(norm_w) + 2 * c;
      const float2 w0 = __bfloat1622float2(wp[0]), w1 = __bfloat1622float2(wp[1]);
      const float s0 = offset ? 1.f + w0.x : w0.x, s1 = offset ? 1.f + w0.y : w0.y;
      const float s2 = offset ? 1.f + w1.x : w1.x, s3 = offset ? 1.f + w1.y : w1.y;
      __nv_bfloat162* xp = reinterpret_cast<__nv_bfloat162*>(out_x + size_t(row) * N) + 2 * c;
      xp[0] = __floats2bfloat162_rn(acc[i].x * rs * s0, acc[i].y * rs * s1);
      xp[1] = __floats2bfloat162_rn(acc[i].z * rs * s2, acc[i].w * rs * s3);
    }
  }
  // the last CTA past the wait resets this parity's counters and advances the call counter
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned old = atomicAdd(ch.done, 1u);
    if (old == gridDim.x - 1) {
      for (int r = 0; r < world; ++r) ch.arrive[parity * kMaxRanks + r] = 0u;
      *ch.done = 0u;
      __threadfence();
      atomicAdd(ch.calls, 1u);
    }
  }
}

struct Peers {
  float2* xbuf[kMaxRanks];   // exchange area of every rank: [2][kMaxRanks][max_rows] (value, index as float bits)
  unsigned* arrive[kMaxRanks];  // channel arrive words of every rank
};

// One CTA: publish this rank's (max, argmax + lo) per row to every rank, wait for all ranks, pick the global best
// (ties to the lower vocabulary id, as in the single-GPU head).
__global__ void __launch_bounds__(256) argmax_exchange_kernel(
    const int64_t* __restrict__ ids, const float* __restrict__ val, int T, int lo, int world, int rank, int max_rows,
    Peers peers, Channel ch, int64_t* __restrict__ out_ids, float* __restrict__ out_val, int* err) {
  pdl_wait();
  const unsigned parity = *reinterpret_cast<volatile unsigned*>(ch.calls) & 1u;
  const size_t mine = (size_t(parity) * kMaxRanks + rank) * max_rows;
  for (int j = threadIdx.x; j < T; j += blockDim.x) {
    const float2 e = make_float2(val[j], __int_as_float(int(ids[j]) + lo));
    for (int r = 0; r < world; ++r) peers.xbuf[r][mine + j] = e;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int r = 0; r < world; ++r) red_release_sys(peers.arrive[r] + parity * kMaxRanks + rank, 1u);
  }
  if (!wait_arrivals(ch, parity, world, 1u) && threadIdx.x == 0) record_error(err, kErrTimeoutPeer);
  pdl_trigger();
  const float2* local = peers.xbuf[rank];
  for (int j = threadIdx.x; j < T; j += blockDim.x) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int r = 0; r < world; ++r) {
      const float2 e = __ldcg(local + (size_t(parity) * kMaxRanks + r) * max_rows + j);
      const int i = __float_as_int(e.y);
      if (e.x > best || (e.x == best && i < bi)) { best = e.x; bi = i; }
    }
    out_ids[j] = bi;
    out_val[j] = best;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int r = 0; r < world; ++r) ch.arrive[parity * kMaxRanks + r] = 0u;
    __threadfence();
    atomicAdd(ch.calls, 1u);
  }
}

Channel channel(int64_t base) {
  unsigned* b = reinterpret_cast<unsigned*>(base);
  return Channel{b, b + 2 * kMaxRanks, b + 2 * kMaxRanks + 1};
}

}  // namespace comm

// ---------------------------------------------------------------------------------------------- symmetric buffers
int64_t sym_alloc(int64_t bytes, int64_t device) {
  const at::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, size_t(bytes)));
  C10_CUDA_CHECK(cudaMemset(p, 0, size_t(bytes)));
  return reinterpret_cast<int64_t>(p);
}

void sym_free(int64_t ptr) {
  if (ptr) C10_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr)));
}

torch::Tensor sym_handle(int64_t ptr) {
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)));
  auto t = torch::empty({int64_t(sizeof(h))}, torch::TensorOptions().dtype(torch::kUInt8));
  std::memcpy(t.data_ptr(), &h, sizeof(h));
  return t;
}

int64_t sym_open(const torch::Tensor& handle, int64_t device) {
  TORCH_CHECK(handle.numel() == int64_t(sizeof(cudaIpcMemHandle_t)), "sym_open: bad handle");
  const at::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.contiguous().data_ptr(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void sym_close(int64_t ptr) {
  if (ptr) C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}

// A tensor view of ``numel`` elements at ``ptr + offset`` (no ownership).
torch::Tensor sym_view(int64_t ptr, int64_t offset, int64_t numel, int64_t dtype_code, int64_t device) {
  const auto dtype = dtype_code == 0 ? torch::kFloat32 : (dtype_code == 1 ? torch::kInt32 : torch::kUInt8);
  return torch::from_blob(reinterpret_cast<char*>(ptr) + offset, {numel},
                          torch::TensorOptions().dtype(dtype).device(torch::kCUDA, device));
}

// h, x = reduce(recv partials) + residual, rmsnorm(h) (x only when ``norm_w`` is given).
void tp_reduce(int64_t recv, int64_t world, int64_t slot_stride, const torch::Tensor& residual,
               const c10::optional<torch::Tensor>& norm_w, double eps, bool offset, torch::Tensor out_h,
               c10::optional<torch::Tensor> out_x, int64_t channel, int64_t expect, torch::Tensor err) {
  const at::cuda::CUDAGuard g(residual.device());
  const int T = residual.size(0), N = residual.size(1);
  TORCH_CHECK(N % 4 == 0 && N <= 8192, "tp_reduce: features must be a multiple of 4, at most 8192");
  TORCH_CHECK(residual.stride(1) == 1 && out_h.is_contiguous(), "tp_reduce: row-major tensors expected");
  const bool norm = norm_w.has_value() && norm_w->defined();
  if (T == 0) return;
  C10_CUDA_CHECK(launch_pdl(comm::reduce_residual_norm_kernel, T, 256, 0, at::cuda::getCurrentCUDAStream().stream(),
                            reinterpret_cast<const float*>(recv), int(world), long(slot_stride), N,
                            reinterpret_cast<const __nv_bfloat16*>(residual.data_ptr()), int(residual.stride(0)),
                            norm ? reinterpret_cast<const __nv_bfloat16*>(norm_w->data_ptr()) : nullptr, float(eps),
                            int(offset), reinterpret_cast<__nv_bfloat16*>(out_h.data_ptr()),
                            norm ? reinterpret_cast<__nv_bfloat16*>(out_x->data_ptr()) : nullptr,
                            comm::channel(channel), unsigned(expect), err.data_ptr<int>()));
}

void tp_argmax(const torch::Tensor& ids, const torch::Tensor& val, int64_t lo, const std::vector<int64_t>& xbufs,
               const std::vector<int64_t>& arrives, int64_t rank, int64_t max_rows, int64_t channel,
               torch::Tensor out_ids, torch::Tensor out_val, torch::Tensor err) {
  const at::cuda::CUDAGuard g(ids.device());
  const int world = int(xbufs.size());
  TORCH_CHECK(world <= comm::kMaxRanks && int(arrives.size()) == world, "tp_argmax: 1..8 ranks");
  const int T = ids.size(0);
  TORCH_CHECK(T <= max_rows, "tp_argmax: more rows than the exchange area holds");
  comm::Peers peers{};
  for (int r = 0; r < world; ++r) {
    peers.xbuf[r] = reinterpret_cast<float2*>(xbufs[r]);
    peers.arrive[r] = reinterpret_cast<unsigned*>(arrives[r]);
  }
  C10_CUDA_CHECK(launch_pdl(comm::argmax_exchange_kernel, 1, 256, 0, at::cuda::getCurrentCUDAStream().stream(),
                            ids.data_ptr<int64_t>(), val.data_ptr<float>(), T, int(lo), world, int(rank),
                            int(max_rows), peers, comm::channel(channel), out_ids.data_ptr<int64_t>(),
                            out_val.data_ptr<float>(), err.data_ptr<int>()));
}

}  // namespace e4
