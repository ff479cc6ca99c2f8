// Tensor-parallel communication over NVLink peer memory: symmetric buffers shared through CUDA IPC, the reduce that
// completes a row-parallel GEMM (partial sums + residual + the next RMSNorm), and the greedy head's cross-rank
// (max, argmax) exchange.
//
// Each rank owns one buffer of the same layout; peers map it with cudaIpcOpenMemHandle, so a kernel stores into
// another GPU's buffer through a plain pointer. Data travel as (value, tag) pairs written by single aligned 8-byte
// stores: a pair lands whole, and the reader knows it is this call's when the tag equals the call counter + 1. So no
// fence, flag or counter sits between the producer's stores and the consumer's loads, and a consumer starts on the
// elements that have landed while the rest are in flight. A channel's words in the buffer:
//   done    CTAs of the local reduce that have finished (the last one advances the call counter)
//   calls   local call counter; its low bit selects the buffer half of the call, calls + 1 is the call's tag
// Consecutive calls alternate halves, so a rank may run one call ahead of a slower peer without overwriting data the
// peer still reads: a rank cannot finish call n + 1 (and so start writing call n + 2) before every rank has written
// its call n + 1 data, which each does only after finishing call n. A launch's waits share one 1 s deadline per thread; past it the
// kernel records kErrTimeoutPeer and finishes with what it has (zeros for missing partials) instead of spinning.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace e4 {
namespace comm {

constexpr int kMaxRanks = 8;

struct Peers {
  uint2* xbuf[kMaxRanks];  // exchange area of every rank
};

struct Channel {
  unsigned* done;
  unsigned* calls;
};

E4_DEV uint4 ld_volatile_v4(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p) : "memory");
  return v;
}
E4_DEV uint2 ld_volatile_v2(const void* p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}
E4_DEV void st_volatile_v2(void* p, unsigned a, unsigned b) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(a), "r"(b) : "memory");
}

constexpr uint64_t kPeerWaitNs = 1000000000ull;  // 1 s: one deadline for all of a thread's waits in a launch

// Re-reads two consecutive (value, tag) pairs until both carry ``tag``; false (v unchanged) once the thread's
// deadline has passed. ``deadline`` is 0 until the first wait of the launch sets it.
E4_DEV bool settle(const uint2* p, unsigned tag, uint4& v, uint64_t& deadline) {
  if (v.y == tag && v.w == tag) return true;
  if (deadline == 0) deadline = globaltimer() + kPeerWaitNs;
  do {
    if (globaltimer() > deadline) return false;
    v = ld_volatile_v4(p);
  } while (v.y != tag || v.w != tag);
  return true;
}

// One CTA per row: h = residual + sum over ranks (rank order) of the fp32 partials; x = rmsnorm(h) (optional).
// Each thread owns the 2-element groups c = threadIdx.x + i * kReduceThreads, i < G (N even, N <= 2 * G * 1024).
// Its G x W pair loads are issued in batches of 8 before any is checked, so a batch costs one memory latency;
// pairs still in flight are re-read until their tag matches. Sums run in rank order on every rank.
constexpr int kReduceThreads = 1024;
template <int W, int G>
__global__ void __launch_bounds__(kReduceThreads) reduce_residual_norm_kernel(
    const uint2* __restrict__ recv, long slot_stride, int N, const __nv_bfloat16* __restrict__ residual, int ldr,
    const __nv_bfloat16* __restrict__ norm_w, float eps, int offset, __nv_bfloat16* __restrict__ out_h,
    __nv_bfloat16* __restrict__ out_x, Channel ch, int* err) {
  constexpr int kLoads = W * G, kBatch = 8;
  pdl_wait();
  pdl_trigger();  // the next kernel's prologue may start; anything it reads of ours comes after its own wait
  const unsigned calls = *reinterpret_cast<volatile unsigned*>(ch.calls);
  const unsigned half = calls & 1u, tag = calls + 1u;
  const int row = blockIdx.x;
  __shared__ float red[kReduceThreads / 32];
  const uint2* base = recv + size_t(half) * W * size_t(slot_stride) + size_t(row) * N;
  float2 sum[G];
#pragma unroll
  for (int i = 0; i < G; ++i) sum[i] = make_float2(0.f, 0.f);
  bool ok = true;
  uint64_t deadline = 0;
#pragma unroll
  for (int b0 = 0; b0 < kLoads; b0 += kBatch) {
    uint4 v[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int i = (b0 + k) / W, r = (b0 + k) % W, c = threadIdx.x + i * kReduceThreads;
      if (b0 + k < kLoads && c * 2 < N) v[k] = ld_volatile_v4(base + size_t(r) * slot_stride + 2 * c);
    }
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int i = (b0 + k) / W, r = (b0 + k) % W, c = threadIdx.x + i * kReduceThreads;
      if (b0 + k < kLoads && c * 2 < N) {
        if (!settle(base + size_t(r) * slot_stride + 2 * c, tag, v[k], deadline)) {
          ok = false;
          v[k] = make_uint4(0u, 0u, 0u, 0u);  // a missing partial counts as zero
        }
        sum[i].x += __uint_as_float(v[k].x);
        sum[i].y += __uint_as_float(v[k].z);
      }
    }
  }
  float2 acc[G];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < G; ++i) {
    const int c = threadIdx.x + i * kReduceThreads;
    if (c * 2 >= N) break;
    const float2 rv = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(residual + size_t(row) * ldr)[c]);
    // the residual stream is bf16: round h once, and normalise the rounded values
    const __nv_bfloat162 h = __floats2bfloat162_rn(sum[i].x + rv.x, sum[i].y + rv.y);
    reinterpret_cast<__nv_bfloat162*>(out_h + size_t(row) * N)[c] = h;
    acc[i] = __bfloat1622float2(h);
    ss = fmaf(acc[i].x, acc[i].x, ss);
    ss = fmaf(acc[i].y, acc[i].y, ss);
  }
  if (!ok) record_error(err, kErrTimeoutPeer);
  if (norm_w != nullptr) {
    float tot = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = tot;
    __syncthreads();
    tot = 0.f;
#pragma unroll
    for (int w = 0; w < kReduceThreads / 32; ++w) tot += red[w];
    const float rs = rsqrtf(tot / N + eps);
#pragma unroll
    for (int i = 0; i < G; ++i) {
      const int c = threadIdx.x + i * kReduceThreads;
      if (c * 2 >= N) break;
      const float2 wv = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(norm_w)[c]);
      const float s0 = offset ? 1.f + wv.x : wv.x, s1 = offset ? 1.f + wv.y : wv.y;
      reinterpret_cast<__nv_bfloat162*>(out_x + size_t(row) * N)[c] =
          __floats2bfloat162_rn(acc[i].x * rs * s0, acc[i].y * rs * s1);
    }
  }
  // the last CTA to finish advances the call counter (every CTA read it above)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(ch.done, 1u) == gridDim.x - 1) {
      *ch.done = 0u;
      __threadfence();
      atomicAdd(ch.calls, 1u);
    }
  }
}

// One CTA: publish this rank's (max, argmax + lo) per row to every rank as one tagged 16-byte pair of pairs
// ((max, tag), (id, tag)), then pick the global best from every rank's entries (ties to the lower vocabulary id,
// as in the single-GPU head). Exchange area of each rank: [2 halves][kMaxRanks][max_rows] entries of 16 bytes.
__global__ void __launch_bounds__(256) argmax_exchange_kernel(
    const int64_t* __restrict__ ids, const float* __restrict__ val, int T, int lo, int world, int rank, int max_rows,
    const __grid_constant__ Peers peers, Channel ch, int64_t* __restrict__ out_ids, float* __restrict__ out_val,
    int* err) {
  pdl_wait();
  pdl_trigger();
  const unsigned calls = *reinterpret_cast<volatile unsigned*>(ch.calls);
  const unsigned half = calls & 1u, tag = calls + 1u;
  const size_t mine = (size_t(half) * kMaxRanks + rank) * max_rows;
  for (int j = threadIdx.x; j < T; j += blockDim.x) {
    const unsigned v = __float_as_uint(val[j]), i = unsigned(int(ids[j]) + lo);
    for (int r = 0; r < world; ++r) {
      uint2* dst = peers.xbuf[r] + 2 * (mine + j);
      st_volatile_v2(dst, v, tag);
      st_volatile_v2(dst + 1, i, tag);
    }
  }
  bool ok = true;
  uint64_t deadline = 0;
  const uint2* local = peers.xbuf[rank];
  for (int j = threadIdx.x; j < T; j += blockDim.x) {
    uint4 e[kMaxRanks];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < world) e[r] = ld_volatile_v4(local + 2 * ((size_t(half) * kMaxRanks + r) * max_rows + j));
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r >= world) break;
      if (!settle(local + 2 * ((size_t(half) * kMaxRanks + r) * max_rows + j), tag, e[r], deadline)) {
        ok = false;
        continue;  // a rank that never answered offers no candidate
      }
      const float x = __uint_as_float(e[r].x);
      const int i = int(e[r].z);
      if (x > best || (x == best && i < bi)) { best = x; bi = i; }
    }
    out_ids[j] = bi;
    out_val[j] = best;
  }
  if (!ok) record_error(err, kErrTimeoutPeer);
  __syncthreads();
  if (threadIdx.x == 0) atomicAdd(ch.calls, 1u);
}

Channel channel(int64_t base) {
  unsigned* b = reinterpret_cast<unsigned*>(base);
  return Channel{b, b + 1};
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
               c10::optional<torch::Tensor> out_x, int64_t channel, torch::Tensor err) {
  const at::cuda::CUDAGuard g(residual.device());
  const int T = residual.size(0), N = residual.size(1);
  TORCH_CHECK(N % 2 == 0 && N <= 8192, "tp_reduce: features must be even, at most 8192");
  TORCH_CHECK(world == 1 || world == 2 || world == 4 || world == 8, "tp_reduce: 1, 2, 4 or 8 ranks");
  TORCH_CHECK(residual.stride(1) == 1 && out_h.is_contiguous(), "tp_reduce: row-major tensors expected");
  const bool norm = norm_w.has_value() && norm_w->defined();
  if (T == 0) return;
  auto launch = [&](auto kernel) {
    C10_CUDA_CHECK(launch_pdl(kernel, T, comm::kReduceThreads, 0, at::cuda::getCurrentCUDAStream().stream(),
                              reinterpret_cast<const uint2*>(recv), long(slot_stride), N,
                              reinterpret_cast<const __nv_bfloat16*>(residual.data_ptr()), int(residual.stride(0)),
                              norm ? reinterpret_cast<const __nv_bfloat16*>(norm_w->data_ptr()) : nullptr,
                              float(eps), int(offset), reinterpret_cast<__nv_bfloat16*>(out_h.data_ptr()),
                              norm ? reinterpret_cast<__nv_bfloat16*>(out_x->data_ptr()) : nullptr,
                              comm::channel(channel), err.data_ptr<int>()));
  };
  const int groups = (N / 2 + comm::kReduceThreads - 1) / comm::kReduceThreads;  // 1..4
  auto by_groups = [&](auto w_tag) {
    constexpr int W = decltype(w_tag)::value;
    switch (groups) {
      case 1: launch(comm::reduce_residual_norm_kernel<W, 1>); break;
      case 2: launch(comm::reduce_residual_norm_kernel<W, 2>); break;
      case 3: launch(comm::reduce_residual_norm_kernel<W, 3>); break;
      default: launch(comm::reduce_residual_norm_kernel<W, 4>); break;
    }
  };
  switch (world) {
    case 1: by_groups(std::integral_constant<int, 1>{}); break;
    case 2: by_groups(std::integral_constant<int, 2>{}); break;
    case 4: by_groups(std::integral_constant<int, 4>{}); break;
    default: by_groups(std::integral_constant<int, 8>{}); break;
  }
}

void tp_argmax(const torch::Tensor& ids, const torch::Tensor& val, int64_t lo, const std::vector<int64_t>& xbufs,
               int64_t rank, int64_t max_rows, int64_t channel, torch::Tensor out_ids, torch::Tensor out_val,
               torch::Tensor err) {
  const at::cuda::CUDAGuard g(ids.device());
  const int world = int(xbufs.size());
  TORCH_CHECK(world <= comm::kMaxRanks, "tp_argmax: 1..8 ranks");
  const int T = ids.size(0);
  TORCH_CHECK(T <= max_rows, "tp_argmax: more rows than the exchange area holds");
  comm::Peers peers{};
  for (int r = 0; r < world; ++r) peers.xbuf[r] = reinterpret_cast<uint2*>(xbufs[r]);
  C10_CUDA_CHECK(launch_pdl(comm::argmax_exchange_kernel, 1, 256, 0, at::cuda::getCurrentCUDAStream().stream(),
                            ids.data_ptr<int64_t>(), val.data_ptr<float>(), T, int(lo), world, int(rank),
                            int(max_rows), peers, comm::channel(channel), out_ids.data_ptr<int64_t>(),
                            out_val.data_ptr<float>(), err.data_ptr<int>()));
}

}  // namespace e4
