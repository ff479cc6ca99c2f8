// Tensor-parallel communication over NVLink peer memory: the symmetric buffers shared through CUDA IPC and the
// greedy head's cross-rank (max, argmax) exchange. (The row-parallel projections' all-reduce is fused into the GEMM:
// see the kAllReduce epilogue in gemm.cu.)
//
// Each rank owns one buffer of the same layout; peers map it with cudaIpcOpenMemHandle, so a kernel stores into
// another GPU's buffer through a plain pointer. The exchange's entries travel as (value, tag) pairs written by single
// aligned 8-byte stores: a pair lands whole, and the reader knows it is this call's when the tag equals the call
// counter + 1, so no fence or flag sits between the producer's stores and the consumer's loads. A channel's words:
//   done    CTAs of the exchange that have finished (the last one advances the call counter)
//   calls   local call counter; its low bit selects the buffer half of the call, calls + 1 is the call's tag
// Consecutive calls alternate halves, so a rank may run one call ahead of a slower peer without overwriting entries
// the peer still reads. A launch's waits share one 1 s deadline per thread; past it the kernel records
// kErrTimeoutPeer and finishes with what it has instead of spinning.
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

// The vocabulary-parallel greedy head's reduce and exchange in one launch. A warp per token row: reduce this rank's
// per-tile (max, argmax) partials of the LM-head GEMM (ties to the lower id), publish (max, argmax + lo) to every
// rank as one tagged 16-byte pair of pairs ((max, tag), (id, tag)), then pick the global best from every rank's
// entries (ties to the lower vocabulary id, as in the single-GPU head). Partials: for token chunk c of 256 rows,
// entry (tile, j) at val[c * 256 * n_tiles + tile * tc + j] (tc: the chunk's rows). Exchange area of each rank:
// [2 halves][kMaxRanks][max_rows] entries of 16 bytes.
constexpr int kExchangeWarps = 8;
__global__ void __launch_bounds__(kExchangeWarps * 32) argmax_exchange_kernel(
    const float* __restrict__ pval, const int* __restrict__ pidx, int n_tiles, int T, int lo, int world, int rank,
    int max_rows, const __grid_constant__ Peers peers, Channel ch, int64_t* __restrict__ out_ids,
    float* __restrict__ out_val, int* err) {
  pdl_wait();
  pdl_trigger();
  const unsigned calls = *reinterpret_cast<volatile unsigned*>(ch.calls);
  const unsigned half = calls & 1u, tag = calls + 1u;
  const int lane = threadIdx.x & 31;
  const int j = blockIdx.x * kExchangeWarps + (threadIdx.x >> 5);
  bool ok = true;
  if (j < T) {
    const int chunk = j / 256, jj = j % 256;
    const int tc = min(256, T - chunk * 256);
    const float* v = pval + size_t(chunk) * 256 * n_tiles;
    const int* ix = pidx + size_t(chunk) * 256 * n_tiles;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = lane; i < n_tiles; i += 32) {
      const float ov = v[size_t(i) * tc + jj];
      const int oi = ix[size_t(i) * tc + jj];
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    const size_t mine = (size_t(half) * kMaxRanks + rank) * max_rows + j;
    if (lane < world) {
      uint2* dst = peers.xbuf[lane] + 2 * mine;
      st_volatile_v2(dst, __float_as_uint(best), tag);
      st_volatile_v2(dst + 1, unsigned(bi + lo), tag);
    }
    // lane r reads rank r's entry; the merge order does not matter (a strict order: larger value, then lower id)
    uint4 e = make_uint4(0u, 0u, 0u, 0u);
    uint64_t deadline = 0;
    const uint2* local = peers.xbuf[rank];
    float x = -INFINITY;
    int xi = 0x7fffffff;
    if (lane < world) {
      const uint2* src = local + 2 * ((size_t(half) * kMaxRanks + lane) * max_rows + j);
      e = ld_volatile_v4(src);
      if (settle(src, tag, e, deadline)) {
        x = __uint_as_float(e.x);
        xi = int(e.z);
      } else {
        ok = false;  // a rank that never answered offers no candidate
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, x, o);
      const int oi = __shfl_xor_sync(0xffffffffu, xi, o);
      if (ov > x || (ov == x && oi < xi)) { x = ov; xi = oi; }
    }
    if (lane == 0) {
      out_ids[j] = xi;
      out_val[j] = x;
    }
  }
  if (!__all_sync(0xffffffffu, ok) && lane == 0) record_error(err, kErrTimeoutPeer);
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

// Greedy ids over the whole vocabulary from every rank's LM-head partials (``val`` / ``idx``: this rank's per-tile
// (max, argmax) of the kArgmax GEMM epilogue over its vocabulary rows [lo, lo + rows)).
void tp_argmax(const torch::Tensor& val, const torch::Tensor& idx, int64_t n_tiles, int64_t lo,
               const std::vector<int64_t>& xbufs, int64_t rank, int64_t max_rows, int64_t channel,
               torch::Tensor out_ids, torch::Tensor out_val, torch::Tensor err) {
  const at::cuda::CUDAGuard g(val.device());
  const int world = int(xbufs.size());
  TORCH_CHECK(world <= comm::kMaxRanks, "tp_argmax: 1..8 ranks");
  const int T = out_ids.size(0);
  TORCH_CHECK(T <= max_rows, "tp_argmax: more rows than the exchange area holds");
  if (T == 0) return;
  comm::Peers peers{};
  for (int r = 0; r < world; ++r) peers.xbuf[r] = reinterpret_cast<uint2*>(xbufs[r]);
  const int grid = (T + comm::kExchangeWarps - 1) / comm::kExchangeWarps;
  C10_CUDA_CHECK(launch_pdl(comm::argmax_exchange_kernel, grid, comm::kExchangeWarps * 32, 0,
                            at::cuda::getCurrentCUDAStream().stream(), val.data_ptr<float>(), idx.data_ptr<int>(),
                            int(n_tiles), T, int(lo), world, int(rank), int(max_rows), peers, comm::channel(channel),
                            out_ids.data_ptr<int64_t>(), out_val.data_ptr<float>(), err.data_ptr<int>()));
}

}  // namespace e4
