// Latent ReLU^2 MoE of EAGLE-4 Nemotron-class drafts: the routed experts' MLPs over (token, expert) pairs.
//
// A draft step routes T rows to k experts each (P = T k pairs). moe_route_kernel buckets the pairs by expert (counts,
// offsets, the list of experts that received any pair, and each expert's pairs); then one grouped GEMV launch per
// projection: CTA (active expert s, tile of RT output rows) streams that expert's RT weight rows once (16-byte loads)
// and applies them to all of the expert's pairs, whose input rows are staged in shared memory kPairChunk at a time.
//   up:    h[p, i]  = bf16(relu(up_e[i, :] . latent[t_p, :])^2)     (latent = fc1_latent_proj(x), [T, L])
//   down:  y[p, l]  = down_e[l, :] . h[p, :]                        (fp32)
//   mix:   out[t, l] = bf16(sum_j w[t, j] y[t k + j, l])            (j in routing order)
// Every dot product is a lane-ordered partial sum followed by a fixed xor-butterfly, and the mix sums a token's k
// terms in routing order, so a row's result never depends on which other rows share the launch (batch invariance).
// Reference: eagle_harness/sglang/models/llama_eagle4.py:125-145 (build_latent_moe) and its test
// tests/test_eagle4_model.py:370-392 (the block expert by expert).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace e4 {
namespace {

constexpr int kRouteThreads = 1024;
constexpr int kMaxExperts = 1024;
constexpr int kGemvRows = 32;    // output rows per CTA
constexpr int kPairChunk = 16;   // pairs staged in shared memory at a time
constexpr int kGemvThreads = 256;

// Exclusive scan of one value per thread over a 1024-thread block (warp shuffles, then the warp totals).
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = lane < (blockDim.x >> 5) ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += u;
    }
    warp_tot[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  const int before = warp ? warp_tot[warp - 1] : 0;
  __syncthreads();
  return before + incl - v;
}

// One CTA: bucket the P pairs by expert. offsets[E + 1], active[n_active] (experts with pairs, ascending),
// pairs[P] (pair indices grouped by expert; the order inside an expert's group is arbitrary and does not matter).
__global__ void __launch_bounds__(kRouteThreads) moe_route_kernel(const int* __restrict__ chosen, int P, int E,
                                                                  int* __restrict__ offsets, int* __restrict__ active,
                                                                  int* __restrict__ n_active, int* __restrict__ pairs) {
  pdl_wait();
  pdl_trigger();
  __shared__ int cnt[kMaxExperts], cur[kMaxExperts], warp_tot[32];
  const int t = threadIdx.x;
  for (int e = t; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int p = t; p < P; p += blockDim.x) {
    const int e = chosen[p];
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  // experts are scanned in blocks of 1024 (E <= kMaxExperts = one block)
  const int c = t < E ? cnt[t] : 0;
  const int off = block_exclusive_scan(c, warp_tot);
  const int act = block_exclusive_scan(c > 0 ? 1 : 0, warp_tot);
  if (t < E) {
    offsets[t] = off;
    cur[t] = off;
    if (c > 0) active[act] = t;
    if (t == E - 1) {
      offsets[E] = off + c;
      *n_active = act + (c > 0 ? 1 : 0);
    }
  }
  __syncthreads();
  for (int p = t; p < P; p += blockDim.x) {
    const int e = chosen[p];
    if (e >= 0 && e < E) pairs[atomicAdd(&cur[e], 1)] = p;
  }
}

// Grouped GEMV: CTA (active slot s, row tile) computes out[p, r] for every pair p of expert e = active[s] and rows
// r of its tile: dot(W[e, r, :K], in[row_of(p), :K]). kUp: in row = pair / k (a latent row), out = bf16(relu^2) at
// [P, N]; otherwise in row = pair (an h row), out fp32 at [P, N].
template <bool kUp>
__global__ void __launch_bounds__(kGemvThreads) moe_gemv_kernel(const __nv_bfloat16* __restrict__ in, int k,
                                                                 const int* __restrict__ offsets,
                                                                 const int* __restrict__ active,
                                                                 const int* __restrict__ n_active,
                                                                 const int* __restrict__ pairs,
                                                                 const __nv_bfloat16* __restrict__ W, int N, int K,
                                                                 void* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) float moe_in[];  // [kPairChunk][K]
  const int s = blockIdx.x;
  if (s >= *n_active) return;
  const int e = active[s];
  const int r0 = blockIdx.y * kGemvRows;
  const int p0 = offsets[e], np = offsets[e + 1] - p0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kRowsPerWarp = kGemvRows / (kGemvThreads / 32);
  const int pieces = K / 8;  // 16-byte pieces of a row
  const __nv_bfloat16* We = W + size_t(e) * N * K;
  for (int c0 = 0; c0 < np; c0 += kPairChunk) {
    const int cn = min(kPairChunk, np - c0);
    __syncthreads();
    for (int i = threadIdx.x; i < cn * pieces; i += blockDim.x) {
      const int c = i / pieces, q = i % pieces;
      const int pair = pairs[p0 + c0 + c];
      const int row = kUp ? pair / k : pair;
      const uint4 raw = *reinterpret_cast<const uint4*>(in + size_t(row) * K + 8 * q);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
      float* dst = moe_in + c * K + 8 * q;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h2[j]);
        dst[2 * j] = f.x;
        dst[2 * j + 1] = f.y;
      }
    }
    __syncthreads();
    for (int rr = 0; rr < kRowsPerWarp; ++rr) {
      const int r = r0 + warp * kRowsPerWarp + rr;
      if (r >= N) break;
      const __nv_bfloat16* wr = We + size_t(r) * K;
      float acc[kPairChunk];
#pragma unroll
      for (int c = 0; c < kPairChunk; ++c) acc[c] = 0.f;
      // lane l takes pieces l, l + 32, ...: eight weights per piece against each staged input row
      for (int q = lane; q < pieces; q += 32) {
        const uint4 raw = *reinterpret_cast<const uint4*>(wr + 8 * q);
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
        float wv[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h2[j]);
          wv[2 * j] = f.x;
          wv[2 * j + 1] = f.y;
        }
#pragma unroll
        for (int c = 0; c < kPairChunk; ++c) {
          if (c < cn) {
            const float4 a = *reinterpret_cast<const float4*>(moe_in + c * K + 8 * q);
            const float4 b = *reinterpret_cast<const float4*>(moe_in + c * K + 8 * q + 4);
            float sacc = acc[c];
            sacc = fmaf(wv[0], a.x, sacc);
            sacc = fmaf(wv[1], a.y, sacc);
            sacc = fmaf(wv[2], a.z, sacc);
            sacc = fmaf(wv[3], a.w, sacc);
            sacc = fmaf(wv[4], b.x, sacc);
            sacc = fmaf(wv[5], b.y, sacc);
            sacc = fmaf(wv[6], b.z, sacc);
            sacc = fmaf(wv[7], b.w, sacc);
            acc[c] = sacc;
          }
        }
      }
#pragma unroll
      for (int c = 0; c < kPairChunk; ++c) {
        if (c < cn) {
          const float v = warp_sum(acc[c]);
          if (lane == 0) {
            const int pair = pairs[p0 + c0 + c];
            if (kUp) {
              const float a = fmaxf(v, 0.f);
              reinterpret_cast<__nv_bfloat16*>(out)[size_t(pair) * N + r] = __float2bfloat16(a * a);
            } else {
              reinterpret_cast<float*>(out)[size_t(pair) * N + r] = v;
            }
          }
        }
      }
    }
  }
}

// out[t, l] = bf16(sum_j w[t, j] y[t k + j, l]) with j in routing order.
__global__ void moe_mix_kernel(const float* __restrict__ y, const float* __restrict__ w, int T, int k, int L,
                               __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * L) return;
  const int t = i / L, l = i % L;
  float s = 0.f;
  for (int j = 0; j < k; ++j) s = fmaf(w[t * k + j], y[(size_t(t) * k + j) * L + l], s);
  out[i] = __float2bfloat16(s);
}

}  // namespace

#define CBF(t) reinterpret_cast<const __nv_bfloat16*>((t).data_ptr())

// Routed experts of a latent MoE: latent [T, L] bf16, chosen [T, k] int32 (expert ids), weights [T, k] fp32 (the
// routed scaling already applied), up [E, F, L], down [E, L, F] bf16 -> [T, L] bf16.
torch::Tensor moe_experts(const torch::Tensor& latent, const torch::Tensor& chosen, const torch::Tensor& weights,
                          const torch::Tensor& up, const torch::Tensor& down) {
  const at::cuda::CUDAGuard g(latent.device());
  TORCH_CHECK(latent.scalar_type() == at::kBFloat16 && up.scalar_type() == at::kBFloat16 &&
              down.scalar_type() == at::kBFloat16, "moe_experts: bf16 latent and expert weights");
  TORCH_CHECK(latent.is_contiguous() && up.is_contiguous() && down.is_contiguous());
  const int T = latent.size(0), L = latent.size(1), k = chosen.size(1);
  const int E = up.size(0), F = up.size(1);
  TORCH_CHECK(up.size(2) == L && down.size(0) == E && down.size(1) == L && down.size(2) == F);
  TORCH_CHECK(E <= kMaxExperts, "moe_experts: at most 1024 experts");
  TORCH_CHECK(L % 8 == 0 && F % 8 == 0, "moe_experts: latent and expert widths must be multiples of 8");
  auto out = torch::empty({T, L}, latent.options());
  if (!T) return out;
  const int P = T * k;
  auto i32 = latent.options().dtype(torch::kInt32);
  auto ch = chosen.to(torch::kInt32).contiguous();
  auto wt = weights.to(torch::kFloat32).contiguous();
  auto offsets = torch::empty({E + 1}, i32), active = torch::empty({E}, i32), n_active = torch::empty({1}, i32);
  auto pairs = torch::empty({P}, i32);
  auto h = torch::empty({P, F}, latent.options());
  auto y = torch::empty({P, L}, latent.options().dtype(torch::kFloat32));
  auto st = at::cuda::getCurrentCUDAStream();
  C10_CUDA_CHECK(launch_pdl(moe_route_kernel, 1, kRouteThreads, 0, st.stream(), ch.data_ptr<int>(), P, E,
                            offsets.data_ptr<int>(), active.data_ptr<int>(), n_active.data_ptr<int>(),
                            pairs.data_ptr<int>()));
  const int slots = std::min(E, P);
  const size_t smem_up = size_t(kPairChunk) * L * sizeof(float), smem_dn = size_t(kPairChunk) * F * sizeof(float);
  TORCH_CHECK(smem_up <= 200 * 1024 && smem_dn <= 200 * 1024, "moe_experts: widths too large for the staging");
  cudaFuncSetAttribute(moe_gemv_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem_up));
  cudaFuncSetAttribute(moe_gemv_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem_dn));
  C10_CUDA_CHECK(launch_pdl(moe_gemv_kernel<true>, dim3(slots, (F + kGemvRows - 1) / kGemvRows), kGemvThreads, smem_up,
                            st.stream(), CBF(latent), k, offsets.data_ptr<int>(), active.data_ptr<int>(),
                            n_active.data_ptr<int>(), pairs.data_ptr<int>(), CBF(up), F, L,
                            static_cast<void*>(h.data_ptr())));
  C10_CUDA_CHECK(launch_pdl(moe_gemv_kernel<false>, dim3(slots, (L + kGemvRows - 1) / kGemvRows), kGemvThreads,
                            smem_dn, st.stream(), CBF(h), k, offsets.data_ptr<int>(), active.data_ptr<int>(),
                            n_active.data_ptr<int>(), pairs.data_ptr<int>(), CBF(down), L, F,
                            static_cast<void*>(y.data_ptr())));
  C10_CUDA_CHECK(launch_pdl(moe_mix_kernel, (T * L + 255) / 256, 256, 0, st.stream(), y.data_ptr<float>(),
                            wt.data_ptr<float>(), T, k, L, reinterpret_cast<__nv_bfloat16*>(out.data_ptr())));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

}  // namespace e4
