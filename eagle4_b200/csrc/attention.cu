// Tree attention over a paged KV cache.
//
// Every query row attends to a *logical key sequence*: the committed context positions [ctx_start, ctx_len) of its
// request (resolved through the block table), followed by up to 64 extra physical slots (its tree ancestors and
// itself, in depth order). The sequence is cut into fixed 128-key logical chunks counted from ctx_start; a CTA
// handles one (row, kv head, chunk) for all query heads of the kv group, and a second kernel merges the chunks of
// a row in chunk order. The arithmetic applied to a key depends only on its logical index, so a token decoded alone
// (context [0, L+d) plus itself) and the same token verified inside a tree (context [0, L) plus its d ancestors and
// itself) get bit-identical attention outputs. Within a chunk each lane scores one key, so the score of a key is a
// sequential dot product that depends on that key alone.
//
// The same kernel serves prefill chunks (context [0, p+1), no extras), tree verify, plain decode and the draft
// head's rows (a sliding window through ctx_start plus the row's draft ancestors).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace e4 {
namespace {

constexpr int kChunk = 128;   // logical keys per CTA: 4 warps x 32 keys
constexpr int kWarps = 4;
constexpr int kMaxG = 8;      // query heads per kv head handled by one CTA
constexpr int kMaxDPL = 8;    // head dims per lane (D <= 256)

// One CTA per (chunk, kv head, row). Lane l of warp w scores logical key chunk*128 + w*32 + l against the G query
// heads (a sequential dot product over D), the warp takes the softmax statistics of its 32 keys, then every lane
// accumulates P.V for its D/32 head dims over the warp's keys in key order. Warps merge in index order.
template <int DPL>
__global__ void __launch_bounds__(kWarps * 32)
attn_chunk_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ kc,
                  const __nv_bfloat16* __restrict__ vc, const int* __restrict__ bt, int bt_ld, int page,
                  const int* __restrict__ req, const int* __restrict__ ctx_start, const int* __restrict__ ctx_len,
                  const int* __restrict__ extra, int extra_ld, const int* __restrict__ n_extra, float scale, int Hq,
                  int Hk, int nchunks, float* __restrict__ ws) {
  pdl_wait();
  pdl_trigger();
  constexpr int D = DPL * 32;
  const int chunk = blockIdx.x, h = blockIdx.y, r = blockIdx.z;
  const int G = Hq / Hk;
  const int c0 = ctx_start[r], c1 = ctx_len[r], ne = n_extra[r];
  const int nctx = max(c1 - c0, 0);
  const int total = nctx + ne;
  const int k_begin = chunk * kChunk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ __align__(16) float sq[kMaxG * D];
  __shared__ float sm_m[kWarps][kMaxG], sm_l[kWarps][kMaxG];
  __shared__ float sm_acc[kWarps][kMaxG][D];
  if (k_begin >= total) {
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
      float* o = ws + ((size_t(r) * Hq + h * G + g) * nchunks + chunk) * (D + 2);
      o[D] = -INFINITY;
      o[D + 1] = 0.f;
    }
    return;
  }
  const int b = req[r];
  for (int i = threadIdx.x; i < G * D; i += blockDim.x)
    sq[i] = __bfloat162float(q[(size_t(r) * Hq + h * G) * D + i]) * scale;
  __syncthreads();
  // this lane's key
  const int kk = k_begin + warp * 32 + lane;
  const bool live = kk < total;
  int64_t slot = 0;
  if (live) {
    if (kk < nctx) {
      const int p = c0 + kk;
      slot = int64_t(bt[size_t(b) * bt_ld + p / page]) * page + p % page;
    } else {
      slot = extra[size_t(r) * extra_ld + (kk - nctx)];
    }
  }
  float s[kMaxG];
#pragma unroll
  for (int g = 0; g < kMaxG; ++g) s[g] = 0.f;
  if (live) {
    const uint4* kp = reinterpret_cast<const uint4*>(kc + (size_t(slot) * Hk + h) * D);
    const float4* q4 = reinterpret_cast<const float4*>(sq);
    // kKB 16-byte pieces of the key are requested before any is used (independent loads in flight), then consumed
    // in dimension order: the dot product's summation order does not change.
    constexpr int kKB = (D / 8) < 8 ? (D / 8) : 8;
    for (int c0k = 0; c0k < D / 8; c0k += kKB) {
      uint4 kr[kKB];
#pragma unroll
      for (int u = 0; u < kKB; ++u) kr[u] = kp[c0k + u];
#pragma unroll
      for (int u = 0; u < kKB; ++u) {
        const int c = c0k + u;
        const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&kr[u]);
        float kf[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(k2[j]);
          kf[2 * j] = f.x;
          kf[2 * j + 1] = f.y;
        }
#pragma unroll
        for (int g = 0; g < kMaxG; ++g) {
          if (g < G) {
            const float4 qa = q4[(g * D + c * 8) / 4], qb = q4[(g * D + c * 8) / 4 + 1];
            s[g] = fmaf(qa.x, kf[0], s[g]);
            s[g] = fmaf(qa.y, kf[1], s[g]);
            s[g] = fmaf(qa.z, kf[2], s[g]);
            s[g] = fmaf(qa.w, kf[3], s[g]);
            s[g] = fmaf(qb.x, kf[4], s[g]);
            s[g] = fmaf(qb.y, kf[5], s[g]);
            s[g] = fmaf(qb.z, kf[6], s[g]);
            s[g] = fmaf(qb.w, kf[7], s[g]);
          }
        }
      }
    }
  }
  // warp softmax statistics over its 32 keys
  float m[kMaxG], l[kMaxG], p[kMaxG];
#pragma unroll
  for (int g = 0; g < kMaxG; ++g) {
    if (g >= G) break;
    const float sv = live ? s[g] : -INFINITY;
    m[g] = warp_max(sv);
    p[g] = live ? __expf(sv - m[g]) : 0.f;
    l[g] = warp_sum(p[g]);
  }
  // P.V: lane owns dims [lane*DPL, lane*DPL + DPL); keys of the warp in lane order
  float acc[kMaxG][DPL];
#pragma unroll
  for (int g = 0; g < kMaxG; ++g)
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[g][i] = 0.f;
  const int nlive = min(32, total - (k_begin + warp * 32));
  // V rows of kVB keys are loaded together (independent loads in flight), then accumulated in key order.
  constexpr int kVB = DPL == 8 ? 4 : 8;
  for (int j0 = 0; j0 < nlive; j0 += kVB) {
    float vf[kVB][DPL];
#pragma unroll
    for (int u = 0; u < kVB; ++u) {
      const int64_t sj = __shfl_sync(0xffffffffu, slot, (j0 + u) & 31);
      if (j0 + u < nlive) {
        const __nv_bfloat16* vp = vc + (size_t(sj) * Hk + h) * D + lane * DPL;
        if constexpr (DPL == 8) {
          const uint4 raw = *reinterpret_cast<const uint4*>(vp);
          const __nv_bfloat162* v2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(v2[i]);
            vf[u][2 * i] = f.x;
            vf[u][2 * i + 1] = f.y;
          }
        } else {
#pragma unroll
          for (int i = 0; i < DPL; ++i) vf[u][i] = __bfloat162float(vp[i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < DPL; ++i) vf[u][i] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < kVB; ++u) {
      if (j0 + u >= nlive) break;
#pragma unroll
      for (int g = 0; g < kMaxG; ++g) {
        if (g >= G) break;
        const float pj = __shfl_sync(0xffffffffu, p[g], j0 + u);
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[g][i] = fmaf(pj, vf[u][i], acc[g][i]);
      }
    }
  }
#pragma unroll
  for (int g = 0; g < kMaxG; ++g) {
    if (g >= G) break;
    if (lane == 0) {
      sm_m[warp][g] = nlive > 0 ? m[g] : -INFINITY;
      sm_l[warp][g] = nlive > 0 ? l[g] : 0.f;
    }
#pragma unroll
    for (int i = 0; i < DPL; ++i) sm_acc[warp][g][lane * DPL + i] = nlive > 0 ? acc[g][i] : 0.f;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int g = idx / D, d = idx % D;
    float M = -INFINITY;
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sm_m[w][g]);
    float L = 0.f, A = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      const float mw = sm_m[w][g];
      if (mw == -INFINITY) continue;
      const float c = __expf(mw - M);
      L += sm_l[w][g] * c;
      A += sm_acc[w][g][d] * c;
    }
    float* o = ws + ((size_t(r) * Hq + h * G + g) * nchunks + chunk) * (D + 2);
    o[d] = A;
    if (d == 0) {
      o[D] = M;
      o[D + 1] = L;
    }
  }
}

// Merge a row's chunks in chunk order and normalise: one block per (row, qhead). With ``gate`` the output is
// multiplied by sigmoid(gate) (the gated-attention output gate), saving a separate pass.
__global__ void attn_merge_kernel(const float* __restrict__ ws, int nchunks, int D, int Hq,
                                  const __nv_bfloat16* __restrict__ gate, int ldg, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const size_t rh = blockIdx.x;
  const float* base = ws + rh * nchunks * (D + 2);
  float M = -INFINITY;
  for (int c = 0; c < nchunks; ++c) M = fmaxf(M, base[size_t(c) * (D + 2) + D]);
  const size_t r = rh / Hq, hh = rh % Hq;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float L = 0.f, A = 0.f;
    for (int c = 0; c < nchunks; ++c) {
      const float* o = base + size_t(c) * (D + 2);
      const float mc = o[D];
      if (mc == -INFINITY) continue;
      const float w = __expf(mc - M);
      L += o[D + 1] * w;
      A += o[d] * w;
    }
    float v = L > 0.f ? A / L : 0.f;
    if (gate) {
      v = __bfloat162float(__float2bfloat16(v));
      v *= sigmoidf_(__bfloat162float(gate[r * ldg + hh * D + d]));
    }
    out[rh * D + d] = __float2bfloat16(v);
  }
}

}  // namespace

// q [T, Hq, D] bf16; caches [slots, Hk, D]; returns [T, Hq, D]. ``max_keys`` bounds every row's logical length.
torch::Tensor attention(const torch::Tensor& q, const torch::Tensor& kc, const torch::Tensor& vc,
                        const torch::Tensor& bt, int64_t page, const torch::Tensor& req, const torch::Tensor& ctx_start,
                        const torch::Tensor& ctx_len, const torch::Tensor& extra, const torch::Tensor& n_extra,
                        double scale, int64_t max_keys, const c10::optional<torch::Tensor>& gate) {
  const at::cuda::CUDAGuard g(q.device());
  const int T = q.size(0), Hq = q.size(1), D = q.size(2), Hk = kc.size(1);
  TORCH_CHECK(q.is_contiguous() && kc.is_contiguous() && vc.is_contiguous());
  TORCH_CHECK(Hq % Hk == 0 && Hq / Hk <= kMaxG, "attention: query heads per kv head must be <= 8");
  TORCH_CHECK(D % 32 == 0 && D <= 32 * kMaxDPL, "attention: head dim must be a multiple of 32 up to 256");
  auto out = torch::empty_like(q);
  if (T == 0) return out;
  const int nchunks = std::max<int64_t>(1, (max_keys + kChunk - 1) / kChunk);
  auto ws = torch::empty({int64_t(T) * Hq * nchunks * (D + 2)}, q.options().dtype(torch::kFloat32));
  auto i32 = [](const torch::Tensor& t) { return t.to(torch::kInt32).contiguous(); };
  auto bt_ = i32(bt), req_ = i32(req), cs = i32(ctx_start), cl = i32(ctx_len), ex = i32(extra), ne = i32(n_extra);
  dim3 grid(nchunks, Hk, T);
  auto stream = at::cuda::getCurrentCUDAStream();
#define E4_ATTN(DPL)                                                                                              \
  C10_CUDA_CHECK(launch_pdl(attn_chunk_kernel<DPL>, grid, kWarps * 32, 0, stream.stream(),                                                       \
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(kc.data_ptr()), \
      reinterpret_cast<const __nv_bfloat16*>(vc.data_ptr()), bt_.data_ptr<int>(), bt_.size(1), page,             \
      req_.data_ptr<int>(), cs.data_ptr<int>(), cl.data_ptr<int>(), ex.data_ptr<int>(), ex.size(1),              \
      ne.data_ptr<int>(), float(scale), Hq, Hk, nchunks, ws.data_ptr<float>()))
  switch (D / 32) {
    case 2: E4_ATTN(2); break;
    case 4: E4_ATTN(4); break;
    case 8: E4_ATTN(8); break;
    default: TORCH_CHECK(false, "attention: head dim must be 64, 128 or 256");
  }
#undef E4_ATTN
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const __nv_bfloat16* gp = gate ? reinterpret_cast<const __nv_bfloat16*>(gate->data_ptr()) : nullptr;
  const int ldg = gate ? int(gate->stride(0)) : 0;
  if (gate) TORCH_CHECK(gate->stride(1) == 1 && gate->size(0) == T, "attention: gate must be [T, Hq*D] rows");
  C10_CUDA_CHECK(launch_pdl(attn_merge_kernel, T * Hq, 128, 0, stream.stream(), ws.data_ptr<float>(), nchunks, D, Hq, gp, ldg,
                                                reinterpret_cast<__nv_bfloat16*>(out.data_ptr())));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

}  // namespace e4
