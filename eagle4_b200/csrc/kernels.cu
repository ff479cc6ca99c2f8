// Row-wise kernels: RMSNorm variants, embedding gather, output gates, GDN gate math, the attention projection's
// post-processing (q/k norm, RoPE, K/V cache write) and the greedy head's cross-tile argmax.
//
// Every reduction runs in a fixed order per row (thread-strided partial sums, a butterfly within the warp, then
// the warps in index order), so a row's result never depends on how many rows share the launch.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace e4 {

namespace {

constexpr int kRowThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < nw; ++i) s += red[i];
  return s;
}

__device__ __forceinline__ float bf(const __nv_bfloat16 x) { return __bfloat162float(x); }

// y = x * rsqrt(mean(x^2) + eps) * (w or 1 + w). Rows of H <= 8192 elements (H % 8 == 0): each thread loads its
// 16-byte vectors up front (the loads are independent, so they overlap), then reduces.
constexpr int kMaxVec = 4;  // 16-byte vectors per thread: 256 threads x 4 x 8 = 8192 elements
__device__ __forceinline__ void load_row(const __nv_bfloat16* __restrict__ x, int H, uint4* v, int& nv) {
  nv = 0;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < H / 8) { v[i] = reinterpret_cast<const uint4*>(x)[c]; nv = i + 1; }
  }
}
__device__ __forceinline__ float sumsq(const uint4* v, int nv) {
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    if (i >= nv) break;
    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(p[j]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
  return ss;
}
__device__ __forceinline__ void store_normed(const uint4* v, int nv, const __nv_bfloat16* __restrict__ w, int offset,
                                             float rs, __nv_bfloat16* __restrict__ y) {
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    if (i >= nv) break;
    const int c = threadIdx.x + i * blockDim.x;
    const uint4 wv = reinterpret_cast<const uint4*>(w)[c];
    const __nv_bfloat162* xp = reinterpret_cast<const __nv_bfloat162*>(&v[i]);
    const __nv_bfloat162* wp = reinterpret_cast<const __nv_bfloat162*>(&wv);
    uint4 out;
    __nv_bfloat162* op = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 xf = __bfloat1622float2(xp[j]), wf = __bfloat1622float2(wp[j]);
      const float sx = offset ? 1.f + wf.x : wf.x, sy = offset ? 1.f + wf.y : wf.y;
      op[j] = __floats2bfloat162_rn(xf.x * rs * sx, xf.y * rs * sy);
    }
    reinterpret_cast<uint4*>(y)[c] = out;
  }
}

__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int ldx, const __nv_bfloat16* __restrict__ w,
                               __nv_bfloat16* __restrict__ y, int ldy, int H, float eps, int offset) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  const size_t r = blockIdx.x;
  uint4 v[kMaxVec];
  int nv;
  load_row(x + r * ldx, H, v, nv);
  const float rs = rsqrtf(block_sum(sumsq(v, nv), red) / H + eps);
  store_normed(v, nv, w, offset, rs, y + r * ldy);
}

// y[r] = [rmsnorm(e[r], we) | rmsnorm(h[r], wh)]
__global__ void concat_norms_kernel(const __nv_bfloat16* __restrict__ e, const __nv_bfloat16* __restrict__ h, int ldh,
                                    const __nv_bfloat16* __restrict__ we, const __nv_bfloat16* __restrict__ wh,
                                    __nv_bfloat16* __restrict__ y, int H, float eps) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  const size_t r = blockIdx.x;
  uint4 ve[kMaxVec], vh[kMaxVec];
  int ne, nh;
  load_row(e + r * H, H, ve, ne);
  load_row(h + r * ldh, H, vh, nh);
  const float re = rsqrtf(block_sum(sumsq(ve, ne), red) / H + eps);
  const float rh = rsqrtf(block_sum(sumsq(vh, nh), red) / H + eps);
  store_normed(ve, ne, we, 0, re, y + r * 2 * H);
  store_normed(vh, nh, wh, 0, rh, y + r * 2 * H + H);
}

__global__ void embedding_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                 __nv_bfloat16* __restrict__ y, int H, int64_t V, int* err) {
  pdl_wait();
  pdl_trigger();
  const int64_t id = ids[blockIdx.x];
  if (id < 0 || id >= V) {
    if (threadIdx.x == 0) record_error(err, kErrBadIndex);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + id * H);
  uint4* dst = reinterpret_cast<uint4*>(y + size_t(blockIdx.x) * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

// per (row, group): rmsnorm over D then * silu(z)
// ``wg``: the weight's stride between groups (0: one [D] weight shared by every group; D: a [G, D] weight).
// ``gate_first`` 0: y = rmsnorm(o) * w * silu(z) (Qwen3.5 GDN); 1: y = rmsnorm(o * silu(z)) * w (Mamba2 / Nemotron-H).
__global__ void gated_rmsnorm_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ z, int ldz,
                                     const __nv_bfloat16* __restrict__ w, int wg, int gate_first,
                                     __nv_bfloat16* __restrict__ y, int T, int G, int D, float eps) {
  pdl_wait();
  pdl_trigger();
  // one warp per (row, group)
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int r = warp / G, g = warp % G;
  if (r >= T) return;
  const __nv_bfloat16* orow = o + (size_t(r) * G + g) * D;
  const __nv_bfloat16* zrow = z + size_t(r) * ldz + size_t(g) * D;
  float ss = 0.f;
  for (int i = lane; i < D; i += 32) {
    const float v = gate_first ? bf(orow[i]) * silu(bf(zrow[i])) : bf(orow[i]);
    ss += v * v;
  }
  const float rs = rsqrtf(warp_sum(ss) / D + eps);
  for (int i = lane; i < D; i += 32) {
    const float gz = silu(bf(zrow[i]));
    const float wv = bf(w[size_t(g) * wg + i]);
    const float n = gate_first ? bf(orow[i]) * gz * rs * wv : bf(orow[i]) * rs * wv * gz;
    y[(size_t(r) * G + g) * D + i] = __float2bfloat16(n);
  }
}

// Split the fused attention projection, RMS-normalise q and k per head (optional), rotate the first ``rot`` dims
// (NeoX halves, cos/sin from a table), write K and V at the row's cache slot and q to a contiguous buffer.
// One block per row, one warp per head; a head's D values are loaded as 16-byte vectors into shared memory first.
// ``qkv`` row layout [q (Hq*D) | gate (Hq*D, optional) | k (Hk*D) | v (Hk*D)].
constexpr int kPrepWarps = 8;
__global__ void __launch_bounds__(kPrepWarps * 32)
qkv_prepare_kernel(const __nv_bfloat16* __restrict__ qkv, int ldq, const int64_t* __restrict__ pos,
                   const int64_t* __restrict__ slot, __nv_bfloat16* kc, __nv_bfloat16* vc,
                   const __nv_bfloat16* __restrict__ qn, const __nv_bfloat16* __restrict__ kn, int norm_offset,
                   const float* __restrict__ cos_t, const float* __restrict__ sin_t, __nv_bfloat16* __restrict__ qout,
                   int Hq, int Hk, int D, int rot, int gated, float eps) {
  pdl_wait();
  pdl_trigger();
  __shared__ float buf[kPrepWarps][256];
  const size_t r = blockIdx.x;
  const __nv_bfloat16* row = qkv + r * ldq;
  const int64_t p = pos[r];
  const int64_t s = slot[r];
  const int half = rot / 2;
  const int koff = Hq * D * (gated ? 2 : 1);
  const int voff = koff + Hk * D;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* hb = buf[warp];
  // grid.y splits the heads: warp w of CTA (r, y) handles heads y * kPrepWarps + w, stepping by the whole grid
  for (int hh = blockIdx.y * kPrepWarps + warp; hh < Hq + Hk; hh += kPrepWarps * gridDim.y) {
    const bool isq = hh < Hq;
    const __nv_bfloat16* src = row + (isq ? hh * D : koff + (hh - Hq) * D);
    const __nv_bfloat16* nw = isq ? qn : kn;
    for (int c = lane; c < D / 8; c += 32) {
      const uint4 raw = reinterpret_cast<const uint4*>(src)[c];
      const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(p2[j]);
        hb[c * 8 + 2 * j] = f.x;
        hb[c * 8 + 2 * j + 1] = f.y;
      }
    }
    __syncwarp();
    if (nw) {
      float ss = 0.f;
      for (int i = lane; i < D; i += 32) ss = fmaf(hb[i], hb[i], ss);
      const float rs = rsqrtf(warp_sum(ss) / D + eps);
      __syncwarp();
      for (int i = lane; i < D; i += 32) {
        const float wv = __bfloat162float(nw[i]);
        hb[i] = __bfloat162float(__float2bfloat16(hb[i] * rs * (norm_offset ? 1.f + wv : wv)));
      }
      __syncwarp();
    }
    __nv_bfloat16* dst = isq ? qout + (r * Hq + hh) * D : kc + (size_t(s) * Hk + (hh - Hq)) * D;
    for (int i = lane; i < D; i += 32) {
      float v = hb[i];
      if (i < rot) {
        const int j = i < half ? i : i - half;
        const float other = hb[i < half ? i + half : i - half];
        const float c = cos_t[p * half + j], sn = sin_t[p * half + j];
        v = i < half ? v * c - other * sn : v * c + other * sn;
      }
      dst[i] = __float2bfloat16(v);
    }
    __syncwarp();
  }
  const uint4* vs = reinterpret_cast<const uint4*>(row + voff);
  uint4* vd = reinterpret_cast<uint4*>(vc + size_t(s) * Hk * D);
  for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < Hk * D / 8; i += blockDim.x * gridDim.y) vd[i] = vs[i];
}

// Greedy head: reduce per-tile (max, argmax) partials to one id per token (ties to the lower id).
__global__ void argmax_reduce_kernel(const float* __restrict__ val, const int* __restrict__ idx, int n_tiles, int T,
                                     int64_t* __restrict__ out_id, float* __restrict__ out_val) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int chunk = t / 256, j = t % 256;
  const int tc = min(256, T - chunk * 256);
  const float* v = val + size_t(chunk) * 256 * n_tiles;
  const int* ix = idx + size_t(chunk) * 256 * n_tiles;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < n_tiles; i += blockDim.x) {
    const float ov = v[size_t(i) * tc + j];
    const int oi = ix[size_t(i) * tc + j];
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[warp] = best; si[warp] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    best = sv[0];
    bi = si[0];
    for (int w = 1; w < int(blockDim.x >> 5); ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < bi)) { best = sv[w]; bi = si[w]; }
    out_id[t] = bi;
    out_val[t] = best;
  }
}

// Copy accepted rows' K/V (all attention layers at once): pointers of every layer's cache in ``kp`` / ``vp``.
__global__ void kv_commit_kernel(const int64_t* __restrict__ kp, const int64_t* __restrict__ vp, int layers,
                                 const int64_t* __restrict__ src, const int64_t* __restrict__ dst, int n, int row_elems) {
  pdl_wait();
  pdl_trigger();
  const int item = blockIdx.x;  // (layer, move)
  const int l = item / n, m = item % n;
  if (l >= layers) return;
  const int64_t s = src[m], d = dst[m];
  if (s == d) return;
  uint4* k = reinterpret_cast<uint4*>(kp[l]);
  uint4* v = reinterpret_cast<uint4*>(vp[l]);
  const int vec = row_elems / 8;
  for (int i = threadIdx.x; i < vec; i += blockDim.x) {
    k[d * vec + i] = k[s * vec + i];
    v[d * vec + i] = v[s * vec + i];
  }
}

}  // namespace

torch::Tensor gemm_error_word(torch::Device dev);

#define BF16(t) reinterpret_cast<__nv_bfloat16*>((t).data_ptr())
#define CBF16(t) reinterpret_cast<const __nv_bfloat16*>((t).data_ptr())

torch::Tensor rmsnorm(const torch::Tensor& x, const torch::Tensor& w, double eps, bool offset) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(-1) == 1);
  const at::cuda::CUDAGuard g(x.device());
  const int H = x.size(-1);
  TORCH_CHECK(H % 8 == 0 && H <= kRowThreads * kMaxVec * 8, "rmsnorm: H must be a multiple of 8 up to 8192");
  auto x2 = x.reshape({-1, H});
  auto y = torch::empty({x2.size(0), H}, x.options());
  if (x2.size(0))
    C10_CUDA_CHECK(launch_pdl(rmsnorm_kernel, x2.size(0), kRowThreads, 0, at::cuda::getCurrentCUDAStream().stream(), 
        CBF16(x2), x2.stride(0), CBF16(w), BF16(y), H, H, float(eps), offset ? 1 : 0));
  return y.view(x.sizes());
}

torch::Tensor concat_norms(const torch::Tensor& e, const torch::Tensor& h, const torch::Tensor& we,
                           const torch::Tensor& wh, double eps) {
  const at::cuda::CUDAGuard g(e.device());
  const int T = e.size(0), H = e.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= kRowThreads * kMaxVec * 8 && h.stride(0) % 8 == 0);
  auto y = torch::empty({T, 2 * H}, e.options());
  if (T)
    C10_CUDA_CHECK(launch_pdl(concat_norms_kernel, T, kRowThreads, 0, at::cuda::getCurrentCUDAStream().stream(), 
        CBF16(e.contiguous()), CBF16(h), h.stride(0), CBF16(we), CBF16(wh), BF16(y), H, float(eps)));
  return y;
}

torch::Tensor embedding(const torch::Tensor& ids, const torch::Tensor& table) {
  const at::cuda::CUDAGuard g(table.device());
  const int T = ids.size(0), H = table.size(1);
  TORCH_CHECK(H % 8 == 0 && table.is_contiguous());
  auto y = torch::empty({T, H}, table.options());
  auto id64 = ids.to(torch::kInt64).contiguous();
  if (T)
    C10_CUDA_CHECK(launch_pdl(embedding_kernel, T, 128, 0, at::cuda::getCurrentCUDAStream().stream(), 
        id64.data_ptr<int64_t>(), CBF16(table), BF16(y), H, table.size(0),
        gemm_error_word(table.device()).data_ptr<int>()));
  return y;
}

torch::Tensor gated_rmsnorm(const torch::Tensor& o, const torch::Tensor& z, const torch::Tensor& w, double eps,
                            bool gate_first) {
  const at::cuda::CUDAGuard g(o.device());
  auto oc = o.contiguous();
  const int T = oc.size(0), G = oc.size(1), D = oc.size(2);
  TORCH_CHECK(z.stride(-1) == 1);
  TORCH_CHECK(w.numel() == D || w.numel() == int64_t(G) * D,
              "gated_rmsnorm: the weight is one [D] row shared by the groups or one row per group");
  const int wg = w.numel() == D ? 0 : D;
  auto wc = w.contiguous();
  auto y = torch::empty({T, G * D}, o.options());
  const int warps = T * G;
  if (T) {
    C10_CUDA_CHECK(launch_pdl(gated_rmsnorm_kernel, (warps * 32 + 255) / 256, 256, 0,
                              at::cuda::getCurrentCUDAStream().stream(), CBF16(oc), CBF16(z), z.stride(0), CBF16(wc),
                              wg, gate_first ? 1 : 0, BF16(y), T, G, D, float(eps)));
  }
  return y;
}

torch::Tensor qkv_prepare(const torch::Tensor& qkv, const torch::Tensor& pos, const torch::Tensor& slot,
                          torch::Tensor kc, torch::Tensor vc, const c10::optional<torch::Tensor>& qn,
                          const c10::optional<torch::Tensor>& kn, bool norm_offset, const torch::Tensor& cos_t,
                          const torch::Tensor& sin_t, int64_t Hq, int64_t Hk, int64_t D, int64_t rot, bool gated,
                          double eps) {
  const at::cuda::CUDAGuard g(qkv.device());
  const int T = qkv.size(0);
  TORCH_CHECK(D % 8 == 0 && D <= 256 && qkv.stride(0) % 8 == 0, "qkv_prepare: D must be a multiple of 8 up to 256");
  auto q = torch::empty({T, Hq, D}, qkv.options());
  if (T)
    C10_CUDA_CHECK(launch_pdl(qkv_prepare_kernel, dim3(T, (Hq + Hk + kPrepWarps - 1) / kPrepWarps), kPrepWarps * 32, 0,
                              at::cuda::getCurrentCUDAStream().stream(),
        CBF16(qkv), qkv.stride(0), pos.data_ptr<int64_t>(), slot.data_ptr<int64_t>(), BF16(kc), BF16(vc),
        qn ? CBF16(*qn) : nullptr, kn ? CBF16(*kn) : nullptr, norm_offset ? 1 : 0, cos_t.data_ptr<float>(),
        sin_t.data_ptr<float>(), BF16(q), Hq, Hk, D, rot, gated ? 1 : 0, float(eps)));
  return q;
}

std::vector<torch::Tensor> argmax_reduce(const torch::Tensor& val, const torch::Tensor& idx, int64_t n_tiles,
                                         int64_t T) {
  const at::cuda::CUDAGuard g(val.device());
  auto ids = torch::empty({T}, val.options().dtype(torch::kInt64));
  auto best = torch::empty({T}, val.options().dtype(torch::kFloat32));
  if (T)
    C10_CUDA_CHECK(launch_pdl(argmax_reduce_kernel, T, 256, 0, at::cuda::getCurrentCUDAStream().stream(), 
        val.data_ptr<float>(), idx.data_ptr<int>(), n_tiles, T, ids.data_ptr<int64_t>(), best.data_ptr<float>()));
  return {ids, best};
}

void kv_commit(const torch::Tensor& kp, const torch::Tensor& vp, const torch::Tensor& src, const torch::Tensor& dst,
               int64_t row_elems) {
  const at::cuda::CUDAGuard g(src.device());
  const int n = src.size(0), layers = kp.size(0);
  TORCH_CHECK(row_elems % 8 == 0);
  if (n && layers)
    C10_CUDA_CHECK(launch_pdl(kv_commit_kernel, n * layers, 128, 0, at::cuda::getCurrentCUDAStream().stream(), 
        kp.data_ptr<int64_t>(), vp.data_ptr<int64_t>(), layers, src.data_ptr<int64_t>(), dst.data_ptr<int64_t>(), n,
        row_elems));
}

}  // namespace e4
