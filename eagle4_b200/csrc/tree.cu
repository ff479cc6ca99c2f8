// Draft-tree kernels: the candidate head's exact re-score and tail (softmax over the candidates, top-K children),
// and the fused greedy accept walk.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace e4 {
namespace {

// logit[r, c] = lm_head[idx[r, c]] . h[r] in fp32; one warp per (row, candidate), 16-byte loads.
__global__ void gather_dot_kernel(const __nv_bfloat16* __restrict__ h, const __nv_bfloat16* __restrict__ w,
                                  const int64_t* __restrict__ idx, float* __restrict__ out, int R, int C, int H,
                                  int64_t V, int* err) {
  pdl_wait();
  pdl_trigger();
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= R * C) return;
  const int r = gw / C;
  const int64_t id = idx[gw];
  if (id < 0 || id >= V) {
    if (lane == 0) { record_error(err, kErrBadIndex); out[gw] = -INFINITY; }
    return;
  }
  const uint4* wr = reinterpret_cast<const uint4*>(w + id * H);
  const uint4* hr = reinterpret_cast<const uint4*>(h + size_t(r) * H);
  float acc = 0.f;
  for (int i = lane; i < H / 8; i += 32) {
    const uint4 a = wr[i], b = hr[i];
    const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 fa = __bfloat1622float2(a2[j]), fb = __bfloat1622float2(b2[j]);
      acc = fmaf(fa.x, fb.x, acc);
      acc = fmaf(fa.y, fb.y, acc);
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) out[gw] = acc;
}

// Per row: softmax (temperature) over C candidate logits, then the top K probabilities (ties to the lower
// candidate position) and their ids. One block of 128 threads per row; C <= 1024.
__global__ void softmax_topk_kernel(const float* __restrict__ logit, const int64_t* __restrict__ ids, int C, int K,
                                    float inv_temp, float* __restrict__ probs, int64_t* __restrict__ out_ids) {
  pdl_wait();
  pdl_trigger();
  __shared__ float p[1024];
  __shared__ float red[32];
  const int r = blockIdx.x;
  const float* lr = logit + size_t(r) * C;
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < C; i += blockDim.x) mx = fmaxf(mx, lr[i] * inv_temp);
  mx = warp_max(mx);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = red[0];
  for (int i = 1; i < nw; ++i) mx = fmaxf(mx, red[i]);
  __syncthreads();
  float s = 0.f;
  for (int i = threadIdx.x; i < C; i += blockDim.x) {
    const float e = __expf(lr[i] * inv_temp - mx);
    p[i] = e;
    s += e;
  }
  s = warp_sum(s);
  if (lane == 0) red[warp] = s;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < nw; ++i) tot += red[i];
  const float inv = 1.f / tot;
  for (int i = threadIdx.x; i < C; i += blockDim.x) p[i] *= inv;
  __syncthreads();
  // K rounds of block argmax (K <= 8)
  __shared__ float bv[32];
  __shared__ int bi[32];
  for (int k = 0; k < K; ++k) {
    float best = -1.f;
    int besti = 0x7fffffff;
    for (int i = threadIdx.x; i < C; i += blockDim.x)
      if (p[i] > best || (p[i] == best && i < besti)) { best = p[i]; besti = i; }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
      if (ov > best || (ov == best && oi < besti)) { best = ov; besti = oi; }
    }
    if (lane == 0) { bv[warp] = best; bi[warp] = besti; }
    __syncthreads();
    if (threadIdx.x == 0) {
      float b = bv[0];
      int ix = bi[0];
      for (int w = 1; w < nw; ++w)
        if (bv[w] > b || (bv[w] == b && bi[w] < ix)) { b = bv[w]; ix = bi[w]; }
      probs[size_t(r) * K + k] = b;
      out_ids[size_t(r) * K + k] = ids ? ids[size_t(r) * C + ix] : ix;
      p[ix] = -2.f;
    }
    __syncthreads();
  }
}

// Greedy accept walk, one thread per request: from row 0 follow the child whose token equals the target's argmax
// at the current row (lowest row on duplicates); the bonus token is the argmax at the last accepted row.
__global__ void accept_greedy_kernel(const int64_t* __restrict__ tid, const int64_t* __restrict__ tokens,
                                     const int* __restrict__ parent, const int* __restrict__ nrows, int B, int N,
                                     int* __restrict__ acc, int* __restrict__ cnt, int64_t* __restrict__ bonus) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int n = nrows[b];
  const int64_t* tk = tokens + size_t(b) * N;
  const int* pr = parent + size_t(b) * N;
  int* ac = acc + size_t(b) * N;
  for (int i = 0; i < N; ++i) ac[i] = -1;
  int cur = 0, c = 1;
  ac[0] = 0;
  while (true) {
    const int64_t want = tid[size_t(b) * N + cur];
    int nxt = -1;
    for (int r = 1; r < n; ++r)
      if (pr[r] == cur && tk[r] == want) { nxt = r; break; }
    if (nxt < 0) { bonus[b] = want; break; }
    ac[c++] = nxt;
    cur = nxt;
  }
  cnt[b] = c;
}

}  // namespace

torch::Tensor gemm_error_word(torch::Device dev);

torch::Tensor gather_dot(const torch::Tensor& h, const torch::Tensor& w, const torch::Tensor& idx) {
  const at::cuda::CUDAGuard g(h.device());
  const int R = idx.size(0), C = idx.size(1), H = h.size(1);
  TORCH_CHECK(H % 8 == 0 && h.is_contiguous() && w.is_contiguous());
  auto out = torch::empty({R, C}, h.options().dtype(torch::kFloat32));
  auto ix = idx.to(torch::kInt64).contiguous();
  const int warps = R * C;
  if (warps)
    C10_CUDA_CHECK(launch_pdl(gather_dot_kernel, (warps * 32 + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream().stream(), 
        reinterpret_cast<const __nv_bfloat16*>(h.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
        ix.data_ptr<int64_t>(), out.data_ptr<float>(), R, C, H, w.size(0),
        gemm_error_word(h.device()).data_ptr<int>()));
  return out;
}

std::vector<torch::Tensor> softmax_topk(const torch::Tensor& logit, const c10::optional<torch::Tensor>& ids, int64_t K,
                                        double temperature) {
  const at::cuda::CUDAGuard g(logit.device());
  const int R = logit.size(0), C = logit.size(1);
  TORCH_CHECK(C <= 1024 && K <= 8 && logit.is_contiguous());
  auto probs = torch::empty({R, K}, logit.options());
  auto oid = torch::empty({R, K}, logit.options().dtype(torch::kInt64));
  torch::Tensor idc;
  if (ids) idc = ids->to(torch::kInt64).contiguous();
  if (R)
    C10_CUDA_CHECK(launch_pdl(softmax_topk_kernel, R, 128, 0, at::cuda::getCurrentCUDAStream().stream(), 
        logit.data_ptr<float>(), ids ? idc.data_ptr<int64_t>() : nullptr, C, K, float(1.0 / temperature),
        probs.data_ptr<float>(), oid.data_ptr<int64_t>()));
  return {probs, oid};
}

std::vector<torch::Tensor> accept_greedy(const torch::Tensor& tid, const torch::Tensor& tokens,
                                         const torch::Tensor& parent, const torch::Tensor& nrows) {
  const at::cuda::CUDAGuard g(tokens.device());
  const int B = tokens.size(0), N = tokens.size(1);
  auto o = tokens.options();
  auto acc = torch::empty({B, N}, o.dtype(torch::kInt32));
  auto cnt = torch::empty({B}, o.dtype(torch::kInt32));
  auto bonus = torch::empty({B}, o.dtype(torch::kInt64));
  auto t = tid.to(torch::kInt64).contiguous(), tk = tokens.to(torch::kInt64).contiguous(),
       pr = parent.to(torch::kInt32).contiguous(), nr = nrows.to(torch::kInt32).contiguous();
  if (B)
    C10_CUDA_CHECK(launch_pdl(accept_greedy_kernel, (B + 127) / 128, 128, 0, at::cuda::getCurrentCUDAStream().stream(), 
        t.data_ptr<int64_t>(), tk.data_ptr<int64_t>(), pr.data_ptr<int>(), nr.data_ptr<int>(), B, N,
        acc.data_ptr<int>(), cnt.data_ptr<int>(), bonus.data_ptr<int64_t>()));
  return {acc, cnt, bonus};
}

}  // namespace e4

// =====================================================================================================================
// Top-C selection over long rows (the candidate shortlist over the draft vocabulary) and the draft-tree updates.
// =====================================================================================================================
namespace e4 {
namespace {

// Order-preserving map of fp32 to uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kSelThreads = 256;
constexpr int kSelPer = 16;  // elements per thread: a CTA selects within 4096 elements

// Radix select inside one CTA: among ``n`` (<= 4096) elements (key, index) find the ``C`` largest keys (ties to the
// lower index) and write them in index order to (ov, oi). Elements of thread t are [t*16, t*16+16) (index order).
__device__ void cta_select(const uint32_t* key, const int* idx, const float* val, int n, int C, float* ov, int* oi) {
  __shared__ int hist[256];
  __shared__ uint32_t s_prefix;
  __shared__ int s_remaining, s_digit_above;
  __shared__ int scan[kSelThreads];
  const int t = threadIdx.x;
  uint32_t prefix = 0, mask = 0;
  int remaining = min(C, n);
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = t; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int i = 0; i < kSelPer; ++i) {
      const int e = t * kSelPer + i;
      if (e < n && (key[i] & mask) == prefix) atomicAdd(&hist[(key[i] >> shift) & 255], 1);
    }
    __syncthreads();
    if (t < 32) {
      // lane l owns bins [255 - 8l - 7, 255 - 8l] (descending); suffix counts from the top bin down
      int c[8], tot = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) { c[i] = hist[255 - 8 * t - i]; tot += c[i]; }
      int incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (t >= o) incl += v;
      }
      const int before = incl - tot;  // count in bins above this lane's range
      // the digit: first bin (from the top) where the running count reaches ``remaining``
      int found = -1, above_d = 0, run = before;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (found < 0 && run + c[i] >= remaining) { found = 255 - 8 * t - i; above_d = run; }
        run += c[i];
      }
      const unsigned hit = __ballot_sync(0xffffffffu, found >= 0);
      const int src = hit ? __ffs(hit) - 1 : 31;
      int d = __shfl_sync(0xffffffffu, found, src);
      int above = __shfl_sync(0xffffffffu, above_d, src);
      if (!hit) { d = 0; above = __shfl_sync(0xffffffffu, incl, 31) - hist[0]; }
      if (t == 0) {
        s_prefix = prefix | (uint32_t(d) << shift);
        s_remaining = remaining - above;
        s_digit_above = above;
      }
    }
    __syncthreads();
    prefix = s_prefix;
    mask |= 255u << shift;
    remaining = s_remaining;
    __syncthreads();
  }
  // threshold key = prefix; take every key above it and the first ``remaining`` keys equal to it (index order)
  int n_gt = 0, n_eq = 0;
  for (int i = 0; i < kSelPer; ++i) {
    const int e = t * kSelPer + i;
    if (e < n) { n_gt += key[i] > prefix; n_eq += key[i] == prefix; }
  }
  // exclusive block scans of n_eq then of the combined counts (index order)
  scan[t] = n_eq;
  __syncthreads();
  for (int off = 1; off < kSelThreads; off <<= 1) {
    const int v = t >= off ? scan[t - off] : 0;
    __syncthreads();
    scan[t] += v;
    __syncthreads();
  }
  const int eq_before = scan[t] - n_eq;
  __syncthreads();
  const int take_eq = max(0, min(n_eq, remaining - eq_before));
  const int mine = n_gt + take_eq;
  scan[t] = mine;
  __syncthreads();
  for (int off = 1; off < kSelThreads; off <<= 1) {
    const int v = t >= off ? scan[t - off] : 0;
    __syncthreads();
    scan[t] += v;
    __syncthreads();
  }
  int pos = scan[t] - mine;
  for (int i = n + t; i < C; i += blockDim.x) {  // fewer than C elements: pad with -inf
    ov[i] = -INFINITY;
    oi[i] = 0x7fffffff;
  }
  int eq_taken = 0;
  for (int i = 0; i < kSelPer; ++i) {
    const int e = t * kSelPer + i;
    if (e >= n) break;
    bool take = key[i] > prefix;
    if (!take && key[i] == prefix && eq_taken < take_eq) { take = true; ++eq_taken; }
    if (take) { ov[pos] = val[i]; oi[pos] = idx[i]; ++pos; }
  }
}

// Stage 1: CTA (slice, row) selects the top C of scores[row, slice*4096 : ...].
__global__ void __launch_bounds__(kSelThreads) topk_slice_kernel(const float* __restrict__ scores, int ld, int V, int C,
                                                                 int nslices, float* __restrict__ ov,
                                                                 int* __restrict__ oi) {
  pdl_wait();
  pdl_trigger();
  const int slice = blockIdx.x, r = blockIdx.y;
  const int base = slice * kSelThreads * kSelPer;
  const int n = min(kSelThreads * kSelPer, V - base);
  uint32_t key[kSelPer];
  int idx[kSelPer];
  float val[kSelPer];
  for (int i = 0; i < kSelPer; ++i) {
    const int e = threadIdx.x * kSelPer + i;
    const bool in = e < n;
    val[i] = in ? scores[size_t(r) * ld + base + e] : -INFINITY;
    key[i] = in ? fkey(val[i]) : 0u;
    idx[i] = base + e;
  }
  cta_select(key, idx, val, n, C, ov + (size_t(r) * nslices + slice) * C, oi + (size_t(r) * nslices + slice) * C);
}

// Merge pass: CTA (row, group) selects the top C of candidates [group*gsize, +gsize) of the row's m candidates.
// Intermediate passes write unsorted groups (value, id int32); the final pass (one group) sorts (value desc, id asc)
// and writes int64 ids.
__global__ void __launch_bounds__(kSelThreads) topk_merge_kernel(const float* __restrict__ iv, const int* __restrict__ ii,
                                                                 int m, int gsize, int C, float* __restrict__ ov,
                                                                 int* __restrict__ oi32, int64_t* __restrict__ oi) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x, grp = blockIdx.y, ngroups = gridDim.y;
  __shared__ float sv[1024];
  __shared__ int si[1024];
  uint32_t key[kSelPer];
  int idx[kSelPer];
  float val[kSelPer];
  const int g0 = grp * gsize;
  const int n = min(gsize, m - g0);
  for (int i = 0; i < kSelPer; ++i) {
    const int e = threadIdx.x * kSelPer + i;
    const bool in = e < n;
    val[i] = in ? iv[size_t(r) * m + g0 + e] : -INFINITY;
    idx[i] = in ? ii[size_t(r) * m + g0 + e] : 0x7fffffff;
    key[i] = in ? fkey(val[i]) : 0u;
  }
  if (oi == nullptr) {
    cta_select(key, idx, val, n, C, ov + (size_t(r) * ngroups + grp) * C, oi32 + (size_t(r) * ngroups + grp) * C);
    return;
  }
  cta_select(key, idx, val, n, C, sv, si);
  __syncthreads();
  // bitonic sort of C (power of two <= 1024) entries: value desc, id asc
  int P = 1;
  while (P < C) P <<= 1;
  for (int i = threadIdx.x + C; i < P; i += blockDim.x) { sv[i] = -INFINITY; si[i] = 0x7fffffff; }
  __syncthreads();
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int l = i ^ j;
        if (l > i) {
          const bool a_first = sv[i] > sv[l] || (sv[i] == sv[l] && si[i] < si[l]);
          const bool up = (i & k) == 0;
          if (up != a_first) {
            const float tv = sv[i]; sv[i] = sv[l]; sv[l] = tv;
            const int ti = si[i]; si[i] = si[l]; si[l] = ti;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < C; i += blockDim.x) {
    ov[size_t(r) * C + i] = sv[i];
    oi[size_t(r) * C + i] = si[i];
  }
}

// Work deltas of request b (DraftTree definition): for j = 0..K, the running sums of the first ``max_verify`` values of
// merge(old best set, the layer's top j) (both descending), written to ``rows[b][v][j]``; the last CTA of the launch
// to finish stores the batch mean (requests summed in order) into ``out[v][j]`` and resets the arrival counter.
// ``old_best`` / ``top`` are this CTA's shared-memory copies. Threads 0..K each merge one j.
__device__ __forceinline__ void store_work_deltas(int b, int bs, int K, int work_cap, int max_verify,
                                                  const float* old_best, const float* top, float* rows, float* out,
                                                  unsigned* counter) {
  const int t = threadIdx.x;
  __syncthreads();
  if (t <= K) {
    float sum = 0.f;
    int a = 0, c = 0;
    for (int v = 0; v < max_verify; ++v) {
      float x;
      if (c < t && (a >= work_cap || top[c] > old_best[a])) x = top[c++];
      else x = a < work_cap ? old_best[a++] : 0.f;
      sum += x;
      rows[(size_t(b) * max_verify + v) * (K + 1) + t] = sum;
    }
  }
  __shared__ int last;
  __threadfence();
  __syncthreads();
  if (t == 0) last = atomicAdd(counter, 1u) == unsigned(bs - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  const int n = max_verify * (K + 1);
  for (int i = t; i < n; i += blockDim.x) {
    float s = 0.f;
    for (int r = 0; r < bs; ++r) s += __ldcg(rows + size_t(r) * n + i);
    out[i] = s / float(bs);
  }
  if (t == 0) *counter = 0u;
}

// Copy ``rows`` rows of H bf16 values in 16-byte pieces: dst row k <- src row src_row[k] (shared memory). A thread
// issues up to eight loads before its stores, so the copy costs a few memory round trips instead of one per piece.
__device__ __forceinline__ void gather_rows16(__nv_bfloat16* __restrict__ dst, const __nv_bfloat16* __restrict__ src,
                                              const int* src_row, int rows, int H) {
  constexpr int U = 8;
  const int vec = H / 8, total = rows * vec;
  for (int i0 = threadIdx.x; i0 < total; i0 += blockDim.x * U) {
    uint4 tmp[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i < total) tmp[u] = reinterpret_cast<const uint4*>(src + size_t(src_row[i / vec]) * H)[i % vec];
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i < total) reinterpret_cast<uint4*>(dst + size_t(i / vec) * H)[i % vec] = tmp[u];
    }
  }
}

// The tree's first level for request b (DraftTree.begin semantics): the root's K children (sorted by probability,
// ties to the lower child, unless the draw order is kept), the frontier (tokens, scores, nodes, the root's hidden
// row for every lane), the best set {root, children} and, when asked, the depth-0 work deltas.
__global__ void tree_begin_kernel(const float* __restrict__ root_probs, const int64_t* __restrict__ root_tokens,
                                  const __nv_bfloat16* __restrict__ root_hidden, int H, int K, int keep_order,
                                  float root_score, int work_cap, int cap, float* scores, int64_t* tokens,
                                  float* front_scores, int64_t* front_tokens, __nv_bfloat16* front_hidden,
                                  int64_t* front_nodes, float* best, float* best_prev, float* layer_top,
                                  int max_verify, float* delta_rows, float* deltas_out, unsigned* counter) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x, t = threadIdx.x;
  __shared__ float pr[8], ranked[8], old_best[64];
  __shared__ int64_t tk[8];
  if (t < K) {
    const float v = root_probs[b * K + t];
    int rank = 0;  // descending, ties to the lower child
    for (int i = 0; i < K; ++i) {
      const float o = root_probs[b * K + i];
      rank += (o > v) || (o == v && i < t);
    }
    const int at = keep_order ? t : rank;
    pr[at] = v;
    tk[at] = root_tokens[b * K + t];
    ranked[rank] = v;
  }
  for (int i = t; i < work_cap; i += blockDim.x) old_best[i] = i == 0 ? root_score : 0.f;
  __syncthreads();
  if (t < K) {
    scores[size_t(b) * cap + t] = pr[t];
    tokens[size_t(b) * cap + t] = tk[t];
    front_scores[b * K + t] = pr[t];
    front_tokens[b * K + t] = tk[t];
    front_nodes[b * K + t] = t;
    layer_top[b * K + t] = ranked[t];
  }
  for (int i = t; i < work_cap; i += blockDim.x) {
    best_prev[size_t(b) * work_cap + i] = old_best[i];
    best[size_t(b) * work_cap + i] = i == 0 ? root_score : (i <= K ? ranked[i - 1] : 0.f);
  }
  __shared__ int src_row[8];
  if (t < K) src_row[t] = b;
  __syncthreads();
  gather_rows16(front_hidden + size_t(b) * K * H, root_hidden, src_row, K, H);
  if (deltas_out != nullptr)
    store_work_deltas(b, gridDim.x, K, work_cap, max_verify, old_best, ranked, delta_rows, deltas_out, counter);
}

// One draft-tree step for request b (one CTA): children scores, frontier top-K (ties to the lower child), tokens,
// parents, frontier hidden rows and ancestor slots gathered by the picked lanes, and the best-score set merged with
// the new layer. (DraftTree.step semantics.)
__global__ void tree_step_kernel(const float* __restrict__ probs, const int64_t* __restrict__ toks,
                                 const __nv_bfloat16* __restrict__ hidden, int H, int K, int step, int layer_start,
                                 int parent_col, int work_cap, int cap, int pcap, int depth_cap, float* scores,
                                 int64_t* tokens, int64_t* parents, float* front_scores, int64_t* front_tokens,
                                 __nv_bfloat16* front_hidden, int64_t* front_nodes, int* ancestors, float* best,
                                 float* best_prev, float* layer_top, int max_verify, float* delta_rows,
                                 float* deltas_out, unsigned* counter) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  __shared__ float layer[64];
  __shared__ int pick[8];
  __shared__ float top[8];
  __shared__ int anc_tmp[8 * 32];
  __shared__ float merged[64 + 64];
  const int t = threadIdx.x;
  const int KK = K * K;
  if (t < KK) {
    const int lane = t / K;
    layer[t] = front_scores[b * K + lane] * probs[size_t(b * K + lane) * K + (t % K)];
  }
  __syncthreads();
  if (t < KK) {
    scores[size_t(b) * cap + layer_start + t] = layer[t];
    tokens[size_t(b) * cap + layer_start + t] = toks[size_t(b * K + t / K) * K + (t % K)];
  }
  if (t < KK) {
    // top-K of the layer by rank (ties to the lower index): one thread per value, no serial scan
    const float v = layer[t];
    int rank = 0;
    for (int i = 0; i < KK; ++i) rank += (layer[i] > v) || (layer[i] == v && i < t);
    if (rank < K) { pick[rank] = t; top[rank] = v; }
  }
  __syncthreads();
  // ancestors of the picked lanes (read all before writing)
  for (int i = t; i < K * depth_cap; i += blockDim.x) anc_tmp[i] = ancestors[(size_t(b) * K + pick[i / depth_cap] / K) * depth_cap + i % depth_cap];
  __syncthreads();
  for (int i = t; i < K * depth_cap; i += blockDim.x) ancestors[size_t(b) * K * depth_cap + i] = anc_tmp[i];
  if (t < K) {
    parents[size_t(b) * pcap + parent_col + t] = pick[t] + layer_start;
    front_scores[b * K + t] = top[t];
    front_tokens[b * K + t] = toks[size_t(b * K + pick[t] / K) * K + (pick[t] % K)];
    front_nodes[b * K + t] = pick[t] + layer_start;
    layer_top[b * K + t] = top[t];
  }
  // frontier hidden rows: the picked lanes' draft hidden states
  __shared__ int src_row[8];
  if (t < K) src_row[t] = b * K + pick[t] / K;
  __syncthreads();
  gather_rows16(front_hidden + size_t(b) * K * H, hidden, src_row, K, H);
  // best set: the work_cap largest values of (best list ++ layer), descending; every value finds its rank in
  // parallel (ties by position), values ranked below work_cap are written at their rank
  const int m = work_cap + KK;
  for (int i = t; i < m; i += blockDim.x) merged[i] = i < work_cap ? best[size_t(b) * work_cap + i] : layer[i - work_cap];
  __syncthreads();
  if (t < work_cap) best_prev[size_t(b) * work_cap + t] = merged[t];
  for (int i = t; i < m; i += blockDim.x) {
    const float v = merged[i];
    int rank = 0;
    for (int j = 0; j < m; ++j) rank += (merged[j] > v) || (merged[j] == v && j < i);
    if (rank < work_cap) best[size_t(b) * work_cap + rank] = v;
  }
  // the step's work deltas: the old best set (merged[0, work_cap)) with the new layer's top
  if (deltas_out != nullptr)
    store_work_deltas(b, gridDim.x, K, work_cap, max_verify, merged, top, delta_rows, deltas_out, counter);
}

// The best ``count`` nodes of each request's tree as verify rows (DraftTree.verify_rows semantics): rank by
// depth-decayed score (ties to the lower node), emit in node order; tokens and parent rows (root row 0 = -1).
__global__ void select_rows_kernel(const float* __restrict__ scores, const float* __restrict__ decay,
                                   const int64_t* __restrict__ tokens, const int64_t* __restrict__ parents, int n,
                                   int cap, int pcap, int K, int count, int64_t* __restrict__ out_tok,
                                   int* __restrict__ out_parent, int64_t* __restrict__ out_node) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  __shared__ float d[1024];
  __shared__ int sel_pos[1024];
  __shared__ int row_node[64];
  for (int i = threadIdx.x; i < n; i += blockDim.x) d[i] = scores[size_t(b) * cap + i] * decay[i];
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    int rank = 0;
    const float di = d[i];
    for (int j = 0; j < n; ++j) rank += (d[j] > di) || (d[j] == di && j < i);
    sel_pos[i] = rank < count ? 1 : 0;
  }
  __syncthreads();
  // compaction in node order: thread t owns the nodes [t*per, (t+1)*per); an exclusive scan of the per-thread
  // counts (warp shuffles, then the warp totals) gives each selected node its row
  {
    __shared__ int warp_sum[32];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int per = (n + blockDim.x - 1) / blockDim.x;
    const int i0 = t * per, i1 = min(n, i0 + per);
    int cnt = 0;
    for (int i = i0; i < i1; ++i) cnt += sel_pos[i];
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) warp_sum[warp] = incl;
    __syncthreads();
    int r = incl - cnt;
    for (int w = 0; w < warp; ++w) r += warp_sum[w];
    for (int i = i0; i < i1; ++i) {
      if (sel_pos[i]) { row_node[r] = i; sel_pos[i] = r + 1; ++r; }
    }
  }
  __syncthreads();
  for (int r = threadIdx.x; r < count; r += blockDim.x) {
    const int node = row_node[r];
    out_tok[size_t(b) * count + r] = tokens[size_t(b) * cap + node];
    out_node[size_t(b) * (count + 1) + r + 1] = node;
    // parent node: depth 1 nodes hang off the root; depth >= 2 nodes read their frontier column
    int pnode = -1;
    if (node >= K) {
      const int layer = (node - K) / (K * K) + 2;  // depth of the node
      const int local = node - (K + (layer - 2) * K * K);
      const int base = layer - 1 > 1 ? (K + 1) + (layer - 1 - 2) * K : 1;  // frontier column of depth layer-1
      pnode = int(parents[size_t(b) * pcap + base + local / K]);
    }
    out_parent[size_t(b) * (count + 1) + r + 1] = pnode >= 0 ? sel_pos[pnode] : 0;
  }
  if (threadIdx.x == 0) {
    out_parent[size_t(b) * (count + 1)] = -1;
    out_node[size_t(b) * (count + 1)] = -1;
  }
}

// Row metadata of draft step ``s`` in one launch (the frontier's K rows per request): RoPE position L - 1 + s, the
// request's block-table row, the KV slot of position L + (s - 1) * K + k, the window start, the visible context
// length L, and the ancestor slots (depth-1 .. s, this row's own slot last), which are also recorded in the tree.
__global__ void draft_step_rows_kernel(const int64_t* __restrict__ L, const int* __restrict__ slot,
                                       const int* __restrict__ block_table, int bt_stride, int* ancestors,
                                       int depth_cap, int R, int K, int s, int page, int window, int64_t* pos,
                                       int* req, int64_t* slots, int* start, int* ctx_len, int* extra, int* n_extra) {
  pdl_wait();
  pdl_trigger();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= R) return;
  const int b = i / K, k = i % K;
  const int64_t l = L[b];
  const int rq = slot[b];
  const int64_t p_kv = l + int64_t(s - 1) * K + k;
  const int64_t sl = int64_t(block_table[size_t(rq) * bt_stride + p_kv / page]) * page + p_kv % page;
  pos[i] = l - 1 + s;
  req[i] = rq;
  slots[i] = sl;
  start[i] = window > 0 ? int(l - window > 0 ? l - window : 0) : 0;
  ctx_len[i] = int(l);
  n_extra[i] = s;
  int* anc = ancestors + (size_t(b) * K + k) * depth_cap;
  anc[s - 1] = int(sl);
  for (int j = 0; j < s - 1; ++j) extra[size_t(i) * s + j] = anc[j];
  extra[size_t(i) * s + s - 1] = int(sl);
}

// Everything the verify forward needs about its rows, one CTA per request and one thread per row (n <= 64): the
// row's tokens (root first), ancestor-or-self set (walking the parent rows; rows follow node order, parents first),
// RoPE position L + depth, KV slot of position L + r, the ancestor slots in row order (the attention's extra keys),
// their count, the parent row in the flattened batch, and the request's block-table row / context length.
__global__ void verify_rows_meta_kernel(const int* __restrict__ prow, const int64_t* __restrict__ toks,
                                        const int64_t* __restrict__ root, const int64_t* __restrict__ L,
                                        const int* __restrict__ slot, const int* __restrict__ block_table,
                                        int bt_stride, int n, int page, int64_t* tokens, int64_t* pos, int64_t* slots,
                                        int* extra, int* n_extra, int* parent, int* req, int* ctx_len) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x, r = threadIdx.x;
  __shared__ int64_t s_slot[64];
  const bool live = r < n;
  const int64_t l = L[b];
  const int rq = slot[b];
  int64_t sl = 0;
  uint64_t mask = 0;
  if (live) {
    const int64_t p = l + r;
    sl = int64_t(block_table[size_t(rq) * bt_stride + p / page]) * page + p % page;
    s_slot[r] = sl;
    int depth = -1;
    for (int j = r, hops = 0; j >= 0 && hops <= n; j = prow[size_t(b) * n + j], ++hops) {
      mask |= 1ull << j;
      ++depth;
    }
    const size_t i = size_t(b) * n + r;
    tokens[i] = r == 0 ? root[b] : toks[size_t(b) * (n - 1) + r - 1];
    pos[i] = l + depth;
    slots[i] = sl;
    const int pr = prow[size_t(b) * n + r];
    parent[i] = pr >= 0 ? b * n + pr : -1;
    req[i] = rq;
    ctx_len[i] = int(l);
  }
  __syncthreads();
  if (live) {
    const size_t i = size_t(b) * n + r;
    int c = 0;
    for (int j = 0; j < n; ++j)
      if ((mask >> j) & 1ull) extra[i * n + c++] = int(s_slot[j]);
    n_extra[i] = c;
    for (int j = c; j < n; ++j) extra[i * n + j] = int(sl);
  }
}

}  // namespace

// Top-C (value desc, id asc) of each row of fp32 scores [R, V]: (values [R, C], ids int64 [R, C]).
std::vector<torch::Tensor> topk_large(const torch::Tensor& scores, int64_t C) {
  const at::cuda::CUDAGuard g(scores.device());
  TORCH_CHECK(scores.scalar_type() == torch::kFloat32 && scores.stride(1) == 1 && C <= 1024);
  const int R = scores.size(0), V = scores.size(1);
  const int per = kSelThreads * kSelPer;
  TORCH_CHECK(2 * C <= per, "topk_large: C too large");
  const int ns = (V + per - 1) / per;
  auto o = scores.options();
  auto sv = torch::empty({R, ns, C}, o), si = torch::empty({R, ns, C}, o.dtype(torch::kInt32));
  auto ov = torch::empty({R, C}, o), oi = torch::empty({R, C}, o.dtype(torch::kInt64));
  if (!R) return {ov, oi};
  auto st = at::cuda::getCurrentCUDAStream();
  C10_CUDA_CHECK(launch_pdl(topk_slice_kernel, dim3(ns, R), kSelThreads, 0, st.stream(), scores.data_ptr<float>(), scores.stride(0), V, int(C), ns,
                                                         sv.data_ptr<float>(), si.data_ptr<int>()));
  // merge groups of whole slices until one group of candidates remains
  const int gsize = (per / int(C)) * int(C);
  int m = ns * int(C);
  while (m > gsize) {
    const int ng = (m + gsize - 1) / gsize;
    auto nv = torch::empty({R, ng, C}, o), ni = torch::empty({R, ng, C}, o.dtype(torch::kInt32));
    C10_CUDA_CHECK(launch_pdl(topk_merge_kernel, dim3(R, ng), kSelThreads, 0, st.stream(), sv.data_ptr<float>(), si.data_ptr<int>(), m, gsize,
                                                           int(C), nv.data_ptr<float>(), ni.data_ptr<int>(), nullptr));
    sv = nv;
    si = ni;
    m = ng * int(C);
  }
  C10_CUDA_CHECK(launch_pdl(topk_merge_kernel, dim3(R, 1), kSelThreads, 0, st.stream(), sv.data_ptr<float>(), si.data_ptr<int>(), m, m, int(C),
                                                        ov.data_ptr<float>(), nullptr, oi.data_ptr<int64_t>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {ov, oi};
}

void tree_step(const torch::Tensor& probs, const torch::Tensor& toks, const torch::Tensor& hidden, int64_t bs,
               int64_t K, int64_t step, int64_t layer_start, int64_t parent_col, torch::Tensor scores,
               torch::Tensor tokens, torch::Tensor parents, torch::Tensor front_scores, torch::Tensor front_tokens,
               torch::Tensor front_hidden, torch::Tensor front_nodes, torch::Tensor ancestors, torch::Tensor best,
               torch::Tensor best_prev, torch::Tensor layer_top, torch::Tensor delta_rows, torch::Tensor deltas_out,
               torch::Tensor counter) {
  const at::cuda::CUDAGuard g(probs.device());
  TORCH_CHECK(K <= 8 && best.size(1) <= 64 && ancestors.size(2) <= 32);
  auto p = probs.to(torch::kFloat32).contiguous();
  auto tk = toks.to(torch::kInt64).contiguous();
  auto h = hidden.contiguous();
  const int H = h.size(1);
  TORCH_CHECK(H % 8 == 0);
  C10_CUDA_CHECK(launch_pdl(tree_step_kernel, bs, 512, 0, at::cuda::getCurrentCUDAStream().stream(), 
      p.data_ptr<float>(), tk.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(h.data_ptr()), H, K, step,
      layer_start, parent_col, best.size(1), scores.size(1), parents.size(1), ancestors.size(2),
      scores.data_ptr<float>(), tokens.data_ptr<int64_t>(), parents.data_ptr<int64_t>(),
      front_scores.data_ptr<float>(), front_tokens.data_ptr<int64_t>(),
      reinterpret_cast<__nv_bfloat16*>(front_hidden.data_ptr()), front_nodes.data_ptr<int64_t>(),
      ancestors.data_ptr<int>(), best.data_ptr<float>(), best_prev.data_ptr<float>(), layer_top.data_ptr<float>(),
      deltas_out.numel() ? int(deltas_out.size(0)) : 0, deltas_out.numel() ? delta_rows.data_ptr<float>() : nullptr,
      deltas_out.numel() ? deltas_out.data_ptr<float>() : nullptr,
      deltas_out.numel() ? reinterpret_cast<unsigned*>(counter.data_ptr<int>()) : nullptr));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void tree_begin(const torch::Tensor& root_probs, const torch::Tensor& root_tokens, const torch::Tensor& root_hidden,
                int64_t bs, int64_t K, bool keep_order, double root_score, torch::Tensor scores, torch::Tensor tokens,
                torch::Tensor front_scores, torch::Tensor front_tokens, torch::Tensor front_hidden,
                torch::Tensor front_nodes, torch::Tensor best, torch::Tensor best_prev, torch::Tensor layer_top,
                torch::Tensor delta_rows, torch::Tensor deltas_out, torch::Tensor counter) {
  const at::cuda::CUDAGuard g(root_probs.device());
  TORCH_CHECK(K <= 8 && best.size(1) <= 64 && root_probs.is_contiguous() && root_tokens.is_contiguous() &&
              root_hidden.is_contiguous() && root_probs.scalar_type() == torch::kFloat32 &&
              root_tokens.scalar_type() == torch::kInt64);
  const int H = root_hidden.size(1);
  TORCH_CHECK(H % 8 == 0);
  C10_CUDA_CHECK(launch_pdl(tree_begin_kernel, bs, 512, 0, at::cuda::getCurrentCUDAStream().stream(),
      root_probs.data_ptr<float>(), root_tokens.data_ptr<int64_t>(),
      reinterpret_cast<const __nv_bfloat16*>(root_hidden.data_ptr()), H, int(K), int(keep_order), float(root_score),
      int(best.size(1)), int(scores.size(1)), scores.data_ptr<float>(), tokens.data_ptr<int64_t>(),
      front_scores.data_ptr<float>(), front_tokens.data_ptr<int64_t>(),
      reinterpret_cast<__nv_bfloat16*>(front_hidden.data_ptr()), front_nodes.data_ptr<int64_t>(),
      best.data_ptr<float>(), best_prev.data_ptr<float>(), layer_top.data_ptr<float>(),
      deltas_out.numel() ? int(deltas_out.size(0)) : 0, deltas_out.numel() ? delta_rows.data_ptr<float>() : nullptr,
      deltas_out.numel() ? deltas_out.data_ptr<float>() : nullptr,
      deltas_out.numel() ? reinterpret_cast<unsigned*>(counter.data_ptr<int>()) : nullptr));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

std::vector<torch::Tensor> select_rows(const torch::Tensor& scores, const torch::Tensor& decay,
                                       const torch::Tensor& tokens, const torch::Tensor& parents, int64_t bs,
                                       int64_t n, int64_t K, int64_t count) {
  const at::cuda::CUDAGuard g(scores.device());
  TORCH_CHECK(n <= 1024 && count <= 63);
  auto ot = torch::empty({bs, count}, tokens.options());
  auto op = torch::empty({bs, count + 1}, tokens.options().dtype(torch::kInt32));
  auto on = torch::empty({bs, count + 1}, tokens.options());
  C10_CUDA_CHECK(launch_pdl(select_rows_kernel, bs, 256, 0, at::cuda::getCurrentCUDAStream().stream(),
      scores.data_ptr<float>(), decay.data_ptr<float>(), tokens.data_ptr<int64_t>(), parents.data_ptr<int64_t>(), n,
      scores.size(1), parents.size(1), K, count, ot.data_ptr<int64_t>(), op.data_ptr<int>(), on.data_ptr<int64_t>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {ot, op, on};
}

std::vector<torch::Tensor> verify_rows_meta(const torch::Tensor& prow, const torch::Tensor& toks,
                                            const torch::Tensor& root, const torch::Tensor& L,
                                            const torch::Tensor& slot, const torch::Tensor& block_table, int64_t page) {
  const at::cuda::CUDAGuard g(L.device());
  const int bs = prow.size(0), n = prow.size(1);
  TORCH_CHECK(n >= 1 && n <= 64 && prow.scalar_type() == at::kInt && prow.is_contiguous());
  TORCH_CHECK(n == 1 || (toks.size(0) == bs && toks.size(1) == n - 1 && toks.is_contiguous()));
  auto i64 = L.options(), i32 = L.options().dtype(torch::kInt32);
  auto tokens = torch::empty({bs, n}, i64), pos = torch::empty({bs * n}, i64), slots = torch::empty({bs, n}, i64);
  auto extra = torch::empty({bs * n, n}, i32), ne = torch::empty({bs * n}, i32), par = torch::empty({bs * n}, i32);
  auto req = torch::empty({bs * n}, i32), ctx = torch::empty({bs * n}, i32);
  if (bs)
    C10_CUDA_CHECK(launch_pdl(verify_rows_meta_kernel, bs, 64, 0, at::cuda::getCurrentCUDAStream().stream(),
                              prow.data_ptr<int>(), n > 1 ? toks.data_ptr<int64_t>() : nullptr,
                              root.data_ptr<int64_t>(), L.data_ptr<int64_t>(), slot.data_ptr<int>(),
                              block_table.data_ptr<int>(), int(block_table.stride(0)), n, int(page),
                              tokens.data_ptr<int64_t>(), pos.data_ptr<int64_t>(), slots.data_ptr<int64_t>(),
                              extra.data_ptr<int>(), ne.data_ptr<int>(), par.data_ptr<int>(), req.data_ptr<int>(),
                              ctx.data_ptr<int>()));
  return {tokens, pos, slots, extra, ne, par, req, ctx};
}

std::vector<torch::Tensor> draft_step_rows(const torch::Tensor& L, const torch::Tensor& slot,
                                           const torch::Tensor& block_table, torch::Tensor ancestors, int64_t bs,
                                           int64_t K, int64_t s, int64_t page, int64_t window) {
  const at::cuda::CUDAGuard g(L.device());
  TORCH_CHECK(L.scalar_type() == at::kLong && slot.scalar_type() == at::kInt && block_table.scalar_type() == at::kInt);
  TORCH_CHECK(ancestors.scalar_type() == at::kInt && ancestors.is_contiguous() && s >= 1 && s <= ancestors.size(2));
  const int R = int(bs * K);
  auto i64 = L.options(), i32 = L.options().dtype(torch::kInt32);
  auto pos = torch::empty({R}, i64), slots = torch::empty({R}, i64);
  auto req = torch::empty({R}, i32), start = torch::empty({R}, i32), ctx = torch::empty({R}, i32);
  auto extra = torch::empty({R, s}, i32), ne = torch::empty({R}, i32);
  if (R)
    C10_CUDA_CHECK(launch_pdl(draft_step_rows_kernel, (R + 127) / 128, 128, 0, at::cuda::getCurrentCUDAStream().stream(),
                              L.data_ptr<int64_t>(), slot.data_ptr<int>(), block_table.data_ptr<int>(),
                              int(block_table.stride(0)), ancestors.data_ptr<int>(), int(ancestors.size(2)), R, int(K),
                              int(s), int(page), int(window), pos.data_ptr<int64_t>(), req.data_ptr<int>(),
                              slots.data_ptr<int64_t>(), start.data_ptr<int>(), ctx.data_ptr<int>(),
                              extra.data_ptr<int>(), ne.data_ptr<int>()));
  return {pos, req, slots, start, ctx, extra, ne};
}

}  // namespace e4
