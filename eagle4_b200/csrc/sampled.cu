// Sampled draft trees (temperature > 0): children drawn without replacement from the draft's candidate
// distribution, and the recursive tree rejection that keeps the output distribution equal to the target's.
//
// sample_children_kernel  one warp per expanded row: q = softmax(candidate logits / T) over the row's C candidates,
//                         then K draws without replacement as the K largest log q + Gumbel keys (Gumbel-top-k); the
//                         row's q and candidate ids go to the round's q store, each child's candidate slot to the tree.
// sampled_accept_kernel   one CTA per request: walks the verified tree from the root. At a node the target
//                         distribution p = softmax(logits / T) starts as the residual; its verified children are
//                         tried in draw order, child i accepted with probability min(1, r(y) / (m q_i(y))) where q_i
//                         is q without the earlier draws (renormalised) and m the residual mass; a rejection removes
//                         m q_i from the residual. The walk moves to an accepted child; otherwise (or at a leaf, or at
//                         the first child that was not verified, so the tried children are always the first draws)
//                         the final token is drawn from the normalised residual in vocabulary order. This is the
//                         recursion of Recursive Speculative Decoding (Jeon et al., arXiv:2402.14160).
// advance_round_kernel    bumps the round counter that keys the random streams (one launch per round).
//
// Random numbers: SplitMix64 (Vigna's public-domain mixer) of (seed, round, stream, index) -> 24-bit uniforms in
// (0, 1), so a round's draws and coins are reproducible and independent of launch geometry.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace e4 {
namespace {

E4_DEV uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Uniform in (0, 1) from the key (seed, round, stream, index).
E4_DEV float uniform(uint64_t seed, unsigned round, unsigned stream, unsigned index) {
  uint64_t h = mix64(seed ^ (uint64_t(round) << 32 | stream));
  h = mix64(h ^ index);
  return (float(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
}

constexpr int kMaxCandPerLane = 8;  // C <= 256

// rows: R = requests * lanes; row r belongs to request r / lanes and frontier lane r % lanes.
// q store row of an expanded row: b * S + (root ? 0 : 1 + front_nodes[r]). Child node of draw j of lane k:
// child_base + k * K + j (child_base = 0 for the root's children).
__global__ void sample_children_kernel(const float* __restrict__ logits, const int64_t* __restrict__ cand_ids, int R,
                                       int C, int K, int lanes, float inv_t, uint64_t seed,
                                       const unsigned* __restrict__ round_ctr, unsigned stream,
                                       const int64_t* __restrict__ front_nodes, int S, int cap, int child_base,
                                       float* __restrict__ q_store, int* __restrict__ q_ids,
                                       int* __restrict__ node_slot, float* __restrict__ child_p,
                                       int64_t* __restrict__ child_tok) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= R) return;
  const int r = warp, b = r / lanes, k = r % lanes;
  const unsigned rnd = *round_ctr;
  float x[kMaxCandPerLane];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < kMaxCandPerLane; ++i) {
    const int c = lane + 32 * i;
    x[i] = c < C ? logits[size_t(r) * C + c] * inv_t : -INFINITY;
    mx = fmaxf(mx, x[i]);
  }
  mx = warp_max(mx);
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxCandPerLane; ++i) {
    x[i] = (lane + 32 * i < C) ? __expf(x[i] - mx) : 0.f;
    sum += x[i];
  }
  sum = warp_sum(sum);
  const float inv = 1.f / sum;
  const size_t qrow = size_t(b) * S + (front_nodes ? 1 + size_t(front_nodes[r]) : 0);
  float key[kMaxCandPerLane];
#pragma unroll
  for (int i = 0; i < kMaxCandPerLane; ++i) {
    const int c = lane + 32 * i;
    const float q = x[i] * inv;
    x[i] = q;
    if (c < C) {
      q_store[qrow * C + c] = q;
      q_ids[qrow * C + c] = int(cand_ids[size_t(r) * C + c]);
      const float u = uniform(seed, rnd, stream, unsigned(r * C + c));
      key[i] = q > 0.f ? __logf(q) - __logf(-__logf(u)) : -INFINITY;
    } else {
      key[i] = -INFINITY;
    }
  }
  for (int j = 0; j < K; ++j) {
    // warp argmax of the keys (ties to the lower candidate slot)
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxCandPerLane; ++i) {
      const int c = lane + 32 * i;
      if (key[i] > bv || (key[i] == bv && c < bi)) { bv = key[i]; bi = c; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (bi >= C) bi = 0;  // fewer than K candidates with mass: repeat slot 0 with probability 0 below
    if ((bi & 31) == lane) {
      const float q = bv == -INFINITY ? 0.f : x[bi >> 5];
      child_p[size_t(r) * K + j] = q;
      child_tok[size_t(r) * K + j] = cand_ids[size_t(r) * C + bi];
      node_slot[size_t(b) * cap + child_base + k * K + j] = bi;
      key[bi >> 5] = -INFINITY;
    }
  }
}

constexpr int kWalkThreads = 256;
constexpr int kMaxCand = 256;

struct WalkArgs {
  const float* logits;  // [bs * n, ld] target logits of the verify rows
  int ld, V;
  float inv_t;
  const int* row_parent;     // [bs, n] parent row (-1: root)
  const int64_t* row_tok;    // [bs, n]
  const int64_t* row_node;   // [bs, n] tree node of each row (-1: root)
  const float* q_store;      // [bs, S, C]
  const int* q_ids;          // [bs, S, C]
  const int* node_slot;      // [bs, cap]
  int S, C, cap, K, n;
  uint64_t seed;
  const unsigned* round_ctr;
  unsigned stream;
  int64_t* acc;   // [bs, n] accepted rows (root first)
  int* cnt;       // [bs]
  int64_t* bonus; // [bs] final token
  // vocabulary-parallel mode (p_cand != nullptr): the target probabilities at each verify row's candidate ids,
  // normalised over the whole vocabulary, replace the logits; the walk stops before the final draw and leaves the
  // final row and its residual at the candidates (the draw is done by the ranks that hold the vocabulary shards)
  const float* p_cand;  // [bs * n, C]
  int* final_row;       // [bs]
  float* r_final;       // [bs, C]
};

E4_DEV float block_sum_walk(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < kWalkThreads / 32; ++i) s += red[i];
  return s;
}
E4_DEV float block_max_walk(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float s = -INFINITY;
  for (int i = 0; i < kWalkThreads / 32; ++i) s = fmaxf(s, red[i]);
  return s;
}

__global__ void __launch_bounds__(kWalkThreads) sampled_accept_kernel(WalkArgs a) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x, t = threadIdx.x;
  const unsigned rnd = *a.round_ctr;
  __shared__ float red[kWalkThreads / 32];
  __shared__ float r_c[kMaxCand], q_c[kMaxCand];
  __shared__ int id_c[kMaxCand], order[kMaxCand];
  __shared__ float chunk_sum[kWalkThreads];
  __shared__ int s_row, s_len, s_next, s_tok;
  const int* par = a.row_parent + size_t(b) * a.n;
  const int64_t* node = a.row_node + size_t(b) * a.n;
  if (t == 0) { s_row = 0; s_len = 1; a.acc[size_t(b) * a.n] = 0; }
  __syncthreads();
  for (int depth = 0; depth < a.n; ++depth) {
    const int row = s_row;
    const bool sparse = a.p_cand != nullptr;
    const float* lg = sparse ? nullptr : a.logits + (size_t(b) * a.n + row) * a.ld;
    // target distribution at this row: p_v = exp(l_v / T - mx) / z
    float mx = 0.f, iz = 0.f;
    if (!sparse) {
      mx = -INFINITY;
      for (int v = t; v < a.V; v += kWalkThreads) mx = fmaxf(mx, lg[v] * a.inv_t);
      mx = block_max_walk(mx, red);
      float z = 0.f;
      for (int v = t; v < a.V; v += kWalkThreads) z += __expf(lg[v] * a.inv_t - mx);
      z = block_sum_walk(z, red);
      iz = 1.f / z;
    }
    const int64_t nd = node[row];
    const size_t qrow = size_t(b) * a.S + (nd < 0 ? 0 : 1 + size_t(nd));
    for (int c = t; c < a.C; c += kWalkThreads) {
      id_c[c] = a.q_ids[qrow * a.C + c];
      q_c[c] = a.q_store[qrow * a.C + c];
      r_c[c] = sparse ? a.p_cand[(size_t(b) * a.n + row) * a.C + c] : __expf(lg[id_c[c]] * a.inv_t - mx) * iz;
    }
    __syncthreads();
    float cand_p = 0.f;
    for (int c = t; c < a.C; c += kWalkThreads) cand_p += r_c[c];
    cand_p = block_sum_walk(cand_p, red);
    const float outside = fmaxf(1.f - cand_p, 0.f);
    // verified children of this row, in draw order, while they are the first draws
    if (t == 0) s_next = -1;
    __syncthreads();
    int expect = 0;
    for (int j = row + 1; j < a.n && s_next < 0; ++j) {
      if (par[j] != row) continue;
      const int64_t cn = node[j];
      const int draw = cn < a.K ? int(cn) : int((cn - a.K) % a.K);
      if (draw != expect) break;
      ++expect;
      const int s = a.node_slot[size_t(b) * a.cap + cn];
      float qs = 0.f, rs = 0.f;
      for (int c = t; c < a.C; c += kWalkThreads) { qs += q_c[c]; rs += r_c[c]; }
      const float qsum = block_sum_walk(qs, red);
      const float m = outside + block_sum_walk(rs, red);
      const float qy = qsum > 0.f ? q_c[s] / qsum : 0.f;
      const float u = uniform(a.seed, rnd, a.stream, unsigned(b * a.n + j));
      if (q_c[s] > 0.f && u * m * qy < r_c[s]) {
        if (t == 0) s_next = j;
      } else {
        // reject: remove m * q_i from the residual, then drop the draw from q
        const float scale = qsum > 0.f ? m / qsum : 0.f;
        __syncthreads();
        for (int c = t; c < a.C; c += kWalkThreads) r_c[c] = fmaxf(r_c[c] - scale * q_c[c], 0.f);
        __syncthreads();
        if (t == 0) q_c[s] = 0.f;
      }
      __syncthreads();
    }
    if (s_next >= 0) {
      if (t == 0) {
        a.acc[size_t(b) * a.n + s_len] = s_next;
        s_len += 1;
        s_row = s_next;
      }
      __syncthreads();
      continue;
    }
    if (sparse) {  // the shards' owners draw: leave the final row and its candidates' residual
      for (int c = t; c < a.C; c += kWalkThreads) a.r_final[size_t(b) * a.C + c] = r_c[c];
      if (t == 0) {
        a.cnt[b] = s_len;
        a.final_row[b] = row;
        a.bonus[b] = -1;
      }
      return;
    }
    // final draw from the residual, in vocabulary order: candidates carry r_c, other ids p_v
    // candidate order by id (C <= 256: rank sort in shared memory)
    // (ties by slot: a row that was never expanded holds a stale candidate list, possibly with repeated ids, and
    // the ranks must still form a permutation)
    for (int c = t; c < a.C; c += kWalkThreads) {
      int rank = 0;
      for (int d = 0; d < a.C; ++d) rank += (id_c[d] < id_c[c]) || (id_c[d] == id_c[c] && d < c);
      order[rank] = c;
    }
    __syncthreads();
    const int chunk = (a.V + kWalkThreads - 1) / kWalkThreads;
    const int v0 = t * chunk, v1 = min(a.V, v0 + chunk);
    // first candidate (in id order) at or after v0
    int lo = 0, hi = a.C;
    while (lo < hi) { const int mid = (lo + hi) >> 1; if (id_c[order[mid]] < v0) lo = mid + 1; else hi = mid; }
    float mine = 0.f;
    int ci = lo;
    for (int v = v0; v < v1; ++v) {
      if (ci < a.C && id_c[order[ci]] == v) {
        mine += r_c[order[ci]];
        do { ++ci; } while (ci < a.C && id_c[order[ci]] == v);  // a repeated id counts once
      } else {
        mine += __expf(lg[v] * a.inv_t - mx) * iz;
      }
    }
    chunk_sum[t] = mine;
    __syncthreads();
    if (t == 0) {
      float total = 0.f;
      for (int i = 0; i < kWalkThreads; ++i) total += chunk_sum[i];
      const float target = uniform(a.seed, rnd, a.stream + 1, unsigned(b)) * total;
      float run = 0.f;
      int owner = kWalkThreads - 1;
      for (int i = 0; i < kWalkThreads; ++i) {
        if (run + chunk_sum[i] > target && chunk_sum[i] > 0.f) { owner = i; break; }
        run += chunk_sum[i];
      }
      chunk_sum[0] = target - run;  // remaining mass inside the owner's chunk
      s_next = owner;
    }
    __syncthreads();
    if (t == s_next) {
      const float rem = chunk_sum[0];
      float run = 0.f;
      int tok = -1, last = -1;
      ci = lo;
      for (int v = v0; v < v1; ++v) {
        float pv;
        if (ci < a.C && id_c[order[ci]] == v) {
          pv = r_c[order[ci]];
          do { ++ci; } while (ci < a.C && id_c[order[ci]] == v);
        } else {
          pv = __expf(lg[v] * a.inv_t - mx) * iz;
        }
        if (pv > 0.f) last = v;
        run += pv;
        if (run > rem && pv > 0.f) { tok = v; break; }
      }
      s_tok = tok >= 0 ? tok : (last >= 0 ? last : v0);
    }
    __syncthreads();
    if (t == 0) {
      a.cnt[b] = s_len;
      a.bonus[b] = s_tok;
    }
    return;
  }
}

// Vocabulary-parallel final draw. The residual of request b's final row over this rank's vocabulary shard
// [lo, lo + Vl): p_v = exp(l_v / T - mx) / z (global row statistics), replaced at candidate ids by the walk's residual
// r_c (a repeated id counts once, with its lowest slot, as in the single-GPU draw).
struct ShardDrawArgs {
  const float* logits;  // [bs * n, ld] this rank's shard of the verify rows' logits
  int ld, Vl, lo;
  float inv_t;
  const float* mx;      // [bs * n] global row max of l / T
  const float* z;       // [bs * n] global row sum of exp(l / T - mx)
  const int* final_row; // [bs]
  const int64_t* row_node;
  const int* q_ids;     // [bs, S, C]
  const float* r_final; // [bs, C]
  int S, C, n, world, rank;
  float* mass;          // [bs] this rank's residual mass (mass kernel) / [world, bs] every rank's (draw kernel)
  uint64_t seed;
  const unsigned* round_ctr;
  unsigned stream;
  int64_t* token;       // [bs] the drawn token on the owning rank, -1 elsewhere
};

// Candidates of the final row that fall in this shard, first occurrence per id (the lowest slot), sorted by id into
// id_s / r_s; returns their count.
E4_DEV int shard_candidates(const ShardDrawArgs& a, int b, int* id_s, float* r_s) {
  __shared__ int n_own;
  __shared__ int all_id[kMaxCand], keep[kMaxCand];
  const int row = a.final_row[b];
  const int64_t nd = a.row_node[size_t(b) * a.n + row];
  const size_t qrow = size_t(b) * a.S + (nd < 0 ? 0 : 1 + size_t(nd));
  if (threadIdx.x == 0) n_own = 0;
  for (int c = threadIdx.x; c < a.C; c += blockDim.x) all_id[c] = a.q_ids[qrow * a.C + c];
  __syncthreads();
  for (int c = threadIdx.x; c < a.C; c += blockDim.x) {
    const int id = all_id[c];
    bool k = id >= a.lo && id < a.lo + a.Vl;
    for (int d = 0; d < c && k; ++d) k = all_id[d] != id;
    keep[c] = k;
  }
  __syncthreads();
  for (int c = threadIdx.x; c < a.C; c += blockDim.x) {
    if (!keep[c]) continue;
    int rank = 0;
    for (int d = 0; d < a.C; ++d) rank += keep[d] && all_id[d] < all_id[c];
    id_s[rank] = all_id[c];
    r_s[rank] = a.r_final[size_t(b) * a.C + c];
    atomicAdd(&n_own, 1);
  }
  __syncthreads();
  return n_own;
}

E4_DEV float shard_p(const ShardDrawArgs& a, const float* lg, size_t grow, int v) {
  return __expf(lg[v] * a.inv_t - a.mx[grow]) / a.z[grow];
}

// One CTA per request: this shard's residual mass of the final row (chunk sums in vocabulary order, then in chunk
// order) into mass[b].
__global__ void __launch_bounds__(kWalkThreads) shard_mass_kernel(ShardDrawArgs a) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x, t = threadIdx.x;
  __shared__ int id_s[kMaxCand];
  __shared__ float r_s[kMaxCand], chunk_sum[kWalkThreads];
  const int m = shard_candidates(a, b, id_s, r_s);
  const size_t grow = size_t(b) * a.n + a.final_row[b];
  const float* lg = a.logits + grow * a.ld;
  const int chunk = (a.Vl + kWalkThreads - 1) / kWalkThreads;
  const int v0 = t * chunk, v1 = min(a.Vl, v0 + chunk);
  int ci = 0;
  while (ci < m && id_s[ci] - a.lo < v0) ++ci;
  float mine = 0.f;
  for (int v = v0; v < v1; ++v) {
    if (ci < m && id_s[ci] - a.lo == v) mine += r_s[ci++];
    else mine += shard_p(a, lg, grow, v);
  }
  chunk_sum[t] = mine;
  __syncthreads();
  if (t == 0) {
    float total = 0.f;
    for (int i = 0; i < kWalkThreads; ++i) total += chunk_sum[i];
    a.mass[b] = total;
  }
}

// One CTA per request: target = u * (sum of every rank's mass, rank order); the rank whose cumulative mass passes the
// target scans its shard in vocabulary order for the token; the others write -1.
__global__ void __launch_bounds__(kWalkThreads) shard_draw_kernel(ShardDrawArgs a, int bs) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x, t = threadIdx.x;
  __shared__ int id_s[kMaxCand];
  __shared__ float r_s[kMaxCand], chunk_sum[kWalkThreads];
  __shared__ int s_owner, s_tok;
  __shared__ float s_rem;
  const unsigned rnd = *a.round_ctr;
  if (t == 0) {
    float total = 0.f;
    for (int r = 0; r < a.world; ++r) total += a.mass[size_t(r) * bs + b];
    const float target = uniform(a.seed, rnd, a.stream + 1, unsigned(b)) * total;
    float run = 0.f;
    int owner = -1;
    for (int r = 0; r < a.world; ++r) {
      const float mr = a.mass[size_t(r) * bs + b];
      if (mr > 0.f) owner = r;  // the last rank with mass takes a target at the very end
      if (run + mr > target && mr > 0.f) { owner = r; break; }
      run += mr;
    }
    s_owner = owner;
    s_rem = target - run;
    s_tok = -1;
  }
  __syncthreads();
  if (s_owner != a.rank) {
    if (t == 0) a.token[b] = -1;
    return;
  }
  const int m = shard_candidates(a, b, id_s, r_s);
  const size_t grow = size_t(b) * a.n + a.final_row[b];
  const float* lg = a.logits + grow * a.ld;
  const int chunk = (a.Vl + kWalkThreads - 1) / kWalkThreads;
  const int v0 = t * chunk, v1 = min(a.Vl, v0 + chunk);
  int ci0 = 0;
  while (ci0 < m && id_s[ci0] - a.lo < v0) ++ci0;
  int ci = ci0;
  float mine = 0.f;
  for (int v = v0; v < v1; ++v) {
    if (ci < m && id_s[ci] - a.lo == v) mine += r_s[ci++];
    else mine += shard_p(a, lg, grow, v);
  }
  chunk_sum[t] = mine;
  __syncthreads();
  if (t == 0) {
    float run = 0.f;
    int own = kWalkThreads - 1;
    for (int i = 0; i < kWalkThreads; ++i) {
      if (run + chunk_sum[i] > s_rem && chunk_sum[i] > 0.f) { own = i; break; }
      run += chunk_sum[i];
    }
    chunk_sum[0] = s_rem - run;
    s_owner = own;
  }
  __syncthreads();
  if (t == s_owner) {
    const float rem = chunk_sum[0];
    float run = 0.f;
    int tok = -1, last = -1;
    ci = ci0;
    for (int v = v0; v < v1; ++v) {
      float pv;
      if (ci < m && id_s[ci] - a.lo == v) pv = r_s[ci++];
      else pv = shard_p(a, lg, grow, v);
      if (pv > 0.f) last = v;
      run += pv;
      if (run > rem && pv > 0.f) { tok = v; break; }
    }
    s_tok = a.lo + (tok >= 0 ? tok : (last >= 0 ? last : v0));
  }
  __syncthreads();
  if (t == 0) a.token[b] = s_tok;
}

__global__ void advance_round_kernel(unsigned* ctr) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) *ctr += 1u;
}

}  // namespace

// Draws K children per row; returns (child probs [R, K] fp32, child tokens [R, K] int64). ``front_nodes`` None:
// the rows are the requests' roots (lanes = 1).
std::vector<torch::Tensor> sample_children(const torch::Tensor& logits, const torch::Tensor& cand_ids, int64_t K,
                                           double temperature, int64_t seed, const torch::Tensor& round_ctr,
                                           int64_t stream, const c10::optional<torch::Tensor>& front_nodes,
                                           int64_t lanes, torch::Tensor q_store, torch::Tensor q_ids,
                                           torch::Tensor node_slot, int64_t child_base) {
  const at::cuda::CUDAGuard g(logits.device());
  TORCH_CHECK(logits.dim() == 2 && logits.scalar_type() == at::kFloat && logits.is_contiguous());
  const int R = logits.size(0), C = logits.size(1);
  TORCH_CHECK(C <= 32 * kMaxCandPerLane && K >= 1 && K <= C, "sample_children: 1 <= K <= C <= 256");
  TORCH_CHECK(q_store.dim() == 3 && q_store.size(2) == C && q_ids.sizes() == q_store.sizes());
  auto cp = torch::empty({R, K}, logits.options());
  auto ct = torch::empty({R, K}, cand_ids.options());
  const bool fn = front_nodes.has_value() && front_nodes->defined();
  if (R)
    C10_CUDA_CHECK(launch_pdl(sample_children_kernel, (R * 32 + 255) / 256, 256, 0,
                              at::cuda::getCurrentCUDAStream().stream(), logits.data_ptr<float>(),
                              cand_ids.data_ptr<int64_t>(), R, C, int(K), int(lanes), float(1.0 / temperature),
                              uint64_t(seed), reinterpret_cast<const unsigned*>(round_ctr.data_ptr<int>()),
                              unsigned(stream), fn ? front_nodes->data_ptr<int64_t>() : nullptr,
                              int(q_store.size(1)), int(node_slot.size(1)), int(child_base),
                              q_store.data_ptr<float>(), q_ids.data_ptr<int>(), node_slot.data_ptr<int>(),
                              cp.data_ptr<float>(), ct.data_ptr<int64_t>()));
  return {cp, ct};
}

// Tree rejection over the verify rows; returns (accepted rows [bs, n] int64, counts [bs] int32, final token [bs]).
std::vector<torch::Tensor> sampled_accept(const torch::Tensor& logits, double temperature,
                                          const torch::Tensor& row_parent, const torch::Tensor& row_tok,
                                          const torch::Tensor& row_node, const torch::Tensor& q_store,
                                          const torch::Tensor& q_ids, const torch::Tensor& node_slot, int64_t K,
                                          int64_t seed, const torch::Tensor& round_ctr, int64_t stream) {
  const at::cuda::CUDAGuard g(logits.device());
  const int bs = row_parent.size(0), n = row_parent.size(1);
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1 && logits.size(0) == int64_t(bs) * n);
  TORCH_CHECK(row_parent.scalar_type() == at::kInt && row_parent.is_contiguous());
  TORCH_CHECK(row_node.scalar_type() == at::kLong && row_node.is_contiguous() && row_tok.is_contiguous());
  TORCH_CHECK(q_store.size(2) <= kMaxCand, "sampled_accept: at most 256 candidates");
  auto acc = torch::zeros({bs, n}, row_tok.options());
  auto cnt = torch::zeros({bs}, row_parent.options());
  auto bonus = torch::zeros({bs}, row_tok.options());
  WalkArgs a{};
  a.logits = logits.data_ptr<float>();
  a.ld = int(logits.stride(0));
  a.V = int(logits.size(1));
  a.inv_t = float(1.0 / temperature);
  a.row_parent = row_parent.data_ptr<int>();
  a.row_tok = row_tok.data_ptr<int64_t>();
  a.row_node = row_node.data_ptr<int64_t>();
  a.q_store = q_store.data_ptr<float>();
  a.q_ids = q_ids.data_ptr<int>();
  a.node_slot = node_slot.data_ptr<int>();
  a.S = int(q_store.size(1));
  a.C = int(q_store.size(2));
  a.cap = int(node_slot.size(1));
  a.K = int(K);
  a.n = n;
  a.seed = uint64_t(seed);
  a.round_ctr = reinterpret_cast<const unsigned*>(round_ctr.data_ptr<int>());
  a.stream = unsigned(stream);
  a.acc = acc.data_ptr<int64_t>();
  a.cnt = cnt.data_ptr<int>();
  a.bonus = bonus.data_ptr<int64_t>();
  if (bs)
    C10_CUDA_CHECK(launch_pdl(sampled_accept_kernel, bs, kWalkThreads, 0, at::cuda::getCurrentCUDAStream().stream(),
                              a));
  return {acc, cnt, bonus};
}

// Vocabulary-parallel walk: the tree rejection over the verify rows from the target probabilities at each row's
// candidate ids (``p_cand`` [bs * n, C], normalised over the whole vocabulary). Returns (accepted rows [bs, n],
// counts [bs], final row [bs], residual at the final row's candidates [bs, C]).
std::vector<torch::Tensor> sampled_walk_sparse(const torch::Tensor& p_cand, const torch::Tensor& row_parent,
                                               const torch::Tensor& row_tok, const torch::Tensor& row_node,
                                               const torch::Tensor& q_store, const torch::Tensor& q_ids,
                                               const torch::Tensor& node_slot, int64_t K, int64_t seed,
                                               const torch::Tensor& round_ctr, int64_t stream) {
  const at::cuda::CUDAGuard g(p_cand.device());
  const int bs = row_parent.size(0), n = row_parent.size(1);
  TORCH_CHECK(p_cand.scalar_type() == at::kFloat && p_cand.is_contiguous() && p_cand.size(0) == int64_t(bs) * n &&
              p_cand.size(1) == q_store.size(2), "sampled_walk_sparse: p_cand [bs * n, C] fp32");
  TORCH_CHECK(row_parent.scalar_type() == at::kInt && row_parent.is_contiguous());
  TORCH_CHECK(row_node.scalar_type() == at::kLong && row_node.is_contiguous() && row_tok.is_contiguous());
  TORCH_CHECK(q_store.size(2) <= kMaxCand, "sampled_walk_sparse: at most 256 candidates");
  auto acc = torch::zeros({bs, n}, row_tok.options());
  auto cnt = torch::zeros({bs}, row_parent.options());
  auto bonus = torch::zeros({bs}, row_tok.options());
  auto final_row = torch::zeros({bs}, row_parent.options());
  auto r_final = torch::zeros({bs, q_store.size(2)}, p_cand.options());
  WalkArgs a{};
  a.row_parent = row_parent.data_ptr<int>();
  a.row_tok = row_tok.data_ptr<int64_t>();
  a.row_node = row_node.data_ptr<int64_t>();
  a.q_store = q_store.data_ptr<float>();
  a.q_ids = q_ids.data_ptr<int>();
  a.node_slot = node_slot.data_ptr<int>();
  a.S = int(q_store.size(1));
  a.C = int(q_store.size(2));
  a.cap = int(node_slot.size(1));
  a.K = int(K);
  a.n = n;
  a.seed = uint64_t(seed);
  a.round_ctr = reinterpret_cast<const unsigned*>(round_ctr.data_ptr<int>());
  a.stream = unsigned(stream);
  a.acc = acc.data_ptr<int64_t>();
  a.cnt = cnt.data_ptr<int>();
  a.bonus = bonus.data_ptr<int64_t>();
  a.p_cand = p_cand.data_ptr<float>();
  a.final_row = final_row.data_ptr<int>();
  a.r_final = r_final.data_ptr<float>();
  if (bs)
    C10_CUDA_CHECK(launch_pdl(sampled_accept_kernel, bs, kWalkThreads, 0, at::cuda::getCurrentCUDAStream().stream(),
                              a));
  return {acc, cnt, final_row, r_final};
}

static ShardDrawArgs shard_args(const torch::Tensor& logits, int64_t lo, double temperature, const torch::Tensor& mx,
                                const torch::Tensor& z, const torch::Tensor& final_row, const torch::Tensor& row_node,
                                const torch::Tensor& q_ids, const torch::Tensor& r_final, int64_t S, int64_t n) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1, "shard draw: fp32 logits");
  TORCH_CHECK(mx.is_contiguous() && z.is_contiguous() && final_row.scalar_type() == at::kInt &&
              q_ids.scalar_type() == at::kInt && r_final.is_contiguous());
  ShardDrawArgs a{};
  a.logits = logits.data_ptr<float>();
  a.ld = int(logits.stride(0));
  a.Vl = int(logits.size(1));
  a.lo = int(lo);
  a.inv_t = float(1.0 / temperature);
  a.mx = mx.data_ptr<float>();
  a.z = z.data_ptr<float>();
  a.final_row = final_row.data_ptr<int>();
  a.row_node = row_node.data_ptr<int64_t>();
  a.q_ids = q_ids.data_ptr<int>();
  a.r_final = r_final.data_ptr<float>();
  a.S = int(S);
  a.C = int(r_final.size(1));
  a.n = int(n);
  return a;
}

// This rank's residual mass of each request's final row over its vocabulary shard [lo, lo + Vl): [bs].
torch::Tensor shard_residual_mass(const torch::Tensor& logits, int64_t lo, double temperature, const torch::Tensor& mx,
                                  const torch::Tensor& z, const torch::Tensor& final_row,
                                  const torch::Tensor& row_node, const torch::Tensor& q_ids,
                                  const torch::Tensor& r_final, int64_t S, int64_t n) {
  const at::cuda::CUDAGuard g(logits.device());
  const int bs = final_row.size(0);
  auto mass = torch::zeros({bs}, logits.options());
  ShardDrawArgs a = shard_args(logits, lo, temperature, mx, z, final_row, row_node, q_ids, r_final, S, n);
  a.mass = mass.data_ptr<float>();
  if (bs)
    C10_CUDA_CHECK(launch_pdl(shard_mass_kernel, bs, kWalkThreads, 0, at::cuda::getCurrentCUDAStream().stream(), a));
  return mass;
}

// The final tokens: every rank's masses [world, bs] -> the owning rank's draw from its shard, -1 on the others.
torch::Tensor shard_draw(const torch::Tensor& logits, int64_t lo, double temperature, const torch::Tensor& mx,
                         const torch::Tensor& z, const torch::Tensor& final_row, const torch::Tensor& row_node,
                         const torch::Tensor& q_ids, const torch::Tensor& r_final, int64_t S, int64_t n,
                         const torch::Tensor& masses, int64_t rank, int64_t seed, const torch::Tensor& round_ctr,
                         int64_t stream) {
  const at::cuda::CUDAGuard g(logits.device());
  const int bs = final_row.size(0);
  TORCH_CHECK(masses.dim() == 2 && masses.size(1) == bs && masses.is_contiguous() &&
              masses.scalar_type() == at::kFloat, "shard_draw: masses [world, bs] fp32");
  auto token = torch::empty({bs}, row_node.options());
  ShardDrawArgs a = shard_args(logits, lo, temperature, mx, z, final_row, row_node, q_ids, r_final, S, n);
  a.mass = const_cast<float*>(masses.data_ptr<float>());
  a.world = int(masses.size(0));
  a.rank = int(rank);
  a.seed = uint64_t(seed);
  a.round_ctr = reinterpret_cast<const unsigned*>(round_ctr.data_ptr<int>());
  a.stream = unsigned(stream);
  a.token = token.data_ptr<int64_t>();
  if (bs)
    C10_CUDA_CHECK(launch_pdl(shard_draw_kernel, bs, kWalkThreads, 0, at::cuda::getCurrentCUDAStream().stream(), a,
                              bs));
  return token;
}

void advance_round(torch::Tensor round_ctr) {
  const at::cuda::CUDAGuard g(round_ctr.device());
  C10_CUDA_CHECK(launch_pdl(advance_round_kernel, 1, 32, 0, at::cuda::getCurrentCUDAStream().stream(),
                            reinterpret_cast<unsigned*>(round_ctr.data_ptr<int>())));
}

}  // namespace e4
