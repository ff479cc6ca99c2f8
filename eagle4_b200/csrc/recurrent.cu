// Recurrent token mixers over draft trees: causal depthwise conv, the gated delta rule (GDN) and the Mamba2
// selective state update.
//
// Tree verify never writes a request's committed state: each row replays its own path (ancestors, then itself)
// from the committed state, so branches never see each other's updates. After acceptance the commit kernels replay
// the accepted path once more, in place. Plain decode is a one-row verify plus its commit. All three modes call the
// same per-step device function, so a token decoded alone and the same token verified in a tree produce identical
// states and outputs. Prefill chains use scan mode (rows of a request in order, state updated in place).
//
// Layouts: GDN state [slots, HV, V, K] fp32 (K contiguous; thread v of a CTA keeps column v in registers);
// Mamba2 state [slots, H, P, N] fp32 (thread p keeps row p); conv windows [slots, C, W-1] (oldest first).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <vector>

#include "common.cuh"

namespace e4 {
namespace {

constexpr int kMaxPath = 64;

__device__ __forceinline__ float bf(__nv_bfloat16 x) { return __bfloat162float(x); }

// ----------------------------------------------------------------------------------------------- causal conv
// out[r, c] = silu(bias[c] + sum_j w[c, j] * window_j) over the row's last W inputs along its parent chain (oldest
// first), taking missing ancestors from the committed window; ``bias`` may be null (no bias).
__global__ void conv_tree_kernel(const __nv_bfloat16* __restrict__ x, int ldx, const __nv_bfloat16* __restrict__ cs,
                                 const int* __restrict__ slot, const int* __restrict__ parent,
                                 const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ bias,
                                 __nv_bfloat16* __restrict__ out, int T, int C, int W) {
  pdl_wait();
  pdl_trigger();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int r = blockIdx.y;
  if (c >= C) return;
  int chain[8];
  int n = 0, cur = r;
  while (cur >= 0 && n < W) {
    chain[n++] = cur;
    cur = parent[cur];
  }
  const int s = slot[r];
  float acc = bias ? bf(bias[c]) : 0.f;
  for (int j = 0; j < W; ++j) {
    // window position j (0 oldest); the newest n entries come from the chain (chain[0] is the row itself)
    const int from_end = W - 1 - j;
    float v;
    if (from_end < n) {
      v = bf(x[size_t(chain[from_end]) * ldx + c]);
    } else {
      const int k = (W - 1) - (from_end - n) - 1;  // column in the committed window
      v = bf(cs[(size_t(s) * C + c) * (W - 1) + k]);
    }
    acc = fmaf(bf(w[size_t(c) * W + j]), v, acc);
  }
  out[size_t(r) * C + c] = __float2bfloat16(silu(acc));
}

// conv window update: append the rows rows[b, :n[b]] (in order) to request b's window
__global__ void conv_commit_kernel(const __nv_bfloat16* __restrict__ x, int ldx, __nv_bfloat16* cs,
                                   const int* __restrict__ slots, const int* __restrict__ rows, int rows_ld,
                                   const int* __restrict__ nrows, int C, int W) {
  pdl_wait();
  pdl_trigger();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (c >= C) return;
  const int n = nrows[b];
  if (n <= 0) return;
  const int s = slots[b];
  __nv_bfloat16 hist[8 + kMaxPath];
  int len = 0;
  for (int k = 0; k < W - 1; ++k) hist[len++] = cs[(size_t(s) * C + c) * (W - 1) + k];
  const int first = max(0, n - (W - 1));
  for (int i = first; i < n; ++i) hist[len++] = x[size_t(rows[size_t(b) * rows_ld + i]) * ldx + c];
  for (int k = 0; k < W - 1; ++k) cs[(size_t(s) * C + c) * (W - 1) + k] = hist[len - (W - 1) + k];
}

// ----------------------------------------------------------------------------------------------- GDN
struct GdnArgs {
  const __nv_bfloat16* qkv;   // post-conv [T, 2*HK*K + HV*V] (row stride ldq)
  int ldq;
  const __nv_bfloat16* proj;  // in_proj output rows: raw b at column b_off, raw a at a_off, z at z_off
  int ldp, z_off, b_off, a_off;
  const float* a_log;         // [HV]
  const float* dt_bias;       // [HV]
  float* state;               // [slots, HV, V, K]
  int HK, HV, K, V;
};

// Decay gate and write strength of (row, value head): g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b).
__device__ __forceinline__ float2 gdn_gate(const GdnArgs& a, int row, int h) {
  const __nv_bfloat16* pr = a.proj + size_t(row) * a.ldp;
  const float g = -__expf(a.a_log[h]) * softplusf_(bf(pr[a.a_off + h]) + a.dt_bias[h]);
  const float beta = sigmoidf_(bf(pr[a.b_off + h]));
  return make_float2(g, beta);
}

constexpr int kGdnTile = 32;  // path nodes staged in shared memory at a time

// Shared-memory staging of up to kGdnTile nodes: l2-normalised q (scaled by K^-1/2) and k of the key head, the
// thread's v value of every node, and the node gates.
template <int K>
struct GdnStage {
  float q[kGdnTile][K];
  float k[kGdnTile][K];
  float v[kGdnTile][128];
  float g[kGdnTile], beta[kGdnTile];
};

// Stage ``n`` (<= kGdnTile) nodes ``rows[0..n)``: warp w normalises nodes w, w+4, ... (fixed-order warp sums).
template <int K>
__device__ __forceinline__ void gdn_stage(const GdnArgs& a, const int* rows, int n, int h, int kh, GdnStage<K>& st) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  constexpr int PL = K / 32;
  for (int j = warp; j < n; j += nw) {
    const int row = rows[j];
    const __nv_bfloat16* base = a.qkv + size_t(row) * a.ldq;
    float qv[PL], kv[PL];
    float q2 = 0.f, k2 = 0.f;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      qv[i] = bf(base[kh * K + lane * PL + i]);
      kv[i] = bf(base[a.HK * K + kh * K + lane * PL + i]);
      q2 = fmaf(qv[i], qv[i], q2);
      k2 = fmaf(kv[i], kv[i], k2);
    }
    const float rq = rsqrtf(warp_sum(q2) + 1e-6f) * rsqrtf(float(K));
    const float rk = rsqrtf(warp_sum(k2) + 1e-6f);
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      st.q[j][lane * PL + i] = qv[i] * rq;
      st.k[j][lane * PL + i] = kv[i] * rk;
    }
    if (lane == 0) {
      const float2 gb = gdn_gate(a, row, h);
      st.g[j] = gb.x;
      st.beta[j] = gb.y;
    }
  }
  for (int i = threadIdx.x; i < n * a.V; i += blockDim.x) {
    const int j = i / a.V, c = i % a.V;
    st.v[j][c] = bf(a.qkv[size_t(rows[j]) * a.ldq + 2 * a.HK * K + h * a.V + c]);
  }
  __syncthreads();
}

template <int K>
__device__ __forceinline__ void load_state(float* S, const float* src) {
#pragma unroll
  for (int i = 0; i < K; i += 4) {
    const float4 t4 = *reinterpret_cast<const float4*>(src + i);
    S[i] = t4.x; S[i + 1] = t4.y; S[i + 2] = t4.z; S[i + 3] = t4.w;
  }
}
template <int K>
__device__ __forceinline__ void save_state(const float* S, float* dst) {
#pragma unroll
  for (int i = 0; i < K; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(S[i], S[i + 1], S[i + 2], S[i + 3]);
}

// Scan mode (prefill chains) with the value dimension split over CTAs: the delta rule's value rows are independent
// (S[v, :] only meets v's own value), so CTA (head, request segment, v-slice) owns kScanV value columns of one head
// and writes the raw output o (bf16); the gated RMSNorm over the head's V values follows as its own kernel.
// kScanLanes lanes share a value column, each holding a 1/kScanLanes slice of the state row S[v, :] (elements
// 4 * kScanLanes * m + 4r + e, e < 4, for lane r of the column: the column's lanes read one contiguous run of a staged
// k / q row, no bank conflicts), so a token step is K / kScanLanes multiply-adds per lane and log2(kScanLanes)
// xor-shuffles per K-long reduction; the CTA's warps spread over the SM's four schedulers.
constexpr int kScanV = 32;
constexpr int kScanLanes = 4;
constexpr int kScanThreads = kScanLanes * kScanV;
template <int K>
struct ScanStage {
  float q[kGdnTile][K];
  float k[kGdnTile][K];
  float v[kGdnTile][kScanV];
  float g[kGdnTile], beta[kGdnTile];
};

// Sum over the kScanLanes lanes of a value column by xor butterflies; every lane gets the same value (each level
// adds two equal-shaped partial sums, and float addition is commutative).
__device__ __forceinline__ float column_sum(float x) {
#pragma unroll
  for (int o = 1; o < kScanLanes; o <<= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Tree mode: one CTA of 4 V threads per (value head, row); the row replays its root-to-row path from the committed
// state without writing it. Value column v has kScanLanes lanes, lane r holding K/4 state elements in groups of four
// at 16m + 4r + e (a column's lanes load one contiguous 64-byte run per group; a staged k / q row is read as
// conflict-free 16-byte pieces), so a node step is K/4 multiply-adds per lane and two xor-shuffle reductions. The
// commit kernel runs this same step, so a row decoded alone, verified in a tree, or committed gives the same state.
template <int K>
__device__ __forceinline__ float gdn_step4(float* S, const GdnStage<K>& st, int j, int v, int r) {
  constexpr int NG = K / 16;
  const float decay = __expf(st.g[j]);
  float kp = 0.f;
#pragma unroll
  for (int m = 0; m < NG; ++m) {
    const float4 kk = *reinterpret_cast<const float4*>(&st.k[j][16 * m + 4 * r]);
    S[4 * m] *= decay;
    S[4 * m + 1] *= decay;
    S[4 * m + 2] *= decay;
    S[4 * m + 3] *= decay;
    kp = fmaf(S[4 * m], kk.x, kp);
    kp = fmaf(S[4 * m + 1], kk.y, kp);
    kp = fmaf(S[4 * m + 2], kk.z, kp);
    kp = fmaf(S[4 * m + 3], kk.w, kp);
  }
  const float delta = (st.v[j][v] - column_sum(kp)) * st.beta[j];
  float op = 0.f;
#pragma unroll
  for (int m = 0; m < NG; ++m) {
    const float4 kk = *reinterpret_cast<const float4*>(&st.k[j][16 * m + 4 * r]);
    const float4 qq = *reinterpret_cast<const float4*>(&st.q[j][16 * m + 4 * r]);
    S[4 * m] = fmaf(kk.x, delta, S[4 * m]);
    S[4 * m + 1] = fmaf(kk.y, delta, S[4 * m + 1]);
    S[4 * m + 2] = fmaf(kk.z, delta, S[4 * m + 2]);
    S[4 * m + 3] = fmaf(kk.w, delta, S[4 * m + 3]);
    op = fmaf(S[4 * m], qq.x, op);
    op = fmaf(S[4 * m + 1], qq.y, op);
    op = fmaf(S[4 * m + 2], qq.z, op);
    op = fmaf(S[4 * m + 3], qq.w, op);
  }
  return column_sum(op);
}

template <int K>
__device__ __forceinline__ void load_state4(float* S, const float* row, int r) {
#pragma unroll
  for (int m = 0; m < K / 16; ++m) {
    const float4 t4 = *reinterpret_cast<const float4*>(row + 16 * m + 4 * r);
    S[4 * m] = t4.x; S[4 * m + 1] = t4.y; S[4 * m + 2] = t4.z; S[4 * m + 3] = t4.w;
  }
}
template <int K>
__device__ __forceinline__ void save_state4(const float* S, float* row, int r) {
#pragma unroll
  for (int m = 0; m < K / 16; ++m)
    *reinterpret_cast<float4*>(row + 16 * m + 4 * r) = make_float4(S[4 * m], S[4 * m + 1], S[4 * m + 2], S[4 * m + 3]);
}

// Tree launches walk chains. A request's rows are contiguous and parents precede children, so its tree splits into
// chains: a chain starts at a root or at a row that is not its parent's first (lowest-index) child and continues
// through first children, one chain per leaf. The CTA of row ``row`` returns if no chain starts there; otherwise
// path[0, pre) receives the chain head's ancestors (root first) and path[pre, len) the chain. Replaying path[] from the
// committed state reaches every chain row by the same step sequence as a root-to-row replay, so each row's state and
// output are those of the row alone, and a tree costs the chain heads' ancestors plus one step per row.
// ``win`` / ``fc`` hold 2 kMaxPath ints: the parents of rows [row - 63, row + 64) and each window row's first child.
__device__ __forceinline__ void chain_walk(const int* __restrict__ parent, int T, int row, int* win, int* fc,
                                           int* path, int* meta) {
  const int lo = max(0, row - (kMaxPath - 1)), hi = min(T, row + kMaxPath);
  const int n = hi - lo;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    win[i] = parent[lo + i];
    fc[i] = 0x7fffffff;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int p = win[i];
    if (p >= lo && p < hi) atomicMin(&fc[p - lo], lo + i);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int p = win[row - lo];
    int len = 0, pre = 0;
    if (!(p >= lo && fc[p - lo] == row)) {
      for (int cur = p; cur >= lo && pre < kMaxPath - 1; cur = win[cur - lo]) ++pre;
      int cur = p;
      for (int i = pre - 1; i >= 0; --i) {
        path[i] = cur;
        cur = win[cur - lo];
      }
      len = pre;
      for (cur = row; cur >= 0 && len < kMaxPath; ++len) {
        path[len] = cur;
        const int c = fc[cur - lo];
        cur = c == 0x7fffffff ? -1 : c;
      }
    }
    meta[0] = len;
    meta[1] = pre;
  }
  __syncthreads();
}

// Gated RMSNorm of the chain rows' raw outputs (orow[c][v], fp32): warp w finishes rows w, w + 16, ..., lane l the
// value columns 4l .. 4l+3. o is rounded to bf16, RMS-normalised over the head's V values (a fixed-order warp sum),
// times w, times silu(z); with no norm weight, the rounded o itself.
__device__ __forceinline__ void gdn_norm_rows(const GdnArgs& a, const int* rows, int n, int h, const float* orow,
                                              const __nv_bfloat16* nw, float eps, __nv_bfloat16* out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  for (int c = warp; c < n; c += nwarps) {
    const int row = rows[c];
    float ob[4];
    float x2 = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int v = 4 * lane + e;
      ob[e] = v < a.V ? __bfloat162float(__float2bfloat16(orow[c * 128 + v])) : 0.f;
      x2 = fmaf(ob[e], ob[e], x2);
    }
    const float rs = rsqrtf(warp_sum(x2) / a.V + eps);
    __nv_bfloat16* o = out + (size_t(row) * a.HV + h) * a.V;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int v = 4 * lane + e;
      if (v >= a.V) continue;
      if (nw == nullptr) {
        o[v] = __float2bfloat16(ob[e]);
      } else {
        const float z = bf(a.proj[size_t(row) * a.ldp + a.z_off + h * a.V + v]);
        o[v] = __float2bfloat16(ob[e] * rs * bf(nw[v]) * silu(z));
      }
    }
  }
}

// Tree mode: one CTA of 4 V threads per (value head, chain); the chain's ancestors and rows are replayed from the
// committed state without writing it (value column v has kScanLanes lanes, lane r holding K/4 state elements in groups
// of four at 16m + 4r + e: a column's lanes load one contiguous 64-byte run per group, and a staged k / q row is read
// as conflict-free 16-byte pieces), the chain rows' raw outputs are kept in shared memory and normalised at the end.
// The commit kernel runs the same step, so a row decoded alone, verified in a tree, or committed gives the same state.
template <int K>
__global__ void __launch_bounds__(512) gdn_kernel(GdnArgs a, const int* __restrict__ slot,
                                                  const int* __restrict__ parent, const __nv_bfloat16* __restrict__ nw,
                                                  float eps, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t gdn_smem[];
  GdnStage<K>& st = *reinterpret_cast<GdnStage<K>*>(gdn_smem);
  float* orow = reinterpret_cast<float*>(gdn_smem + sizeof(GdnStage<K>));  // [kMaxPath][128]
  __shared__ int win[2 * kMaxPath], fc[2 * kMaxPath], path[kMaxPath], meta[2];
  const int h = blockIdx.x;
  const int v = threadIdx.x / kScanLanes, r = threadIdx.x % kScanLanes;
  const int kh = h / (a.HV / a.HK);
  const int vc = min(v, a.V - 1);
  // later rows have the longer ancestor runs in a tree's node order: start them first
  const int row = gridDim.y - 1 - blockIdx.y;
  chain_walk(parent, gridDim.y, row, win, fc, path, meta);
  const int len = meta[0], pre = meta[1];
  if (len == 0) return;
  float S[K / 4];
  load_state4<K>(S, a.state + ((size_t(slot[row]) * a.HV + h) * a.V + vc) * K, r);
  for (int p0 = 0; p0 < len; p0 += kGdnTile) {
    const int n = min(kGdnTile, len - p0);
    if (p0) __syncthreads();
    gdn_stage<K>(a, path + p0, n, h, kh, st);
    for (int j = 0; j < n; ++j) {
      const float o = gdn_step4<K>(S, st, j, vc, r);
      if (p0 + j >= pre && r == 0 && v < a.V) orow[(p0 + j - pre) * 128 + v] = o;
    }
  }
  __syncthreads();
  gdn_norm_rows(a, path + pre, len - pre, h, orow, nw, eps, out);
}

template <int K>
__global__ void __launch_bounds__(kScanThreads) gdn_scan_kernel(GdnArgs a, const int* __restrict__ slot,
                                                                const int* __restrict__ seg,
                                                                __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t scan_smem[];
  ScanStage<K>& st = *reinterpret_cast<ScanStage<K>*>(scan_smem);
  const int h = blockIdx.x, vs = blockIdx.z * kScanV;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int col = tid / kScanLanes, qr = tid % kScanLanes;
  const int kh = h / (a.HV / a.HK);
  const int v = vs + col;
  const int vc = min(v, a.V - 1);
  constexpr int PL = K / 32;   // elements per lane in the per-token l2 norms
  constexpr int KQ = K / kScanLanes;  // state elements per lane
  constexpr int NG = KQ / 4;          // float4 groups per lane
  constexpr int GS = 4 * kScanLanes;  // floats between a lane's consecutive groups
  const int r0 = seg[blockIdx.y], r1 = seg[blockIdx.y + 1];
  float* stp = a.state + ((size_t(slot[r0]) * a.HV + h) * a.V + vc) * K;
  float S[KQ];
#pragma unroll
  for (int m = 0; m < NG; ++m) {
    const float4 t4 = *reinterpret_cast<const float4*>(stp + GS * m + 4 * qr);
    S[4 * m] = t4.x; S[4 * m + 1] = t4.y; S[4 * m + 2] = t4.z; S[4 * m + 3] = t4.w;
  }
  for (int p0 = r0; p0 < r1; p0 += kGdnTile) {
    const int n = min(kGdnTile, r1 - p0);
    __syncthreads();
    // stage raw q and k of the tile's tokens with independent 16-byte loads (one memory latency for the tile), the
    // slice's v and the gates (thread j: token j), then l2-normalise q (scaled by K^-1/2) and k (warp w: tokens w,
    // w + 4, ...)
    constexpr int VEC = K / 8;  // 16-byte vectors per head row
    for (int e = tid; e < n * 2 * VEC; e += kScanThreads) {
      const int j = e / (2 * VEC), w = e % (2 * VEC), which = w / VEC, c = w % VEC;
      const __nv_bfloat16* base = a.qkv + size_t(p0 + j) * a.ldq + (which ? a.HK * K : 0) + kh * K;
      const uint4 raw = reinterpret_cast<const uint4*>(base)[c];
      const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
      float* dst = which ? &st.k[j][c * 8] : &st.q[j][c * 8];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 f = __bfloat1622float2(p2[t]);
        dst[2 * t] = f.x;
        dst[2 * t + 1] = f.y;
      }
    }
    for (int e = tid; e < n * kScanV; e += kScanThreads) {
      const int j = e / kScanV, c = e % kScanV;
      st.v[j][c] = bf(a.qkv[size_t(p0 + j) * a.ldq + 2 * a.HK * K + h * a.V + min(vs + c, a.V - 1)]);
    }
    if (tid < n) {
      const float2 gb = gdn_gate(a, p0 + tid, h);
      st.g[tid] = gb.x;
      st.beta[tid] = gb.y;
    }
    __syncthreads();
    for (int j = warp; j < n; j += kScanThreads / 32) {
      float q2 = 0.f, k2 = 0.f;
#pragma unroll
      for (int i = 0; i < PL; ++i) {
        const float qv = st.q[j][lane * PL + i], kv = st.k[j][lane * PL + i];
        q2 = fmaf(qv, qv, q2);
        k2 = fmaf(kv, kv, k2);
      }
      const float rq = rsqrtf(warp_sum(q2) + 1e-6f) * rsqrtf(float(K));
      const float rk = rsqrtf(warp_sum(k2) + 1e-6f);
#pragma unroll
      for (int i = 0; i < PL; ++i) {
        st.q[j][lane * PL + i] *= rq;
        st.k[j][lane * PL + i] *= rk;
      }
    }
    __syncthreads();
    for (int j = 0; j < n; ++j) {
      const float decay = __expf(st.g[j]);
      const float4* kr = reinterpret_cast<const float4*>(st.k[j]) + qr;
      const float4* qrow = reinterpret_cast<const float4*>(st.q[j]) + qr;
      float kk[KQ];
      float k0 = 0.f, k1 = 0.f, k2 = 0.f, k3 = 0.f;
#pragma unroll
      for (int m = 0; m < NG; ++m) {
        const float4 t4 = kr[kScanLanes * m];
        kk[4 * m] = t4.x; kk[4 * m + 1] = t4.y; kk[4 * m + 2] = t4.z; kk[4 * m + 3] = t4.w;
        S[4 * m] *= decay;
        S[4 * m + 1] *= decay;
        S[4 * m + 2] *= decay;
        S[4 * m + 3] *= decay;
        k0 = fmaf(S[4 * m], t4.x, k0);
        k1 = fmaf(S[4 * m + 1], t4.y, k1);
        k2 = fmaf(S[4 * m + 2], t4.z, k2);
        k3 = fmaf(S[4 * m + 3], t4.w, k3);
      }
      const float delta = (st.v[j][col] - column_sum((k0 + k1) + (k2 + k3))) * st.beta[j];
      float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
#pragma unroll
      for (int m = 0; m < NG; ++m) {
        const float4 q4 = qrow[kScanLanes * m];
        S[4 * m] = fmaf(kk[4 * m], delta, S[4 * m]);
        S[4 * m + 1] = fmaf(kk[4 * m + 1], delta, S[4 * m + 1]);
        S[4 * m + 2] = fmaf(kk[4 * m + 2], delta, S[4 * m + 2]);
        S[4 * m + 3] = fmaf(kk[4 * m + 3], delta, S[4 * m + 3]);
        o0 = fmaf(S[4 * m], q4.x, o0);
        o1 = fmaf(S[4 * m + 1], q4.y, o1);
        o2 = fmaf(S[4 * m + 2], q4.z, o2);
        o3 = fmaf(S[4 * m + 3], q4.w, o3);
      }
      const float o = column_sum((o0 + o1) + (o2 + o3));
      if (qr == 0 && v < a.V) out[(size_t(p0 + j) * a.HV + h) * a.V + v] = __float2bfloat16(o);
    }
  }
  if (v < a.V) {
#pragma unroll
    for (int m = 0; m < NG; ++m)
      *reinterpret_cast<float4*>(stp + GS * m + 4 * qr) = make_float4(S[4 * m], S[4 * m + 1], S[4 * m + 2], S[4 * m + 3]);
  }
}

// Per-layer pointers of an all-layers commit.
struct GdnLayer {
  const __nv_bfloat16* qkv;   // post-conv rows
  const __nv_bfloat16* proj;  // in_proj output rows (x_pre at column 0, b / a at b_off / a_off)
  float* state;
  __nv_bfloat16* conv_state;
  const float* a_log;
  const float* dt_bias;
};

constexpr int kMaxLayers = 64;
struct GdnLayerTable {
  GdnLayer l[kMaxLayers];
};

// Commit of every GDN layer in one launch: CTA (value head x 32-column slice, request, layer) replays rows[b, :n[b]]
// in place with the tree kernel's step (value columns are independent, so a slice needs only its own columns).
constexpr int kCommitV = 32;
template <int K>
__global__ void __launch_bounds__(kScanLanes * kCommitV) gdn_commit_kernel(GdnArgs a,
                                                                           const __grid_constant__ GdnLayerTable layers,
                                                                           const int* __restrict__ slots,
                                                                           const int* __restrict__ rows, int rows_ld,
                                                                           const int* __restrict__ nrows) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t gdn_smem[];
  GdnStage<K>& st = *reinterpret_cast<GdnStage<K>*>(gdn_smem);
  const int slices = (a.V + kCommitV - 1) / kCommitV;
  const int h = blockIdx.x / slices, b = blockIdx.y, l = blockIdx.z;
  const int v = (blockIdx.x % slices) * kCommitV + threadIdx.x / kScanLanes, r = threadIdx.x % kScanLanes;
  const int n = nrows[b];
  if (n <= 0) return;
  const GdnLayer L = layers.l[l];
  a.qkv = L.qkv;
  a.proj = L.proj;
  a.state = L.state;
  a.a_log = L.a_log;
  a.dt_bias = L.dt_bias;
  const int kh = h / (a.HV / a.HK);
  const int vc = min(v, a.V - 1);
  float* stp = a.state + ((size_t(slots[b]) * a.HV + h) * a.V + vc) * K;
  float S[K / 4];
  load_state4<K>(S, stp, r);
  for (int p0 = 0; p0 < n; p0 += kGdnTile) {
    const int m = min(kGdnTile, n - p0);
    if (p0) __syncthreads();
    gdn_stage<K>(a, rows + size_t(b) * rows_ld + p0, m, h, kh, st);
    for (int j = 0; j < m; ++j) gdn_step4<K>(S, st, j, vc, r);
  }
  if (v < a.V) save_state4<K>(S, stp, r);
}

// Conv window update of every layer: append rows[b, :n[b]] of the layer's conv inputs (proj columns [0, C)).
__global__ void conv_commit_all_kernel(const __grid_constant__ GdnLayerTable layers, int ldp, const int* __restrict__ slots,
                                       const int* __restrict__ rows, int rows_ld, const int* __restrict__ nrows,
                                       int C, int W) {
  pdl_wait();
  pdl_trigger();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (c >= C) return;
  const int n = nrows[b];
  if (n <= 0) return;
  const GdnLayer L = layers.l[blockIdx.z];
  const int s = slots[b];
  __nv_bfloat16* cs = L.conv_state;
  __nv_bfloat16 hist[8 + kMaxPath];
  int len = 0;
  for (int k = 0; k < W - 1; ++k) hist[len++] = cs[(size_t(s) * C + c) * (W - 1) + k];
  const int first = max(0, n - (W - 1));
  for (int i = first; i < n; ++i) hist[len++] = L.proj[size_t(rows[size_t(b) * rows_ld + i]) * ldp + c];
  for (int k = 0; k < W - 1; ++k) cs[(size_t(s) * C + c) * (W - 1) + k] = hist[len - (W - 1) + k];
}

// ----------------------------------------------------------------------------------------------- Mamba2
struct MambaArgs {
  const __nv_bfloat16* xbc;  // post-conv [T, H*P + 2*G*N]
  int ldx;
  const __nv_bfloat16* dt;   // raw dt [T, H] (row stride lddt)
  int lddt;
  const float* a_log;
  const float* dt_bias;
  const float* dskip;
  float* state;  // [slots, H, P, N]
  int H, P, N, G;
  int vec;       // rows staged as 16-byte pieces (row stride, offsets and the base 16-byte aligned)
};

// Mamba2 selective-state update along a walk of rows: state_t = exp(A dt_t) state + dt_t x_t B_t^T, and
// y_t = C_t . state_t + D x_t. One CTA of 256 threads per (head, walk): thread (p, q) owns a quarter of state row p in
// groups of four columns at 16m + 4q + e (the row's four owners read one contiguous 64-byte run of a staged B / C row
// per group: conflict-free 16-byte shared-memory reads, broadcast over the warp's eight rows), and the walk's x, B, C
// and gate of each row are staged in shared memory 16 rows at a time (16-byte global loads where the row layout
// allows), so a step is register arithmetic only. y sums each owner's columns in group order, then the owners as
// (q0 + q1) + (q2 + q3); every mode runs this same step, so a row verified in a tree, decoded alone, or committed gives
// identical state and output.
// Walks: kMambaTree - the chain starting at row blockIdx.y (its ancestors without output, then its rows with output;
// parents inside the launch); kMambaCommit - the accepted rows of request blockIdx.y, state written back;
// kMambaScan - the rows of segment blockIdx.y in order (prefill), output for every row, state written back.
enum : int { kMambaTree = 0, kMambaCommit = 1, kMambaScan = 2 };
constexpr int kMambaStage = 16;

template <int N>
__global__ void __launch_bounds__(256) mamba_walk_kernel(MambaArgs a, int mode, const int* __restrict__ slot,
                                                         const int* __restrict__ parent, const int* __restrict__ seg,
                                                         const int* __restrict__ rows, int rows_ld,
                                                         const int* __restrict__ nrows,
                                                         const int64_t* __restrict__ slots,
                                                         __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  constexpr int NQ = N / 4;
  constexpr int RW = 64 + 2 * N;  // staged values per row: x (padded to 64), B, C
  __shared__ int path[kMaxPath], win[2 * kMaxPath], fc[2 * kMaxPath], meta[2];
  __shared__ __align__(16) float sx[kMambaStage][64], sB[kMambaStage][N], sC[kMambaStage][N];
  __shared__ float sda[kMambaStage], sdt[kMambaStage];
  const int h = blockIdx.x, t = threadIdx.x, p = t >> 2, q = t & 3;
  const int grp = h / (a.H / a.G);
  const bool live = p < a.P;
  int state_slot = 0, first = 0, len = 0, pre = 0;
  if (mode == kMambaTree) {
    const int r = blockIdx.y;
    chain_walk(parent, gridDim.y, r, win, fc, path, meta);
    len = meta[0];
    pre = meta[1];
    state_slot = slot[r];
  } else if (mode == kMambaCommit) {
    const int b = blockIdx.y;
    len = min(nrows[b], kMaxPath);
    if (t < len) path[t] = rows[size_t(b) * rows_ld + t];
    state_slot = int(slots[b]);
  } else {
    first = seg[blockIdx.y];
    len = seg[blockIdx.y + 1] - first;
    state_slot = slot[first];
  }
  if (len <= 0) return;
  float* st = a.state + ((size_t(state_slot) * a.H + h) * a.P + (live ? p : 0)) * N + 4 * q;
  float S[NQ];
#pragma unroll
  for (int m = 0; m < NQ / 4; ++m) {
    const float4 v = *reinterpret_cast<const float4*>(st + 16 * m);
    S[4 * m] = v.x; S[4 * m + 1] = v.y; S[4 * m + 2] = v.z; S[4 * m + 3] = v.w;
  }
  const float A = -__expf(a.a_log[h]);
  const float dskip = a.dskip[h];
  for (int c0 = 0; c0 < len; c0 += kMambaStage) {
    const int cn = min(kMambaStage, len - c0);
    __syncthreads();
    if (a.vec) {
      // 16-byte pieces: P/8 of x, N/8 of B, N/8 of C per row
      const int px = a.P / 8, pieces = px + N / 4;
      for (int i = t; i < cn * pieces; i += blockDim.x) {
        const int k = i / pieces, e = i % pieces;
        const int row = mode == kMambaScan ? first + c0 + k : path[c0 + k];
        const __nv_bfloat16* base = a.xbc + size_t(row) * a.ldx;
        const __nv_bfloat16* src;
        float* dst;
        if (e < px) {
          src = base + h * a.P + 8 * e;
          dst = &sx[k][8 * e];
        } else if (e < px + N / 8) {
          src = base + a.H * a.P + grp * N + 8 * (e - px);
          dst = &sB[k][8 * (e - px)];
        } else {
          src = base + a.H * a.P + a.G * N + grp * N + 8 * (e - px - N / 8);
          dst = &sC[k][8 * (e - px - N / 8)];
        }
        const uint4 raw = *reinterpret_cast<const uint4*>(src);
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h2[j]);
          dst[2 * j] = f.x;
          dst[2 * j + 1] = f.y;
        }
      }
    } else {
      for (int i = t; i < cn * RW; i += blockDim.x) {
        const int k = i / RW, e = i % RW;
        const int row = mode == kMambaScan ? first + c0 + k : path[c0 + k];
        const __nv_bfloat16* base = a.xbc + size_t(row) * a.ldx;
        if (e < 64) sx[k][e] = e < a.P ? bf(base[h * a.P + e]) : 0.f;
        else if (e < 64 + N) sB[k][e - 64] = bf(base[a.H * a.P + grp * N + (e - 64)]);
        else sC[k][e - 64 - N] = bf(base[a.H * a.P + a.G * N + grp * N + (e - 64 - N)]);
      }
    }
    if (t < cn) {
      const int row = mode == kMambaScan ? first + c0 + t : path[c0 + t];
      const float dt = softplusf_(bf(a.dt[size_t(row) * a.lddt + h]) + a.dt_bias[h]);
      sdt[t] = dt;
      sda[t] = __expf(dt * A);
    }
    __syncthreads();
    for (int k = 0; k < cn; ++k) {
      const float x = live ? sx[k][p] : 0.f;
      const float da = sda[k], dx = sdt[k] * x;
#pragma unroll
      for (int m = 0; m < NQ / 4; ++m) {
        const float4 b4 = *reinterpret_cast<const float4*>(&sB[k][16 * m + 4 * q]);
        S[4 * m] = fmaf(S[4 * m], da, dx * b4.x);
        S[4 * m + 1] = fmaf(S[4 * m + 1], da, dx * b4.y);
        S[4 * m + 2] = fmaf(S[4 * m + 2], da, dx * b4.z);
        S[4 * m + 3] = fmaf(S[4 * m + 3], da, dx * b4.w);
      }
      const bool emit = mode == kMambaScan || (mode == kMambaTree && c0 + k >= pre);
      if (emit) {
        float y = 0.f;
#pragma unroll
        for (int m = 0; m < NQ / 4; ++m) {
          const float4 c4 = *reinterpret_cast<const float4*>(&sC[k][16 * m + 4 * q]);
          y = fmaf(S[4 * m], c4.x, y);
          y = fmaf(S[4 * m + 1], c4.y, y);
          y = fmaf(S[4 * m + 2], c4.z, y);
          y = fmaf(S[4 * m + 3], c4.w, y);
        }
        y += __shfl_xor_sync(0xffffffffu, y, 1);
        y += __shfl_xor_sync(0xffffffffu, y, 2);
        const int row = mode == kMambaScan ? first + c0 + k : path[c0 + k];
        if (live && q == 0) out[(size_t(row) * a.H + h) * a.P + p] = __float2bfloat16(fmaf(dskip, x, y));
      }
    }
  }
  if (mode != kMambaTree && live) {
#pragma unroll
    for (int m = 0; m < NQ / 4; ++m)
      *reinterpret_cast<float4*>(st + 16 * m) = make_float4(S[4 * m], S[4 * m + 1], S[4 * m + 2], S[4 * m + 3]);
  }
}

torch::Tensor segments_of(const torch::Tensor& slot) {
  // consecutive runs of equal slots (rows of a request are contiguous in scan mode)
  auto s = slot.to(torch::kCPU).to(torch::kInt32).contiguous();
  const int* p = s.data_ptr<int>();
  std::vector<int> seg{0};
  for (int i = 1; i < s.numel(); ++i)
    if (p[i] != p[i - 1]) seg.push_back(i);
  seg.push_back(int(s.numel()));
  return torch::tensor(seg, torch::kInt32).to(slot.device());
}

}  // namespace

#define CBF(t) reinterpret_cast<const __nv_bfloat16*>((t).data_ptr())
#define BFP(t) reinterpret_cast<__nv_bfloat16*>((t).data_ptr())

torch::Tensor conv_tree(const torch::Tensor& x, const torch::Tensor& cs, const torch::Tensor& slot,
                        const torch::Tensor& parent, const torch::Tensor& w, const torch::Tensor& bias) {
  const at::cuda::CUDAGuard g(x.device());
  const int T = x.size(0), C = x.size(1), W = w.size(1);
  TORCH_CHECK(W <= 8 && x.stride(1) == 1);
  TORCH_CHECK(bias.numel() == 0 || (bias.numel() == C && bias.scalar_type() == torch::kBFloat16),
              "conv_tree: the bias has one bf16 value per channel");
  auto out = torch::empty({T, C}, x.options());
  if (T) {
    auto sl = slot.to(torch::kInt32).contiguous(), pa = parent.to(torch::kInt32).contiguous();
    auto wc = w.contiguous();
    auto bc = bias.contiguous();
    const __nv_bfloat16* bp = bias.numel() ? CBF(bc) : nullptr;
    C10_CUDA_CHECK(launch_pdl(conv_tree_kernel, dim3((C + 255) / 256, T), 256, 0, at::cuda::getCurrentCUDAStream().stream(), 
        CBF(x), x.stride(0), CBF(cs), sl.data_ptr<int>(), pa.data_ptr<int>(), CBF(wc), bp, BFP(out), T, C, W));
  }
  return out;
}

void conv_commit(const torch::Tensor& x, torch::Tensor cs, const torch::Tensor& slots, const torch::Tensor& rows,
                 const torch::Tensor& nrows, int64_t W) {
  const at::cuda::CUDAGuard g(x.device());
  const int B = rows.size(0), C = x.size(1);
  TORCH_CHECK(x.stride(1) == 1 && rows.size(1) <= kMaxPath);
  if (!B) return;
  auto sl = slots.to(torch::kInt32).contiguous(), rw = rows.to(torch::kInt32).contiguous(),
       nr = nrows.to(torch::kInt32).contiguous();
  C10_CUDA_CHECK(launch_pdl(conv_commit_kernel, dim3((C + 255) / 256, B), 256, 0, at::cuda::getCurrentCUDAStream().stream(), 
      CBF(x), x.stride(0), BFP(cs), sl.data_ptr<int>(), rw.data_ptr<int>(), rw.size(1), nr.data_ptr<int>(), C, W));
}

void conv_commit_scan(torch::Tensor cs, const torch::Tensor& x, const torch::Tensor& slot, int64_t W,
                      const torch::Tensor& seg_in) {
  // rows of each request are contiguous: commit the last W-1 rows of every run (segments from the caller's device
  // table when given; otherwise found from the slots on the host)
  const at::cuda::CUDAGuard g(x.device());
  const torch::Tensor seg = seg_in.numel() ? seg_in.to(torch::kInt32) : segments_of(slot);
  const int64_t nseg = seg.numel() - 1;
  if (nseg <= 0) return;
  const int64_t keep = W - 1;
  auto starts = seg.slice(0, 0, nseg), ends = seg.slice(0, 1, nseg + 1);
  auto nrows = at::clamp_max(ends - starts, keep);
  auto k = at::arange(keep, seg.options());
  auto rows = at::minimum((ends - nrows).unsqueeze(1) + k.unsqueeze(0), (ends - 1).unsqueeze(1));
  auto slots = slot.to(torch::kInt32).index_select(0, starts.to(torch::kLong));
  conv_commit(x, cs, slots, rows.contiguous(), nrows.contiguous(), W);
}

template <typename F>
static void gdn_smem_attr(F* fn, size_t bytes) {
  cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
}

static GdnArgs gdn_args(const torch::Tensor& qkv, const torch::Tensor& proj, int64_t z_off, int64_t b_off,
                        int64_t a_off, const torch::Tensor& a_log, const torch::Tensor& dt_bias, torch::Tensor state,
                        int64_t HK, int64_t HV, int64_t K, int64_t V) {
  TORCH_CHECK(qkv.stride(1) == 1 && proj.stride(1) == 1 && state.is_contiguous());
  TORCH_CHECK(V <= 128 && (K == 128 || K == 64), "gdn: K must be 64 or 128 and V <= 128");
  return GdnArgs{CBF(qkv), int(qkv.stride(0)), CBF(proj), int(proj.stride(0)), int(z_off), int(b_off), int(a_off),
                 a_log.data_ptr<float>(), dt_bias.data_ptr<float>(), state.data_ptr<float>(), int(HK), int(HV),
                 int(K), int(V)};
}

torch::Tensor gated_rmsnorm(const torch::Tensor& o, const torch::Tensor& z, const torch::Tensor& w, double eps,
                            bool gate_first);

// Gated delta rule + gated RMSNorm over a forest of rows; returns [T, HV*V].
torch::Tensor gdn_tree(const torch::Tensor& qkv, const torch::Tensor& proj, int64_t z_off, int64_t b_off,
                       int64_t a_off, const torch::Tensor& a_log, const torch::Tensor& dt_bias, torch::Tensor state,
                       const torch::Tensor& slot, const torch::Tensor& parent, const torch::Tensor& norm_w,
                       double eps, int64_t HK, int64_t HV, int64_t K, int64_t V, bool scan,
                       const torch::Tensor& seg_in) {
  const at::cuda::CUDAGuard gd(qkv.device());
  const int T = qkv.size(0);
  auto out = torch::empty({T, HV * V}, qkv.options());
  if (!T) return out;
  GdnArgs a = gdn_args(qkv, proj, z_off, b_off, a_off, a_log, dt_bias, state, HK, HV, K, V);
  auto sl = slot.to(torch::kInt32).contiguous(), pa = parent.to(torch::kInt32).contiguous();
  if (scan) {
    // prefill: value-sliced scan into the raw output, then the gated RMSNorm (skipped for raw callers)
    torch::Tensor seg = seg_in.numel() ? seg_in.to(torch::kInt32).contiguous() : segments_of(sl);
    dim3 grid(HV, seg.numel() - 1, (V + kScanV - 1) / kScanV);
    auto st = at::cuda::getCurrentCUDAStream();
    auto raw = norm_w.numel() ? torch::empty({T, HV * V}, qkv.options()) : out;
    if (K == 128) {
      gdn_smem_attr(gdn_scan_kernel<128>, sizeof(ScanStage<128>));
      C10_CUDA_CHECK(launch_pdl(gdn_scan_kernel<128>, grid, kScanThreads, sizeof(ScanStage<128>), st.stream(), a,
                                sl.data_ptr<int>(), seg.data_ptr<int>(), BFP(raw)));
    } else {
      gdn_smem_attr(gdn_scan_kernel<64>, sizeof(ScanStage<64>));
      C10_CUDA_CHECK(launch_pdl(gdn_scan_kernel<64>, grid, kScanThreads, sizeof(ScanStage<64>), st.stream(), a,
                                sl.data_ptr<int>(), seg.data_ptr<int>(), BFP(raw)));
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    if (!norm_w.numel()) return out;
    return gated_rmsnorm(raw.view({T, HV, V}), proj.narrow(1, z_off, HV * V), norm_w, eps, false);
  }
  TORCH_CHECK(V <= 128, "gdn tree: at most 128 value columns per head");
  dim3 grid(HV, T);
  const int threads = kScanLanes * int(V);
  auto st = at::cuda::getCurrentCUDAStream();
  constexpr size_t kRowOut = size_t(kMaxPath) * 128 * sizeof(float);  // raw outputs of a chain's rows
  if (K == 128) {
    gdn_smem_attr(gdn_kernel<128>, sizeof(GdnStage<128>) + kRowOut);
    C10_CUDA_CHECK(launch_pdl(gdn_kernel<128>, grid, threads, sizeof(GdnStage<128>) + kRowOut, st.stream(), a,
                              sl.data_ptr<int>(), pa.data_ptr<int>(), norm_w.numel() ? CBF(norm_w) : nullptr,
                              float(eps), BFP(out)));
  } else {
    gdn_smem_attr(gdn_kernel<64>, sizeof(GdnStage<64>) + kRowOut);
    C10_CUDA_CHECK(launch_pdl(gdn_kernel<64>, grid, threads, sizeof(GdnStage<64>) + kRowOut, st.stream(), a,
                              sl.data_ptr<int>(), pa.data_ptr<int>(), norm_w.numel() ? CBF(norm_w) : nullptr,
                              float(eps), BFP(out)));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// Commit the accepted rows of every GDN layer (state replay and conv window) in two launches. The per-layer
// tensors are passed by value in a kernel-parameter table (no device-side pointer array to upload, so the call
// can be captured in a CUDA graph); all layers share the row strides of qkv / proj.
void gdn_commit_all(const std::vector<torch::Tensor>& qkv, const std::vector<torch::Tensor>& proj,
                    const std::vector<torch::Tensor>& state, const std::vector<torch::Tensor>& conv_state,
                    const std::vector<torch::Tensor>& a_log, const std::vector<torch::Tensor>& dt_bias, int64_t b_off,
                    int64_t a_off, const torch::Tensor& slots, const torch::Tensor& rows, const torch::Tensor& nrows,
                    int64_t HK, int64_t HV, int64_t K, int64_t V, int64_t C, int64_t W) {
  const at::cuda::CUDAGuard gd(slots.device());
  const int B = rows.size(0), nl = int(qkv.size());
  TORCH_CHECK(nl <= kMaxLayers && rows.size(1) <= kMaxPath);
  if (!B || !nl) return;
  GdnLayerTable tab{};
  for (int i = 0; i < nl; ++i) {
    TORCH_CHECK(qkv[i].stride(0) == qkv[0].stride(0) && proj[i].stride(0) == proj[0].stride(0));
    tab.l[i] = GdnLayer{CBF(qkv[i]), CBF(proj[i]), state[i].data_ptr<float>(), BFP(conv_state[i]),
                        a_log[i].data_ptr<float>(), dt_bias[i].data_ptr<float>()};
  }
  auto sl = slots.to(torch::kInt32).contiguous(), rw = rows.to(torch::kInt32).contiguous(),
       nr = nrows.to(torch::kInt32).contiguous();
  GdnArgs a{nullptr, int(qkv[0].stride(0)), nullptr, int(proj[0].stride(0)), 0, int(b_off), int(a_off), nullptr,
            nullptr, nullptr, int(HK), int(HV), int(K), int(V)};
  auto st = at::cuda::getCurrentCUDAStream();
  dim3 grid(HV * ((V + kCommitV - 1) / kCommitV), B, nl);
  if (K == 128) {
    gdn_smem_attr(gdn_commit_kernel<128>, sizeof(GdnStage<128>));
    C10_CUDA_CHECK(launch_pdl(gdn_commit_kernel<128>, grid, kScanLanes * kCommitV, sizeof(GdnStage<128>), st.stream(), a, tab, sl.data_ptr<int>(), rw.data_ptr<int>(),
                                                                     rw.size(1), nr.data_ptr<int>()));
  } else {
    gdn_smem_attr(gdn_commit_kernel<64>, sizeof(GdnStage<64>));
    C10_CUDA_CHECK(launch_pdl(gdn_commit_kernel<64>, grid, kScanLanes * kCommitV, sizeof(GdnStage<64>), st.stream(), a, tab, sl.data_ptr<int>(), rw.data_ptr<int>(),
                                                                   rw.size(1), nr.data_ptr<int>()));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  C10_CUDA_CHECK(launch_pdl(conv_commit_all_kernel, dim3((C + 255) / 256, B, nl), 256, 0, st.stream(), tab, int(proj[0].stride(0)),
                                                                        sl.data_ptr<int>(), rw.data_ptr<int>(),
                                                                        rw.size(1), nr.data_ptr<int>(), int(C),
                                                                        int(W)));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static MambaArgs mamba_args(const torch::Tensor& xbc, const torch::Tensor& dt, const torch::Tensor& a_log,
                            const torch::Tensor& dt_bias, const torch::Tensor& dskip, torch::Tensor state, int64_t H,
                            int64_t P, int64_t N, int64_t G) {
  TORCH_CHECK(xbc.stride(1) == 1 && dt.stride(1) == 1 && state.is_contiguous());
  TORCH_CHECK(P <= 64 && (N == 128 || N == 64 || N == 16), "mamba: head dim <= 64 and state 16/64/128");
  const bool vec = (reinterpret_cast<uintptr_t>(xbc.data_ptr()) % 16 == 0) && xbc.stride(0) % 8 == 0 && P % 8 == 0 &&
                   (H * P) % 8 == 0 && (G * N) % 8 == 0;
  return MambaArgs{CBF(xbc), int(xbc.stride(0)), CBF(dt), int(dt.stride(0)), a_log.data_ptr<float>(),
                   dt_bias.data_ptr<float>(), dskip.data_ptr<float>(), state.data_ptr<float>(), int(H), int(P),
                   int(N), int(G), int(vec)};
}

#define E4_MAMBA_DISPATCH(N_, ...)                                                                      \
  switch (N_) {                                                                                         \
    case 128: C10_CUDA_CHECK(launch_pdl(mamba_walk_kernel<128>, grid, 256, 0, st.stream(), __VA_ARGS__)); break; \
    case 64: C10_CUDA_CHECK(launch_pdl(mamba_walk_kernel<64>, grid, 256, 0, st.stream(), __VA_ARGS__)); break;   \
    default: C10_CUDA_CHECK(launch_pdl(mamba_walk_kernel<16>, grid, 256, 0, st.stream(), __VA_ARGS__)); break;   \
  }

torch::Tensor mamba_tree(const torch::Tensor& xbc, const torch::Tensor& dt, const torch::Tensor& a_log,
                         const torch::Tensor& dt_bias, const torch::Tensor& dskip, torch::Tensor state,
                         const torch::Tensor& slot, const torch::Tensor& parent, int64_t H, int64_t P, int64_t N,
                         int64_t G, bool scan, const torch::Tensor& seg_in) {
  const at::cuda::CUDAGuard gd(xbc.device());
  const int T = xbc.size(0);
  auto out = torch::empty({T, H, P}, xbc.options());
  if (!T) return out;
  MambaArgs a = mamba_args(xbc, dt, a_log, dt_bias, dskip, state, H, P, N, G);
  auto sl = slot.to(torch::kInt32).contiguous(), pa = parent.to(torch::kInt32).contiguous();
  // tree mode reads no segment table; scan mode takes the caller's device table when given
  torch::Tensor seg = !scan ? torch::Tensor() : (seg_in.numel() ? seg_in.to(torch::kInt32).contiguous() : segments_of(sl));
  dim3 grid(H, scan ? seg.numel() - 1 : T);
  auto st = at::cuda::getCurrentCUDAStream();
  const int* segp = scan ? seg.data_ptr<int>() : nullptr;
  E4_MAMBA_DISPATCH(N, a, scan ? int(kMambaScan) : int(kMambaTree), sl.data_ptr<int>(), pa.data_ptr<int>(), segp,
                    nullptr, 0, nullptr, nullptr, BFP(out))
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

void mamba_commit(const torch::Tensor& xbc, const torch::Tensor& dt, const torch::Tensor& a_log,
                  const torch::Tensor& dt_bias, const torch::Tensor& dskip, torch::Tensor state,
                  const torch::Tensor& slots, const torch::Tensor& rows, const torch::Tensor& nrows, int64_t H,
                  int64_t P, int64_t N, int64_t G) {
  const at::cuda::CUDAGuard gd(xbc.device());
  const int B = rows.size(0);
  if (!B) return;
  TORCH_CHECK(rows.size(1) <= kMaxPath, "mamba_commit: at most 64 accepted rows per request");
  MambaArgs a = mamba_args(xbc, dt, a_log, dt_bias, dskip, state, H, P, N, G);
  auto sl = slots.to(torch::kInt64).contiguous(), rw = rows.to(torch::kInt32).contiguous(),
       nr = nrows.to(torch::kInt32).contiguous();
  dim3 grid(H, B);
  auto st = at::cuda::getCurrentCUDAStream();
  E4_MAMBA_DISPATCH(N, a, int(kMambaCommit), nullptr, nullptr, nullptr, rw.data_ptr<int>(), int(rw.size(1)),
                    nr.data_ptr<int>(), sl.data_ptr<int64_t>(), nullptr)
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace e4
