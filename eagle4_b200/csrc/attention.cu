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

#include <unordered_map>

#include "common.cuh"

namespace e4 {
namespace {

constexpr int kChunk = 128;   // logical keys per CTA: 4 warps x 32 keys
constexpr int kWarps = 4;
constexpr int kMaxG = 8;      // query heads per kv head handled by one CTA
constexpr int kMaxDPL = 8;    // head dims per lane (D <= 256)

// Chunk partial layout: [rows * Hq][nchunks][D + 4] floats: the D accumulators, then the chunk's max and sum (the
// stride keeps every partial 16-byte aligned).
E4_DEV int part_stride(int D) { return D + 4; }

// Merges ``nheads`` query heads (from ``qh0``) of row ``r`` over their first ``nlc`` chunk partials in chunk order,
// normalises, applies the optional output gate (``out *= sigmoid(gate)``) and writes bf16 outputs. ``w_s`` holds
// 2 * nheads * nlc floats and ``l_s`` nheads floats of shared memory. Partials are read through L2 (other CTAs wrote
// them); the per-chunk weights are computed once per head, and the accumulators' loads are issued 8 chunks at a time.
E4_DEV void merge_heads(const float* ws, int nchunks, int nlc, int D, int Hq, int r, int qh0, int nheads,
                        const __nv_bfloat16* gate, int ldg, __nv_bfloat16* out, float* w_s, float* l_s) {
  const int DS = part_stride(D);
  const size_t rh0 = size_t(r) * Hq + qh0;
  float* m_s = w_s + nheads * nlc;
  for (int i = threadIdx.x; i < nheads * nlc; i += blockDim.x) {
    const int g = i / nlc, c = i % nlc;
    const float* o = ws + ((rh0 + g) * nchunks + c) * DS + D;
    m_s[i] = __ldcg(o);
    w_s[i] = __ldcg(o + 1);  // the chunk's sum for now
  }
  __syncthreads();
  for (int g = threadIdx.x; g < nheads; g += blockDim.x) {
    float M = -INFINITY;
    for (int c = 0; c < nlc; ++c) M = fmaxf(M, m_s[g * nlc + c]);
    float L = 0.f;
    for (int c = 0; c < nlc; ++c) {
      const float mc = m_s[g * nlc + c];
      const float w = mc == -INFINITY ? 0.f : __expf(mc - M);
      L += w_s[g * nlc + c] * w;
      w_s[g * nlc + c] = w;
    }
    l_s[g] = L;
  }
  __syncthreads();
  const int D4 = D / 4;
  for (int it = threadIdx.x; it < nheads * D4; it += blockDim.x) {
    const int g = it / D4, d4 = it % D4;
    const float* base = ws + (rh0 + g) * nchunks * DS + 4 * d4;
    float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c0 = 0; c0 < nlc; c0 += 8) {
      float4 o[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        o[u] = c0 + u < nlc ? __ldcg(reinterpret_cast<const float4*>(base + size_t(c0 + u) * DS))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (c0 + u >= nlc) break;
        const float w = w_s[g * nlc + c0 + u];
        if (w == 0.f) continue;  // empty chunk (its accumulators were never written)
        A.x = fmaf(o[u].x, w, A.x);
        A.y = fmaf(o[u].y, w, A.y);
        A.z = fmaf(o[u].z, w, A.z);
        A.w = fmaf(o[u].w, w, A.w);
      }
    }
    const float L = l_s[g];
    float v[4] = {A.x, A.y, A.z, A.w};
    const size_t rh = rh0 + g;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int d = 4 * d4 + k;
      float x = L > 0.f ? v[k] / L : 0.f;
      if (gate) {
        x = __bfloat162float(__float2bfloat16(x));
        x *= sigmoidf_(__bfloat162float(gate[size_t(r) * ldg + (qh0 + g) * D + d]));
      }
      out[rh * D + d] = __float2bfloat16(x);
    }
  }
}

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
      float* o = ws + ((size_t(r) * Hq + h * G + g) * nchunks + chunk) * part_stride(D);
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
    float* o = ws + ((size_t(r) * Hq + h * G + g) * nchunks + chunk) * part_stride(D);
    o[d] = A;
    if (d == 0) {
      o[D] = M;
      o[D + 1] = L;
    }
  }
}

// ------------------------------------------------------------------------------------------------------------------
// Tensor-core chunk kernel (head dims 128 and 256). One CTA per (chunk, kv head, row), 4 warps:
//   1. the 128 keys' cache slots are resolved (thread t: key t), and each warp copies its 32 keys' K and V rows into
//      shared memory with 16-byte asynchronous copies, straight into the 128-byte-swizzled UMMA layouts (dead keys
//      are zero rows); the G query heads go into a 16-row tile (rows G..15 zero);
//   2. S^T[key, head] = K . Q^T: M = 128 keys, N = 16, K = D (tcgen05.mma, accumulator in TMEM, one thread issues);
//   3. thread t reads key t's 16 scores from TMEM; the chunk's softmax statistics per head (max over the 4 warps in
//      warp order, sum of exp in warp order); P = exp(S - max) is written as bf16 into a K-major tile;
//   4. O^T[d, head] = V^T . P^T: M = 128 head dims per instruction (V read as an MN-major operand), N = 16,
//      K = 128 keys; thread t reads its head dim's 16 outputs and writes the chunk partial;
//   5. the last CTA of (row, kv head) merges the chunks (as in the CUDA-core path).
// The score of a key and its weight in the output depend on that key alone (fixed instruction shapes; the logical
// chunk layout is the same for every batch), so a decoded token and the same token verified in a tree get
// identical outputs.
template <int DPL>
constexpr int tc_smem_bytes() {
  return 2 * (DPL * 32) * 256 + (DPL * 32 / 64) * 2048 + 2 * 2048 + 1024;  // K, V, Q, P tiles + alignment slack
}

E4_DEV uint64_t sdesc_sw128_mn(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= uint64_t((saddr & 0x3FFFFu) >> 4);
  d |= uint64_t((lbo >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

E4_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <int DPL>
__global__ void __launch_bounds__(kWarps * 32)
attn_tc_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ kc,
               const __nv_bfloat16* __restrict__ vc, const int* __restrict__ bt, int bt_ld, int page,
               const int* __restrict__ req, const int* __restrict__ ctx_start, const int* __restrict__ ctx_len,
               const int* __restrict__ extra, int extra_ld, const int* __restrict__ n_extra, float scale, int Hq, int Hk,
               int nchunks, float* __restrict__ ws, int* __restrict__ counters, const __nv_bfloat16* __restrict__ gate,
               int ldg, __nv_bfloat16* __restrict__ out, int* __restrict__ err) {
  constexpr int D = DPL * 32;
  constexpr int KB = D / 64;         // 64-element blocks of the head dim
  constexpr int kTile = 128 * 128;   // bytes of one 64-element block of 128 key rows
  constexpr int NQ = 16;             // query columns per instruction (G padded)
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint64_t mma_bar;
  __shared__ uint32_t tmem_holder;
  __shared__ float red_m[kWarps][kMaxG], red_l[kWarps][kMaxG];
  __shared__ int s_last;
  unsigned char* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  unsigned char* Kt = smem;                    // [KB][128 keys][128 B], K-major SW128
  unsigned char* Vt = smem + D * 256;          // [D/64 atoms][16 key groups][1024 B], MN-major SW128
  unsigned char* Qt = smem + 2 * D * 256;      // [KB][16 heads][128 B], K-major SW128
  unsigned char* Pt = Qt + KB * 2048;          // [2][16 heads][128 B] (keys 0-63, 64-127), K-major SW128
  pdl_wait();
  pdl_trigger();
  const int chunk = blockIdx.x, h = blockIdx.y, r = blockIdx.z;
  const int G = Hq / Hk;
  const int c0 = ctx_start[r], c1 = ctx_len[r], ne = n_extra[r];
  const int nctx = max(c1 - c0, 0);
  const int total = nctx + ne;
  const int nlc = min(max((total + kChunk - 1) / kChunk, 1), nchunks);
  if (chunk >= nlc) {
    if (counters == nullptr) {
      for (int g = threadIdx.x; g < G; g += blockDim.x) {
        float* o = ws + ((size_t(r) * Hq + h * G + g) * nchunks + chunk) * part_stride(D);
        o[D] = -INFINITY;
        o[D + 1] = 0.f;
      }
    }
    return;
  }
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int k_begin = chunk * kChunk;
  const int nk = max(0, min(kChunk, total - k_begin));
  if (warp == 0) tmem_alloc(&tmem_holder, 64);
  if (tid == 32) {
    mbar_init(&mma_bar, 1);
    mbar_fence_init();
  }
  // key tid's cache slot
  const int b = req[r];
  const bool live = tid < nk;
  int64_t slot = 0;
  if (live) {
    const int kk = k_begin + tid;
    if (kk < nctx) {
      const int p = c0 + kk;
      slot = int64_t(bt[size_t(b) * bt_ld + p / page]) * page + p % page;
    } else {
      slot = extra[size_t(r) * extra_ld + (kk - nctx)];
    }
  }
  // K and V rows of the warp's keys: LPR lanes per row (16-byte pieces), RPI rows per pass
  {
    constexpr int LPR = D / 8, RPI = 32 / LPR;
    const int piece = lane % LPR;
    for (int j0 = 0; j0 < 32; j0 += RPI) {
      const int j = j0 + lane / LPR, key = warp * 32 + j;
      const int64_t sj = __shfl_sync(0xffffffffu, slot, j);
      const uint32_t off = uint32_t(piece / 8) * kTile + uint32_t(key) * 128 + uint32_t(((piece & 7) ^ (key & 7)) * 16);
      if (key < nk) {
        const size_t src = (size_t(sj) * Hk + h) * D + piece * 8;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(Kt + off)), "l"(kc + src) : "memory");
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(Vt + off)), "l"(vc + src) : "memory");
      } else {
        *reinterpret_cast<uint4*>(Kt + off) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(Vt + off) = make_uint4(0, 0, 0, 0);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  // query tile: row g = query head h*G + g (bf16 as stored; the scale is applied to the scores)
  {
    const uint4* q4 = reinterpret_cast<const uint4*>(q + (size_t(r) * Hq + h * G) * D);
    for (int i = tid; i < NQ * (D / 8); i += blockDim.x) {
      const int g = i / (D / 8), piece = i % (D / 8);
      const uint4 v = g < G ? q4[g * (D / 8) + piece] : make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(Qt + (piece / 8) * 2048 + g * 128 + ((piece & 7) ^ (g & 7)) * 16) = v;
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  fence_async_smem();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_holder;
  const uint32_t id_s = idesc_bf16_f32(128, NQ);
  if (tid == 0) {
#pragma unroll
    for (int kb = 0; kb < KB; ++kb)
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        umma_bf16(tmem, sdesc_sw128(smem_u32(Kt + kb * kTile + ks * 32)), sdesc_sw128(smem_u32(Qt + kb * 2048 + ks * 32)),
                  id_s, (kb | ks) != 0);
    umma_commit(&mma_bar);
  }
  if (!mbar_wait(&mma_bar, 0)) record_error(err, kErrTimeoutMma);
  tc_fence_after();
  float sv[NQ];
  tmem_ld16(tmem + (uint32_t(warp * 32) << 16), sv);
  // chunk softmax statistics per head
#pragma unroll
  for (int g = 0; g < kMaxG; ++g) {
    if (g >= G) break;
    sv[g] = live ? sv[g] * scale : -INFINITY;
    const float m = warp_max(sv[g]);
    if (lane == 0) red_m[warp][g] = m;
  }
  __syncthreads();
  float pv[NQ];
#pragma unroll
  for (int g = 0; g < NQ; ++g) pv[g] = 0.f;
#pragma unroll
  for (int g = 0; g < kMaxG; ++g) {
    if (g >= G) break;
    float M = red_m[0][g];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) M = fmaxf(M, red_m[w][g]);
    pv[g] = (live && M != -INFINITY) ? __expf(sv[g] - M) : 0.f;
    const float l = warp_sum(pv[g]);
    if (lane == 0) red_l[warp][g] = l;
  }
  // P^T tile: row g holds head g's weights of the 128 keys (two 64-key blocks)
  {
    const int blk = tid / 64, chunk16 = (tid % 64) / 8, e = tid % 8;
#pragma unroll
    for (int g = 0; g < NQ; ++g)
      *reinterpret_cast<__nv_bfloat16*>(Pt + blk * 2048 + g * 128 + ((chunk16 ^ (g & 7)) * 16) + e * 2) =
          __float2bfloat16(pv[g]);
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t id_o = idesc_bf16_f32(128, NQ) | (1u << 15);  // A (V^T) MN-major
  if (tid == 0) {
#pragma unroll
    for (int half = 0; half < D / 128; ++half)
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        umma_bf16(tmem + NQ + half * NQ, sdesc_sw128_mn(smem_u32(Vt + half * 2 * kTile + ks * 2048), kTile, 1024),
                  sdesc_sw128(smem_u32(Pt + (ks / 4) * 2048 + (ks % 4) * 32)), id_o, ks != 0);
    umma_commit(&mma_bar);
  }
  if (!mbar_wait(&mma_bar, 1)) record_error(err, kErrTimeoutMma);
  tc_fence_after();
#pragma unroll
  for (int half = 0; half < D / 128; ++half) {
    float ov[NQ];
    tmem_ld16(tmem + (uint32_t(warp * 32) << 16) + NQ + half * NQ, ov);
    const int d = half * 128 + tid;
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
      if (g >= G) break;
      ws[((size_t(r) * Hq + h * G + g) * nchunks + chunk) * part_stride(D) + d] = ov[g];
    }
  }
  if (tid < G) {
    float M = red_m[0][tid], L = 0.f;
    for (int w = 1; w < kWarps; ++w) M = fmaxf(M, red_m[w][tid]);
    for (int w = 0; w < kWarps; ++w) L += red_l[w][tid];
    float* o = ws + ((size_t(r) * Hq + h * G + tid) * nchunks + chunk) * part_stride(D);
    o[D] = M;
    o[D + 1] = L;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
  if (counters == nullptr) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int prev = atomicAdd(counters + size_t(r) * Hk + h, 1);
    s_last = prev == nlc - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float* w_s = reinterpret_cast<float*>(Kt);
  merge_heads(ws, nchunks, nlc, D, Hq, r, h * G, G, gate, ldg, out, w_s, w_s + 2 * G * nlc);
  if (tid == 0) counters[size_t(r) * Hk + h] = 0;
}

// Merge kernel for launches without the fused merge: one block per (row, query head) over all ``nchunks`` chunks
// (chunks past a row's keys hold an empty partial). Dynamic shared memory: (2 * nchunks + 1) floats.
__global__ void attn_merge_kernel(const float* __restrict__ ws, int nchunks, int D, int Hq,
                                  const __nv_bfloat16* __restrict__ gate, int ldg, __nv_bfloat16* __restrict__ out) {
  extern __shared__ float msm[];
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x / Hq, qh = blockIdx.x % Hq;
  merge_heads(ws, nchunks, nchunks, D, Hq, r, qh, 1, gate, ldg, out, msm, msm + 2 * nchunks);
}

}  // namespace

torch::Tensor gemm_error_word(torch::Device dev);

namespace {
// Per-device arrival counters of the fused chunk merge: allocated zeroed on the first (eager) call, kept for the
// process, and left at zero by every launch. nullptr when ``need`` exceeds them or when they would first be
// allocated inside a stream capture (the caller then merges with attn_merge_kernel).
int* arrival_counters(torch::Device dev, int64_t need) {
  constexpr int64_t kCap = int64_t(1) << 20;
  static std::unordered_map<int, torch::Tensor> per_dev;
  if (need > kCap) return nullptr;
  auto it = per_dev.find(dev.index());
  if (it == per_dev.end()) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    C10_CUDA_CHECK(cudaStreamIsCapturing(at::cuda::getCurrentCUDAStream().stream(), &st));
    if (st != cudaStreamCaptureStatusNone) return nullptr;
    it = per_dev.emplace(dev.index(), torch::zeros({kCap}, torch::TensorOptions().device(dev).dtype(torch::kInt32)))
             .first;
  }
  return it->second.data_ptr<int>();
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
  auto ws = torch::empty({int64_t(T) * Hq * nchunks * (D + 4)}, q.options().dtype(torch::kFloat32));
  auto i32 = [](const torch::Tensor& t) { return t.to(torch::kInt32).contiguous(); };
  auto bt_ = i32(bt), req_ = i32(req), cs = i32(ctx_start), cl = i32(ctx_len), ex = i32(extra), ne = i32(n_extra);
  const __nv_bfloat16* gp = gate ? reinterpret_cast<const __nv_bfloat16*>(gate->data_ptr()) : nullptr;
  const int ldg = gate ? int(gate->stride(0)) : 0;
  if (gate) TORCH_CHECK(gate->stride(1) == 1 && gate->size(0) == T, "attention: gate must be [T, Hq*D] rows");
  const int G = Hq / Hk;
  dim3 grid(nchunks, Hk, T);
  auto stream = at::cuda::getCurrentCUDAStream();
  auto bf = [](const torch::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); };
  __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  int* err = gemm_error_word(q.device()).data_ptr<int>();
  const int dev = q.device().index();
  TORCH_CHECK(dev >= 0 && dev < 64, "attention: device index");
  int* counters = nullptr;
  if (D >= 128) {
    // tensor-core path; the chunk merge runs in the last CTA of each (row, kv head) when its statistics fit in the
    // K tile (D * 256 bytes) and the arrival counters cover T * Hk
    if ((2 * size_t(G) * nchunks + G) * sizeof(float) <= size_t(D) * 256)
      counters = arrival_counters(q.device(), int64_t(T) * Hk);
#define E4_ATTN_TC(DPL)                                                                                            \
  {                                                                                                                \
    static bool attr_set[64] = {};                                                                                 \
    if (!attr_set[dev]) {                                                                                          \
      C10_CUDA_CHECK(cudaFuncSetAttribute(attn_tc_kernel<DPL>, cudaFuncAttributeMaxDynamicSharedMemorySize,        \
                                          tc_smem_bytes<DPL>()));                                                  \
      attr_set[dev] = true;                                                                                        \
    }                                                                                                              \
    C10_CUDA_CHECK(launch_pdl(attn_tc_kernel<DPL>, grid, kWarps * 32, tc_smem_bytes<DPL>(), stream.stream(), bf(q),  \
                              bf(kc), bf(vc), bt_.data_ptr<int>(), int(bt_.size(1)), int(page), req_.data_ptr<int>(), \
                              cs.data_ptr<int>(), cl.data_ptr<int>(), ex.data_ptr<int>(), int(ex.size(1)),         \
                              ne.data_ptr<int>(), float(scale), Hq, Hk, nchunks, ws.data_ptr<float>(), counters,   \
                              gp, ldg, op, err));                                                                  \
  }
    if (D == 128) E4_ATTN_TC(4) else if (D == 256) E4_ATTN_TC(8) else TORCH_CHECK(false, "attention: head dim must be 64, 128 or 256");
#undef E4_ATTN_TC
  } else {
    TORCH_CHECK(D == 64, "attention: head dim must be 64, 128 or 256");
    C10_CUDA_CHECK(launch_pdl(attn_chunk_kernel<2>, grid, kWarps * 32, 0, stream.stream(), bf(q), bf(kc), bf(vc),
                              bt_.data_ptr<int>(), int(bt_.size(1)), int(page), req_.data_ptr<int>(),
                              cs.data_ptr<int>(), cl.data_ptr<int>(), ex.data_ptr<int>(), int(ex.size(1)),
                              ne.data_ptr<int>(), float(scale), Hq, Hk, nchunks, ws.data_ptr<float>()));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (counters == nullptr) {
    const size_t msmem = (2 * size_t(nchunks) + 1) * sizeof(float);
    TORCH_CHECK(msmem <= 200 * 1024, "attention: too many key chunks to merge");
    static bool merge_attr[64] = {};
    if (msmem > 48 * 1024 && !merge_attr[dev]) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(attn_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
      merge_attr[dev] = true;
    }
    C10_CUDA_CHECK(launch_pdl(attn_merge_kernel, T * Hq, 128, msmem, stream.stream(), ws.data_ptr<float>(), nchunks,
                              D, Hq, gp, ldg, op));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return out;
}

}  // namespace e4
