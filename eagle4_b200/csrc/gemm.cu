// Skinny bf16 GEMM for sm_100a: Y[T, N] = X[T, K] . W[N, K]^T with fused epilogues.
//
// Decode and tree-verify GEMMs have few tokens (T <= 256 per launch) and large weights, so the kernel is
// weight-streaming: the MMA's M dimension walks the weight rows (128 per tile) and the tokens are its N dimension
// ("swap AB"). One persistent CTA per SM, warp-specialised:
//   warp 0      TMA producer: W tile [128 x 64] (evict-first) and X tile [NT x 64] (evict-last) per stage
//   warp 1      TMEM owner and UMMA issuer (tcgen05.mma kind::f16, M=128, N=NT, K=16 per instruction)
//   warps 2..5  epilogue: tcgen05.ld of the fp32 accumulator, fused op, global store
// Two TMEM accumulators let the epilogue of one work unit overlap the MMAs of the next.
//
// A work unit is (weight tile, K split). The split count depends only on (N, K) and the token tile only on T, and
// every output element's reduction order is fixed by the split boundaries, so a row's result is the same whatever
// other rows share the launch (plain decode and tree verify give identical logits). A split tile is finished by the
// CTA holding its first k-block (its range ends there, so that piece is done last): it adds the other pieces in
// split order after a bounded wait on a per-tile count the other pieces bump with release adds.
//
// A consumer GEMM of a normalised input can take the raw residual stream instead (the norm weight folded into W):
// its epilogue warps compute each token's inverse RMS from X while the MMAs run and scale the accumulator by it, so
// the separate RMSNorm launch between the residual update and the next projection disappears.
//
// Epilogues: plain bf16 store; residual add; SwiGLU over gate/up rows interleaved in 64-row blocks; squared ReLU;
// fp32 store; a per-tile (max, argmax) for the vocabulary-parallel greedy head; and the tensor-parallel all-reduce
// (kAllReduce, see tp_finish_tile): a row-parallel projection's partial tile goes out over NVLink as bf16 the moment
// it is finished (so the transfer overlaps the MMAs of the next tiles), the tile is summed over the ranks in rank
// order with the residual added by the CTA that finished it, and the kernel ends only when this rank holds the whole
// reduced output. One-shot: every rank receives every partial and reduces every tile (one NVLink hop; small token
// counts). Two-shot: tile t goes to rank t % world only (reduce-scatter), which reduces it and pushes the result to
// every other rank (all-gather into a local staging area the ranks' CTAs copy out), moving 2 (w-1)/w of the bytes
// the one-shot moves w-1 times (large token counts).
#include <cudaTypedefs.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstdlib>
#include <mutex>
#include <unordered_map>

#include "common.cuh"

namespace e4 {
namespace gemm {

enum Epi : int { kPlain = 0, kResidual = 1, kSwiGLU = 2, kReLU2 = 3, kF32 = 4, kArgmax = 5, kAllReduce = 6 };

constexpr int kMaxRanks = 8;
// peer areas of the all-reduce epilogue: rows per launch (the launch's token chunk) and 128-row weight tiles
constexpr int kTpRows = 256;
constexpr int kTpTiles = 64;
constexpr int kTpPartialFlags = 2 * kTpTiles * kMaxRanks;  // [half][tile][source rank]
constexpr int kTpFlags = kTpPartialFlags + 2 * kTpTiles;     // + gathered-tile flags [half][tile]
constexpr uint64_t kTpWaitNs = 1000000000ull;                // 1 s per wait, then the error word and zeros

constexpr int kThreads = 192;
constexpr int kTileM = 128;
constexpr int kTileK = 64;
constexpr int kWTileBytes = kTileM * kTileK * 2;

struct Params {
  int T, N, K;
  int nt;           // token tile (MMA N): multiple of 16, <= 256
  int n_tiles;      // ceil(N / 128)
  int kb_total;     // ceil(K / 64) k-blocks per tile
  // Work units: (weight tile, token chunk of nt rows), unit = tile * chunks + chunk. Decode and verify launches have
  // one chunk (unit = tile). Prefill launches cover every token in ``chunks`` chunks with CTA ranges aligned to whole
  // units (``aligned``): each unit is one CTA's full-K tile, so no tile is split and nothing is merged.
  int chunks;
  int units;        // n_tiles * chunks
  int aligned;
  long total;       // units * kb_total: the linear k-block space split evenly over the CTAs (stream-K)
  int stages;
  int epi;
  __nv_bfloat16* y;  // [T, ldy] bf16 output (plain / residual / swiglu / relu2)
  float* yf;         // [T, ldy] fp32 output (kF32)
  int ldy;
  const __nv_bfloat16* res;  // residual [T, ldr]
  int ldr;
  float* ws;         // partial tiles [2 * grid][nt][128]
  int* counters;     // [n_tiles] arrival counters (zero between launches)
  float* amax_val;   // [n_tiles][T] per-tile max (kArgmax)
  int* amax_idx;     // [n_tiles][T]
  int* err;
  // kAllReduce: every rank's peer areas (CUDA IPC mappings; this rank's own at index ``rank``):
  //   tp_part[r]  partial tiles sent to rank r: [2 halves][kMaxRanks source ranks][kTpRows][ldp] bf16
  //   tp_gath[r]  reduced tiles pushed to rank r (two-shot): [2 halves][kTpRows][ldp] bf16
  //   tp_flag[r]  rank r's arrival flags: partial [half][tile][source], then gathered [half][tile]; a flag holds
  //               the tag (call number + 1) of the call whose data it announces
  // and this rank's call counter (its low bit is the buffer half of the call) and finished-CTA counter.
  __nv_bfloat16* tp_part[kMaxRanks];
  __nv_bfloat16* tp_gath[kMaxRanks];
  unsigned* tp_flag[kMaxRanks];
  unsigned* tp_calls;
  unsigned* tp_done;
  int ldp, two_shot, world, rank;
  unsigned long long* trace;  // optional [grid][8] globaltimer stamps (tuning runs only)
  // RMSNorm folded into the GEMM (fold != 0): X is the raw residual stream, W carries the norm weight in its columns,
  // and every token column of the accumulator is scaled by rsqrt(mean(x^2) + fold_eps) over that token's row of X
  // (xr: the launch's first row, ldx its stride), computed by the epilogue warps while the MMAs run.
  const __nv_bfloat16* xr;
  int ldx;
  float fold_eps;
  int fold;
  const float* rstd;  // prefill launches: the folded norm's per-token scales for all T rows, computed beforehand
  // 1: every output (and residual) row is 16-byte aligned and whole 8-feature pieces fit in N, so the epilogue
  // stages each 16-token chunk in shared memory and moves it with 16-byte loads and stores (set_vector_epilogue)
  int vec;
};

// trace slots: 0 start, 1 setup done, 2 first stage landed (MMA), 3 last MMA issued, 4 first accumulator ready
// (epilogue), 5 epilogue done, 6 end
#define E4_STAMP(p, k) \
  do { if ((p).trace) (p).trace[size_t(blockIdx.x) * 8 + (k)] = globaltimer(); } while (0)

// Stream-K partition: CTA c owns linear k-blocks [start(c), start(c+1)) of the (tile, k-block) space; a tile is
// split into "pieces" where CTA ranges cut it. The cut points depend only on (N, K, grid), never on T.
__device__ __forceinline__ long sk_start(const Params& p, int c) {
  return p.aligned ? (long(c) * p.units / gridDim.x) * p.kb_total : (long(c) * p.total) / gridDim.x;
}
__device__ __forceinline__ int sk_owner(const Params& p, long g) {  // CTA whose range contains k-block g
  return int(((g + 1) * long(gridDim.x) - 1) / p.total);
}

struct Piece {
  int tile, kb0, kb1;
};

// Partial-tile slot of CTA ``c`` for ``tile``: each CTA has at most two partial pieces, the tile its range starts in
// (slot 2c) and the tile it ends in (slot 2c + 1).
__device__ __forceinline__ int ws_slot(const Params& p, int c, int tile) {
  const int first_tile = int(sk_start(p, c) / p.kb_total);
  return 2 * c + (tile == first_tile ? 0 : 1);
}

// Next piece of this CTA's range at linear position ``g`` (< end).
__device__ __forceinline__ Piece next_piece(const Params& p, long g, long end) {
  Piece pc;
  pc.tile = int(g / p.kb_total);
  pc.kb0 = int(g - long(pc.tile) * p.kb_total);
  const long tile_end = long(pc.tile + 1) * p.kb_total;
  pc.kb1 = int((end < tile_end ? end : tile_end) - long(pc.tile) * p.kb_total);
  return pc;
}

// ------------------------------------------------------------------ tensor-parallel all-reduce epilogue
E4_DEV void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
E4_DEV unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Waits until ``*flag == tag``; false after kTpWaitNs (the caller records the error).
E4_DEV bool tp_wait_flag(const unsigned* flag, unsigned tag) {
  if (ld_acquire_sys(flag) == tag) return true;
  const uint64_t t0 = globaltimer();
  while (ld_acquire_sys(flag) != tag) {
    if (globaltimer() - t0 > kTpWaitNs) return false;
    __nanosleep(64);
  }
  return true;
}
E4_DEV size_t tp_part_index(const Params& p, unsigned half, int src, int row, int n) {
  return ((size_t(half) * kMaxRanks + src) * kTpRows + row) * size_t(p.ldp) + n;
}
E4_DEV int tp_home(const Params& p, int tile) { return p.two_shot ? tile % p.world : -1; }

// 16 token columns of this thread's feature row as bf16 partials to the ranks that reduce ``tile`` (every rank, or
// the tile's home rank). The chunk is transposed through shared memory so that each thread stores 16-byte pieces
// (8 consecutive features of one token) and a warp writes 512 contiguous bytes per token row.
__device__ __forceinline__ void tp_send_chunk(const Params& p, int tile, int m, int j0, const float* v, float* xchg,
                                              int ep_tid, unsigned half) {
  __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(xchg);  // [16 tokens][128 features]
#pragma unroll
  for (int i = 0; i < 16; ++i) st[i * kTileM + m] = __float2bfloat16(v[i]);
  named_bar(1, 128);
  const int home = tp_home(p, tile);
  for (int q = ep_tid; q < 16 * 16; q += 128) {
    const int i = q >> 4, piece = q & 15;
    const int j = j0 + i, n = tile * kTileM + piece * 8;
    if (j >= p.T || n >= p.N) continue;
    const uint4 val = *reinterpret_cast<const uint4*>(st + i * kTileM + piece * 8);
    for (int r = 0; r < p.world; ++r) {
      if (home >= 0 && r != home) continue;
      uint4* dst = reinterpret_cast<uint4*>(p.tp_part[r] + tp_part_index(p, half, p.rank, j, n));
      asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "r"(val.x), "r"(val.y), "r"(val.z),
                   "r"(val.w) : "memory");
    }
  }
  named_bar(1, 128);
}

// After the last chunk of ``tile``: announce it (a release store per destination, after every epilogue thread's
// stores), then, where this rank reduces the tile, wait for every rank's partial and write
// h = residual + sum over ranks in rank order (fp32 sums of the bf16 partials, h rounded once to bf16); two-shot
// also pushes h to every other rank and announces it there.
__device__ __forceinline__ void tp_finish_tile(const Params& p, int tile, int ep_tid, unsigned half, unsigned tag,
                                               int* missing) {
  named_bar(1, 128);
  const int home = tp_home(p, tile);
  if (ep_tid < p.world && (home < 0 || ep_tid == home))
    st_release_sys(p.tp_flag[ep_tid] + (size_t(half) * kTpTiles + tile) * kMaxRanks + p.rank, tag);
  if (home >= 0 && home != p.rank) return;
  if (ep_tid < kMaxRanks) missing[ep_tid] = 0;
  named_bar(1, 128);
  if (ep_tid < p.world) {
    const unsigned* f = p.tp_flag[p.rank] + (size_t(half) * kTpTiles + tile) * kMaxRanks + ep_tid;
    if (!tp_wait_flag(f, tag)) {
      record_error(p.err, kErrTimeoutPeer);
      missing[ep_tid] = 1;  // a rank that never answered contributes zeros
    }
  }
  named_bar(1, 128);
  const __nv_bfloat16* mine = p.tp_part[p.rank];
  for (int q = ep_tid; q < p.T * 16; q += 128) {
    const int j = q >> 4, n = tile * kTileM + (q & 15) * 8;
    if (n >= p.N) continue;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    for (int r = 0; r < p.world; ++r) {
      if (missing[r]) continue;
      const uint4 u = __ldcg(reinterpret_cast<const uint4*>(mine + tp_part_index(p, half, r, j, n)));
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h2[e]);
        acc[2 * e] += f.x;
        acc[2 * e + 1] += f.y;
      }
    }
    const uint4 ru = *reinterpret_cast<const uint4*>(p.res + size_t(j) * p.ldr + n);
    const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&ru);
    uint4 out;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(r2[e]);
      o2[e] = __floats2bfloat162_rn(f.x + acc[2 * e], f.y + acc[2 * e + 1]);
    }
    *reinterpret_cast<uint4*>(p.y + size_t(j) * p.ldy + n) = out;
    if (home >= 0) {
      for (int r = 0; r < p.world; ++r) {
        if (r == p.rank) continue;
        uint4* dst = reinterpret_cast<uint4*>(p.tp_gath[r] + (size_t(half) * kTpRows + j) * p.ldp + n);
        asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "r"(out.x), "r"(out.y), "r"(out.z),
                     "r"(out.w) : "memory");
      }
    }
  }
  if (home >= 0) {
    named_bar(1, 128);
    if (ep_tid < p.world && ep_tid != p.rank)
      st_release_sys(p.tp_flag[ep_tid] + kTpPartialFlags + size_t(half) * kTpTiles + tile, tag);
  }
}

// Two-shot, after this CTA's own tiles: copy the reduced tiles other ranks pushed here into the output (tiles
// c, c + grid, ... of CTA c), each after its arrival flag.
__device__ __forceinline__ void tp_gather_tiles(const Params& p, int ep_tid, unsigned half, unsigned tag,
                                                int* missing) {
  for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
    if (tile % p.world == p.rank) continue;
    if (ep_tid == 0) {
      missing[0] = 0;
      if (!tp_wait_flag(p.tp_flag[p.rank] + kTpPartialFlags + size_t(half) * kTpTiles + tile, tag)) {
        record_error(p.err, kErrTimeoutPeer);
        missing[0] = 1;
      }
    }
    named_bar(1, 128);
    const bool ok = !missing[0];
    for (int q = ep_tid; q < p.T * 16; q += 128) {
      const int j = q >> 4, n = tile * kTileM + (q & 15) * 8;
      if (n >= p.N) continue;
      const uint4 u = ok ? __ldcg(reinterpret_cast<const uint4*>(p.tp_gath[p.rank] + (size_t(half) * kTpRows + j) *
                                                                       p.ldp + n))
                         : make_uint4(0u, 0u, 0u, 0u);
      *reinterpret_cast<uint4*>(p.y + size_t(j) * p.ldy + n) = u;
    }
    named_bar(1, 128);
  }
}

// Vectorised final epilogue of one 16-token chunk: the accumulator values go to shared memory as [token][row]
// fp32, then each thread finishes 8 consecutive features of one token (residual, activation) and moves them with
// 16-byte loads and stores. The per-element arithmetic is the scalar path's (fp32 add, one rounding), so both give
// the same bits.
__device__ __forceinline__ void store_chunk_vec(const Params& p, int tile, int m, int j0, const float* v,
                                                float* xchg, int ep_tid, int row0, int Tu) {
  float* st = xchg;  // [16 tokens][128 rows]
  // this thread's two 8-feature residual pieces are requested before the transpose, so their latency overlaps it
  uint4 rres[2];
  if (p.epi == kResidual) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int q = ep_tid + h * 128, j = j0 + (q >> 4), n = tile * kTileM + (q & 15) * 8;
      rres[h] = (j < Tu && n < p.N) ? *reinterpret_cast<const uint4*>(p.res + size_t(row0 + j) * p.ldr + n)
                                     : make_uint4(0u, 0u, 0u, 0u);
    }
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) st[i * kTileM + m] = v[i];
  named_bar(1, 128);
  if (p.epi == kSwiGLU) {
    // rows [0,64) gate, [64,128) up: 16 tokens x 8 pieces of 8 output features, one piece per thread
    const int i = ep_tid >> 3, piece = ep_tid & 7;
    const int j = j0 + i, f = tile * 64 + piece * 8;
    if (j < Tu && f < p.N / 2) {
      const float* g = st + i * kTileM + piece * 8;
      uint4 out;
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        o2[e] = __floats2bfloat162_rn(silu(g[2 * e]) * g[64 + 2 * e], silu(g[2 * e + 1]) * g[64 + 2 * e + 1]);
      *reinterpret_cast<uint4*>(p.y + size_t(row0 + j) * p.ldy + f) = out;
    }
  } else {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int q = ep_tid + h * 128;
      const int i = q >> 4, piece = q & 15;
      const int j = j0 + i, n = tile * kTileM + piece * 8;
      if (j >= Tu || n >= p.N) continue;
      const float4 lo = *reinterpret_cast<const float4*>(st + i * kTileM + piece * 8);
      const float4 hi = *reinterpret_cast<const float4*>(st + i * kTileM + piece * 8 + 4);
      float a[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
      if (p.epi == kF32) {
        float4* dst = reinterpret_cast<float4*>(p.yf + size_t(row0 + j) * p.ldy + n);
        dst[0] = lo;
        dst[1] = hi;
        continue;
      }
      if (p.epi == kResidual) {
        const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rres[h]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(r2[e]);
          a[2 * e] += f.x;
          a[2 * e + 1] += f.y;
        }
      }
      if (p.epi == kReLU2) {
#pragma unroll
        for (int e = 0; e < 8; ++e) { a[e] = fmaxf(a[e], 0.f); a[e] = a[e] * a[e]; }
      }
      uint4 out;
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
      for (int e = 0; e < 4; ++e) o2[e] = __floats2bfloat162_rn(a[2 * e], a[2 * e + 1]);
      *reinterpret_cast<uint4*>(p.y + size_t(row0 + j) * p.ldy + n) = out;
    }
  }
  named_bar(1, 128);
}

// Partial-tile merge: the 16-token chunk at ``j0`` of weight row ``m`` from pieces 1..count of ``tile`` (the pieces
// of CTAs first + 1 .. first + count), and their sum into ``v`` in piece order.
template <int P>
__device__ __forceinline__ void load_pieces(const Params& p, int first, int count, int tile, int m, int j0,
                                            float4 (&buf)[P][4]) {
#pragma unroll
  for (int qq = 0; qq < P; ++qq) {
    if (qq < count) {
      const float4* src = reinterpret_cast<const float4*>(
          p.ws + size_t(ws_slot(p, first + 1 + qq, tile)) * p.nt * kTileM + size_t(m) * p.nt + j0);
#pragma unroll
      for (int u = 0; u < 4; ++u) buf[qq][u] = __ldcg(src + u);
    }
  }
}
template <int P>
__device__ __forceinline__ void add_pieces(float* v, int count, const float4 (&buf)[P][4]) {
#pragma unroll
  for (int qq = 0; qq < P; ++qq) {
    if (qq < count) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        v[4 * u] += buf[qq][u].x;
        v[4 * u + 1] += buf[qq][u].y;
        v[4 * u + 2] += buf[qq][u].z;
        v[4 * u + 3] += buf[qq][u].w;
      }
    }
  }
}

// Final epilogue of 16 token columns [j0, j0+16) held by this thread for weight row ``m`` of ``tile``.
__device__ __forceinline__ void store_chunk(const Params& p, int tile, int m, int j0, const float* v, float* xchg,
                                            int ep_tid, unsigned half, int row0, int Tu) {
  const int n = tile * kTileM + m;
  if (p.epi == kAllReduce) {
    tp_send_chunk(p, tile, m, j0, v, xchg, ep_tid, half);
    return;
  }
  if (p.vec && p.epi != kArgmax) {
    store_chunk_vec(p, tile, m, j0, v, xchg, ep_tid, row0, Tu);
    return;
  }
  if (p.epi == kSwiGLU) {
    // rows [0,64) are gate, [64,128) the matching up rows; output feature tile*64 + (m & 63)
    if (m >= 64) {
#pragma unroll
      for (int i = 0; i < 16; ++i) xchg[i * 64 + (m - 64)] = v[i];
    }
    named_bar(1, 128);
    if (m < 64) {
      const int f = tile * 64 + m;
      if (f < p.N / 2) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int j = j0 + i;
          if (j < Tu) p.y[size_t(row0 + j) * p.ldy + f] = __float2bfloat16(silu(v[i]) * xchg[i * 64 + m]);
        }
      }
    }
    named_bar(1, 128);
    return;
  }
  if (p.epi == kArgmax) {
    // per token: max over the 128 rows of the tile, ties to the lower row
    const int warp = ep_tid >> 5, lane = ep_tid & 31;
    float* sv = xchg;                                      // [4 warps][16]
    int* si = reinterpret_cast<int*>(xchg + 64);           // [4 warps][16]
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float best = (n < p.N) ? v[i] : -INFINITY;
      int bi = n;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
      }
      if (lane == 0) { sv[warp * 16 + i] = best; si[warp * 16 + i] = bi; }
    }
    named_bar(1, 128);
    if (ep_tid < 16) {
      const int j = j0 + ep_tid;
      float best = -INFINITY;
      int bi = 0x7fffffff;
      for (int w = 0; w < 4; ++w) {
        const float ov = sv[w * 16 + ep_tid];
        const int oi = si[w * 16 + ep_tid];
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
      }
      if (j < p.T) {
        p.amax_val[size_t(tile) * p.T + j] = best;
        p.amax_idx[size_t(tile) * p.T + j] = bi;
      }
    }
    named_bar(1, 128);
    return;
  }
  if (n >= p.N) return;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int j = j0 + i;
    if (j >= Tu) break;
    const size_t row = size_t(row0 + j);
    float a = v[i];
    if (p.epi == kF32) {
      p.yf[row * p.ldy + n] = a;
      continue;
    }
    if (p.epi == kResidual) a += __bfloat162float(p.res[row * p.ldr + n]);
    if (p.epi == kReLU2) { a = fmaxf(a, 0.f); a = a * a; }
    p.y[row * p.ldy + n] = __float2bfloat16(a);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x, Params p) {
  // Setup and the first weight loads happen before waiting for the previous kernel (weights never change); every
  // access to activations (X loads, residual reads, output stores, workspace) comes after pdl_wait().
  pdl_trigger();
  if (threadIdx.x == 0) E4_STAMP(p, 0);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // carve: [stages x (W tile | X tile)] 1024-aligned, then barriers, TMEM handle, exchange buffer
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int x_bytes = p.nt * kTileK * 2;
  const int stage_bytes = kWTileBytes + x_bytes;
  uint8_t* tiles = base;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(tiles + p.stages * stage_bytes);
  uint64_t* empty_bar = full_bar + p.stages;
  uint64_t* acc_full = empty_bar + p.stages;   // [2]
  uint64_t* acc_empty = acc_full + 2;          // [2]
  uint32_t* tmem_handle = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* flag = reinterpret_cast<int*>(tmem_handle + 1);
  float* xchg = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(tmem_handle) + 64);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long g_begin = sk_start(p, blockIdx.x), g_end = sk_start(p, blockIdx.x + 1);
  const uint32_t tmem_cols_per_acc = p.nt;
  uint32_t tmem_cols = 32;
  while (tmem_cols < 2 * tmem_cols_per_acc) tmem_cols <<= 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    mbar_fence_init();
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_x);
  }
  if (warp == 1) tmem_alloc(tmem_handle, tmem_cols);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_handle;
  bool ok = true;
  if (threadIdx.x == 0) E4_STAMP(p, 1);

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      // prologue: weight tiles of the first stages, before the dependency wait
      const int pre = int(g_end - g_begin < long(p.stages) ? g_end - g_begin : long(p.stages));
      // unit u = tile * chunks + chunk: the W tile's rows at (u / chunks) * 128, the X chunk's at (u % chunks) * nt.
      // The (unit, k-block) position advances incrementally: this one thread issues every load, so its loop stays
      // free of divisions (the tile and chunk rows are recomputed only when the unit changes).
      struct Pos {
        int kb, unit, wrow, xrow;
      };
      const int unit0 = int(g_begin / p.kb_total);
      const Pos start{int(g_begin - long(unit0) * p.kb_total), unit0, (unit0 / p.chunks) * kTileM,
                      (unit0 % p.chunks) * p.nt};
      auto advance = [&](Pos& q) {
        if (++q.kb == p.kb_total) {
          q.kb = 0;
          ++q.unit;
          if (p.chunks == 1) {
            q.wrow += kTileM;
          } else {
            q.wrow = (q.unit / p.chunks) * kTileM;
            q.xrow = (q.unit % p.chunks) * p.nt;
          }
        }
      };
      Pos q = start;
      for (int i = 0; i < pre; ++i, advance(q)) {
        mbar_expect_tx(&full_bar[i], stage_bytes);
        tma_load_2d(tiles + i * stage_bytes, &tmap_w, &full_bar[i], q.kb * kTileK, q.wrow, pol_w);
      }
      pdl_wait();
      q = start;
      for (int i = 0; i < pre; ++i, advance(q))
        tma_load_2d(tiles + i * stage_bytes + kWTileBytes, &tmap_x, &full_bar[i], q.kb * kTileK, q.xrow, pol_x);
      stage = pre == p.stages ? 0 : pre;
      phase = pre == p.stages ? 1 : 0;
      for (long gg = g_begin + pre; gg < g_end && ok; ++gg, advance(q)) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1)) { record_error(p.err, kErrTimeoutProducer); ok = false; break; }
        uint8_t* st = tiles + stage * stage_bytes;
        mbar_expect_tx(&full_bar[stage], stage_bytes);
        tma_load_2d(st, &tmap_w, &full_bar[stage], q.kb * kTileK, q.wrow, pol_w);
        tma_load_2d(st + kWTileBytes, &tmap_x, &full_bar[stage], q.kb * kTileK, q.xrow, pol_x);
        if (++stage == p.stages) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kTileM, p.nt);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (long g = g_begin; g < g_end && ok; ++local) {
        const Piece pc = next_piece(p, g, g_end);
        g += pc.kb1 - pc.kb0;
        const int kb0 = pc.kb0, kb1 = pc.kb1;
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1)) { record_error(p.err, kErrTimeoutMma); ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * tmem_cols_per_acc;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase)) { record_error(p.err, kErrTimeoutMma); ok = false; break; }
          if (local == 0 && kb == kb0) E4_STAMP(p, 2);
          tc_fence_after();
          const uint32_t sa = smem_u32(tiles + stage * stage_bytes);
          const uint64_t adesc = sdesc_sw128(sa);
          const uint64_t bdesc = sdesc_sw128(sa + kWTileBytes);
#pragma unroll
          for (int k = 0; k < kTileK / 16; ++k) {
            umma_bf16(d_tmem, adesc + uint64_t(k * 2), bdesc + uint64_t(k * 2), idesc,
                      (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == p.stages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);
      }
      E4_STAMP(p, 3);
    }
  } else {
    // epilogue warps 2..5: TMEM lane quarter = warp % 4
    pdl_wait();
    // kAllReduce: this call's number (its low bit picks the buffer half; number + 1 tags its flags)
    const unsigned call = p.epi == kAllReduce ? *reinterpret_cast<const volatile unsigned*>(p.tp_calls) : 0u;
    const unsigned half = call & 1u, tag = call + 1u;
    int* missing = reinterpret_cast<int*>(xchg + 16 * kTileM + 256);  // [kMaxRanks] flags of absent ranks
    const int ep_tid = threadIdx.x - 64;
    const int quarter = warp & 3;
    const int m = quarter * 32 + lane;
    float* rsv = xchg + 16 * kTileM;  // [nt] folded-norm scales
    if (p.fold && p.rstd == nullptr) {
      // token t's sum of squares: lane partials over 16-byte pieces in index order, then a butterfly (fixed order)
      for (int t = warp - 2; t < p.nt; t += 4) {
        float ss = 0.f;
        if (t < p.T) {
          const uint4* xr = reinterpret_cast<const uint4*>(p.xr + size_t(t) * p.ldx);
#pragma unroll 4
          for (int i = lane; i < p.K / 8; i += 32) {
            const uint4 u = xr[i];
            const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __bfloat1622float2(h2[e]);
              ss = fmaf(f.x, f.x, ss);
              ss = fmaf(f.y, f.y, ss);
            }
          }
        }
        ss = warp_sum(ss);
        if (lane == 0) rsv[t] = t < p.T ? rsqrtf(ss / float(p.K) + p.fold_eps) : 0.f;
      }
      named_bar(1, 128);
    }
    int local = 0;
    for (long g = g_begin; g < g_end; ++local) {
      const Piece pc = next_piece(p, g, g_end);
      g += pc.kb1 - pc.kb0;
      const int tile = pc.tile / p.chunks;               // pc.tile is the work unit
      const int row0 = (pc.tile % p.chunks) * p.nt;     // the unit's first token row
      const int Tu = min(p.nt, p.T - row0);
      const float* rs = p.rstd != nullptr ? p.rstd + row0 : rsv;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&acc_full[acc], acc_phase)) { record_error(p.err, kErrTimeoutEpilogue); break; }
      if (local == 0 && ep_tid == 0) E4_STAMP(p, 4);
      tc_fence_after();
      const uint32_t t_addr = tmem_base + (uint32_t(quarter * 32) << 16) + acc * tmem_cols_per_acc;
      if (pc.kb0 == 0 && pc.kb1 == p.kb_total) {
        for (int j0 = 0; j0 < p.nt; j0 += 16) {
          float v[16];
          tmem_ld16(t_addr + j0, v);
          if (j0 + 16 >= p.nt) { tc_fence_before(); mbar_arrive(&acc_empty[acc]); }
          if (p.fold) {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] *= rs[j0 + i];
          }
          store_chunk(p, tile, m, j0, v, xchg, ep_tid, half, row0, Tu);
        }
        if (p.epi == kAllReduce) tp_finish_tile(p, tile, ep_tid, half, tag, missing);
      } else {
        // Partial tile. The CTA holding the tile's first k-block (kb0 == 0) owns it: that piece ends the CTA's range,
        // so it finishes last. Every other piece stores its partial and counts itself in with a release add (no
        // waiting); the owner keeps its own accumulator in registers, waits for the count, adds the other pieces in
        // piece order and stores the tile.
        const long t0 = long(tile) * p.kb_total;
        const int first_cta = sk_owner(p, t0);
        const int pieces = sk_owner(p, t0 + p.kb_total - 1) - first_cta + 1;
        if (pc.kb0 != 0) {
          // partial slot layout [row m][token j]: each thread writes (and the owner reads) 64 contiguous bytes
          float* part = p.ws + size_t(ws_slot(p, blockIdx.x, tile)) * p.nt * kTileM;
          for (int j0 = 0; j0 < p.nt; j0 += 16) {
            float v[16];
            tmem_ld16(t_addr + j0, v);
            float4* dst = reinterpret_cast<float4*>(part + size_t(m) * p.nt + j0);
#pragma unroll
            for (int u = 0; u < 4; ++u) dst[u] = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
          }
          tc_fence_before();
          mbar_arrive(&acc_empty[acc]);
          named_bar(1, 128);  // every thread's partial stores precede the release below
          if (ep_tid == 0)
            asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(p.counters + tile) : "memory");
        } else {
          if (ep_tid == 0) {
            const int* cnt = p.counters + tile;
            int seen;
            asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(seen) : "l"(cnt) : "memory");
            if (seen < pieces - 1) {
              const uint64_t w0 = globaltimer();
              while (seen < pieces - 1) {
                if (globaltimer() - w0 > kWaitLimitNs) { record_error(p.err, kErrTimeoutEpilogue); break; }
                asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(seen) : "l"(cnt) : "memory");
              }
            }
            E4_STAMP(p, 7);
          }
          named_bar(1, 128);
          auto finish = [&](int j0, float* v) {
            if (p.fold) {
#pragma unroll
              for (int i = 0; i < 16; ++i) v[i] *= rs[j0 + i];
            }
            store_chunk(p, tile, m, j0, v, xchg, ep_tid, half, row0, Tu);
          };
          if (pieces - 1 <= 4) {
            // up to four other pieces: a chunk's pieces are summed as soon as they arrive and the next chunk's loads
            // are issued before this chunk is stored, so each store overlaps the next chunk's memory round trip
            const int others = pieces - 1;
            float4 buf[4][4];
            load_pieces(p, first_cta, others, tile, m, 0, buf);
            for (int j0 = 0; j0 < p.nt; j0 += 16) {
              float v[16];
              tmem_ld16(t_addr + j0, v);
              if (j0 + 16 >= p.nt) { tc_fence_before(); mbar_arrive(&acc_empty[acc]); }
              add_pieces(v, others, buf);
              if (j0 + 16 < p.nt) load_pieces(p, first_cta, others, tile, m, j0 + 16, buf);
              finish(j0, v);
            }
          } else {
            for (int j0 = 0; j0 < p.nt; j0 += 16) {
              float v[16];
              tmem_ld16(t_addr + j0, v);
              if (j0 + 16 >= p.nt) { tc_fence_before(); mbar_arrive(&acc_empty[acc]); }
              // pieces 1.. in order, four at a time: their loads are all issued before the first is summed
              for (int q0 = 1; q0 < pieces; q0 += 4) {
                float4 buf[4][4];
                load_pieces(p, first_cta + q0 - 1, min(4, pieces - q0), tile, m, j0, buf);
                add_pieces(v, min(4, pieces - q0), buf);
              }
              finish(j0, v);
            }
          }
          if (ep_tid == 0) p.counters[tile] = 0;
          named_bar(1, 128);
          if (p.epi == kAllReduce) tp_finish_tile(p, tile, ep_tid, half, tag, missing);
        }
      }
    }
    if (p.epi == kAllReduce && p.two_shot) tp_gather_tiles(p, ep_tid, half, tag, missing);
  }
  if (threadIdx.x == 64) E4_STAMP(p, 5);
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
  if (p.epi == kAllReduce && threadIdx.x == 0) {
    // every CTA read the call number before arriving here: the last one to finish advances it
    __threadfence();
    if (atomicAdd(p.tp_done, 1u) == gridDim.x - 1) {
      *p.tp_done = 0u;
      __threadfence();
      atomicAdd(p.tp_calls, 1u);
    }
  }
  if (threadIdx.x == 0) E4_STAMP(p, 6);
}

// ------------------------------------------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    TORCH_CHECK(ptr != nullptr && q == cudaDriverEntryPointSuccess, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 2-D bf16 row-major [rows, cols] with row stride ``ld`` elements; box [box_cols=64, box_rows], 128-byte swizzle.
CUtensorMap make_map(const void* ptr, int rows, int cols, int ld, int box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
  cuuint32_t box[2] = {cuuint32_t(kTileK), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", int(r));
  return m;
}

struct MapKey {
  const void* p;
  int rows, cols, ld, box;
  bool operator==(const MapKey& o) const {
    return p == o.p && rows == o.rows && cols == o.cols && ld == o.ld && box == o.box;
  }
};
struct MapHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.p) ^ (size_t(k.rows) << 1) ^ (size_t(k.cols) << 21) ^ (size_t(k.box) << 43);
  }
};

const CUtensorMap& weight_map(const void* ptr, int rows, int cols, int ld) {
  static std::unordered_map<MapKey, CUtensorMap, MapHash> cache;
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  MapKey k{ptr, rows, cols, ld, kTileM};
  auto it = cache.find(k);
  if (it == cache.end()) it = cache.emplace(k, make_map(ptr, rows, cols, ld, kTileM)).first;
  return it->second;
}

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// Pipeline depth cap (stages of one W + X tile). E4_GEMM_STAGES overrides it for tuning runs.
int max_stages() {
  static int n = [] {
    const char* e = std::getenv("E4_GEMM_STAGES");
    const int v = e ? std::atoi(e) : 10;
    return v >= 2 && v <= 16 ? v : 10;
  }();
  return n;
}

// Fewest k-blocks (64 x 128 weight tiles) one CTA streams. E4_GEMM_MIN_KB overrides it for tuning runs.
long min_kblocks() {
  static long n = [] {
    const char* e = std::getenv("E4_GEMM_MIN_KB");
    const long v = e ? std::atol(e) : 6;
    return v >= 1 && v <= 64 ? v : 6;
  }();
  return n;
}

// CTAs of a GEMM over ``total`` k-blocks: one per SM, but each streams at least min_kblocks() k-blocks, so a small
// weight is split over fewer CTAs (fewer pieces per tile to add up) instead of one k-block per CTA.
int gemm_grid(long total, int max_ctas) {
  const long by_work = (total + min_kblocks() - 1) / min_kblocks();
  return int(std::max<long>(1, std::min<long>(max_ctas, by_work)));
}

// Whether the launch's outputs allow the vectorised epilogue (16-byte aligned rows, whole 8-feature pieces).
void set_vector_epilogue(Params& p) {
  auto al16 = [](const void* q) { return q != nullptr && (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  bool ok = false;
  if (p.epi == kF32) ok = al16(p.yf) && p.ldy % 4 == 0 && p.N % 8 == 0;
  else if (p.epi == kSwiGLU) ok = al16(p.y) && p.ldy % 8 == 0 && (p.N / 2) % 8 == 0;
  else if (p.epi == kPlain || p.epi == kReLU2) ok = al16(p.y) && p.ldy % 8 == 0 && p.N % 8 == 0;
  else if (p.epi == kResidual)
    ok = al16(p.y) && p.ldy % 8 == 0 && p.N % 8 == 0 && al16(p.res) && p.ldr % 8 == 0;
  p.vec = ok ? 1 : 0;
}

// Pipeline stages for a token tile of ``nt`` columns: the stage cap, bounded by 200 KB of tiles.
int stage_count(int nt) {
  const int stage_bytes = kWTileBytes + nt * kTileK * 2;
  return std::min(max_stages(), (200 * 1024) / stage_bytes);
}

// Dynamic shared memory of one launch: 1 KB alignment slack, the stages, barriers and TMEM handle (64 B), the
// epilogue exchange buffer (16 x 128 floats), the folded-norm scales (256 floats), the all-reduce's absent-rank
// flags (kMaxRanks ints) and 1 KB of slack.
size_t smem_bytes(int stages, int nt) {
  const int stage_bytes = kWTileBytes + nt * kTileK * 2;
  return 1024 + size_t(stages) * stage_bytes + 64 + 16 * kTileM * 4 + 256 * 4 + kMaxRanks * 4 + 1024;
}

struct Scratch {
  torch::Tensor ws, counters, err;
};
Scratch& scratch(torch::Device dev) {
  static std::unordered_map<int, Scratch> per_dev;
  Scratch& s = per_dev[dev.index()];
  if (!s.counters.defined()) {
    auto o = torch::TensorOptions().device(dev);
    s.counters = torch::zeros({1 << 16}, o.dtype(torch::kInt32));
    s.err = torch::zeros({1}, o.dtype(torch::kInt32));
    s.ws = torch::empty({1 << 22}, o.dtype(torch::kFloat32));
  }
  return s;
}

}  // namespace gemm

torch::Tensor gemm_error_word(torch::Device dev) { return gemm::scratch(dev).err; }

namespace gemm {
// Prefill GEMMs (set around scan-mode forwards): launches whose epilogue allows it cover every token in one launch of
// whole (weight tile, 256-token chunk) units, CTA ranges aligned to units. Decode and verify launches keep the
// token-count-independent stream-K partition that makes a row's result independent of its launch.
static bool g_prefill = false;

// The folded norm's per-token scale rsqrt(mean(x^2) + eps) of every row of X, one warp per token: lane partials over
// 16-byte pieces in index order, then a butterfly (the GEMM epilogue's own fold arithmetic).
__global__ void fold_rstd_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int K, int T, float eps,
                                 float* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (t >= T) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + size_t(t) * ldx);
  float ss = 0.f;
#pragma unroll 4
  for (int i = lane; i < K / 8; i += 32) {
    const uint4 u = xr[i];
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h2[e]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) out[t] = rsqrtf(ss / float(K) + eps);
}

// Checks the operands and launches the GEMM in chunks of at most 256 tokens; ``chunk(p, t0)`` points the chunk's
// outputs. Returns the number of CTAs launched over all chunks.
template <class F>
int launch_chunks(const torch::Tensor& x, const torch::Tensor& w, int epi, F chunk) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda(), "gemm: CUDA tensors expected");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "gemm: bf16 operands expected");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "gemm: shape mismatch");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1, "gemm: inner dimension must be contiguous");
  TORCH_CHECK((x.stride(0) * 2) % 16 == 0 && (w.stride(0) * 2) % 16 == 0, "gemm: row strides must be 16-byte multiples");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0,
              "gemm: operands must be 16-byte aligned");
  const at::cuda::CUDAGuard guard(x.device());
  const int T = x.size(0), K = x.size(1), N = w.size(0);
  if (T == 0) return 0;
  Scratch& sc = scratch(x.device());
  const int sms = num_sms();
  const int n_tiles = (N + kTileM - 1) / kTileM;
  const int kb_total = (K + kTileK - 1) / kTileK;
  const long total = long(n_tiles) * kb_total;
  const int grid = gemm_grid(total, sms);
  const CUtensorMap& wmap = weight_map(w.data_ptr(), N, K, w.stride(0));
  auto stream = at::cuda::getCurrentCUDAStream();
  TORCH_CHECK(n_tiles <= sc.counters.numel(), "gemm: too many weight tiles");
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    attr_set = true;
  }
  const bool unit_epi = epi == kPlain || epi == kResidual || epi == kSwiGLU || epi == kReLU2 || epi == kF32;
  if (g_prefill && unit_epi && long(n_tiles) * ((T + 255) / 256) >= sms) {
    // prefill: one launch of whole (tile, chunk) units
    Params p{};
    p.T = T;
    p.N = N;
    p.K = K;
    p.chunks = (T + 255) / 256;
    p.nt = p.chunks > 1 ? 256 : std::max(16, (T + 15) / 16 * 16);
    p.n_tiles = n_tiles;
    p.kb_total = kb_total;
    p.units = n_tiles * p.chunks;
    p.aligned = 1;
    p.total = long(p.units) * kb_total;
    p.epi = epi;
    p.stages = stage_count(p.nt);
    const int per = (p.units + sms - 1) / sms;
    const int ugrid = (p.units + per - 1) / per;
    p.ws = sc.ws.data_ptr<float>();  // unused: no tile is split
    p.counters = sc.counters.data_ptr<int>();
    p.err = sc.err.data_ptr<int>();
    chunk(p, 0);
    set_vector_epilogue(p);
    p.xr = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
    p.ldx = int(x.stride(0));
    TORCH_CHECK(!p.fold || K % 8 == 0, "gemm: a folded norm needs K % 8 == 0");
    torch::Tensor rstd;
    if (p.fold) {
      rstd = torch::empty({T}, x.options().dtype(torch::kFloat32));
      C10_CUDA_CHECK(launch_pdl(fold_rstd_kernel, (T + 7) / 8, 256, 0, stream.stream(), p.xr, p.ldx, K, T,
                                p.fold_eps, rstd.data_ptr<float>()));
      p.rstd = rstd.data_ptr<float>();
    }
    CUtensorMap xmap = make_map(x.data_ptr(), T, K, x.stride(0), p.nt);
    C10_CUDA_CHECK(launch_pdl(gemm_kernel, ugrid, kThreads, smem_bytes(p.stages, p.nt), stream.stream(), wmap, xmap,
                              p));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return ugrid;
  }
  int launched = 0;
  for (int t0 = 0; t0 < T; t0 += 256) {
    const int tc = std::min(256, T - t0);
    Params p{};
    p.T = tc;
    p.N = N;
    p.K = K;
    p.nt = std::max(16, (tc + 15) / 16 * 16);
    p.n_tiles = n_tiles;
    p.kb_total = kb_total;
    p.chunks = 1;
    p.units = n_tiles;
    p.total = total;
    p.epi = epi;
    p.stages = stage_count(p.nt);
    const size_t ws_need = size_t(2) * grid * p.nt * kTileM;
    if (size_t(sc.ws.numel()) < ws_need) sc.ws = torch::empty({int64_t(ws_need)}, sc.ws.options());
    p.ws = sc.ws.data_ptr<float>();
    p.counters = sc.counters.data_ptr<int>();
    p.err = sc.err.data_ptr<int>();
    chunk(p, t0);
    set_vector_epilogue(p);
    const __nv_bfloat16* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()) + size_t(t0) * x.stride(0);
    p.xr = xp;
    p.ldx = int(x.stride(0));
    TORCH_CHECK(!p.fold || K % 8 == 0, "gemm: a folded norm needs K % 8 == 0");
    CUtensorMap xmap = make_map(xp, tc, K, x.stride(0), p.nt);
    C10_CUDA_CHECK(launch_pdl(gemm_kernel, grid, kThreads, smem_bytes(p.stages, p.nt), stream.stream(), wmap, xmap, p));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    launched += grid;
  }
  return launched;
}
}  // namespace gemm

// Scan-mode (prefill) forwards switch their GEMMs to whole-unit launches and back.
void gemm_prefill_mode(bool on) { gemm::g_prefill = on; }

// Launch one GEMM over all T tokens (chunks of 256 tokens per launch).
// ``fold_eps`` >= 0 folds an RMSNorm into the GEMM (X raw, norm weight pre-multiplied into W's columns).
void gemm_launch(const torch::Tensor& x, const torch::Tensor& w, int epi, torch::Tensor y, torch::Tensor yf,
                 const torch::Tensor& res, torch::Tensor amax_val, torch::Tensor amax_idx, double fold_eps) {
  using namespace gemm;
  TORCH_CHECK(epi != kAllReduce, "gemm: the all-reduce epilogue has its own entry point");
  const int n_tiles = (w.size(0) + kTileM - 1) / kTileM;
  auto has = [](const torch::Tensor& t) { return t.defined() && t.numel() > 0; };
  launch_chunks(x, w, epi, [&](Params& p, int t0) {
    p.fold = fold_eps >= 0.0;
    p.fold_eps = float(fold_eps);
    if (has(y)) {
      p.y = reinterpret_cast<__nv_bfloat16*>(y.data_ptr()) + size_t(t0) * y.stride(0);
      p.ldy = y.stride(0);
    }
    if (has(yf)) {
      p.yf = yf.data_ptr<float>() + size_t(t0) * yf.stride(0);
      p.ldy = yf.stride(0);
    }
    if (has(res)) {
      p.res = reinterpret_cast<const __nv_bfloat16*>(res.data_ptr()) + size_t(t0) * res.stride(0);
      p.ldr = res.stride(0);
    }
    if (has(amax_val)) {
      // per-tile partials for this chunk live at column offset t0 of a [n_tiles, T_total] layout: use a chunk view
      p.amax_val = amax_val.data_ptr<float>() + size_t(t0) * n_tiles;
      p.amax_idx = amax_idx.data_ptr<int>() + size_t(t0) * n_tiles;
    }
  });
}

// One plain GEMM with per-CTA globaltimer stamps: returns [CTAs][8] (slots documented at E4_STAMP). Tuning only.
torch::Tensor gemm_traced(const torch::Tensor& x, const torch::Tensor& w, int64_t epi) {
  using namespace gemm;
  auto y = torch::empty({x.size(0), w.size(0)}, x.options());
  auto yf = torch::empty({x.size(0), w.size(0)}, x.options().dtype(torch::kFloat32));
  const int grid = gemm_grid(long((w.size(0) + kTileM - 1) / kTileM) * ((x.size(1) + kTileK - 1) / kTileK), num_sms());
  auto tr = torch::zeros({grid, 8}, x.options().dtype(torch::kInt64));
  launch_chunks(x, w, int(epi), [&](Params& p, int) {
    p.y = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
    p.yf = yf.data_ptr<float>();
    p.ldy = int(w.size(0));
    p.res = reinterpret_cast<const __nv_bfloat16*>(y.data_ptr());
    p.ldr = int(w.size(0));
    p.trace = reinterpret_cast<unsigned long long*>(tr.data_ptr<int64_t>());
  });
  return tr;
}

// Tensor-parallel row-parallel GEMM fused with its all-reduce and the residual add:
// y = residual + sum over ranks of X_r . W_r^T, bit-identical on every rank. ``part`` / ``gath`` / ``flags``: int64
// device addresses of every rank's peer areas (this rank's own at ``rank``); ``ctrl``: this rank's call and
// finished-CTA counters (two words). ``two_shot_rows``: launches of more tokens than this use the two-shot form.
// Returns the number of CTAs launched.
int64_t gemm_allreduce(const torch::Tensor& x, const torch::Tensor& w, const torch::Tensor& residual, torch::Tensor y,
                       const std::vector<int64_t>& part, const std::vector<int64_t>& gath,
                       const std::vector<int64_t>& flags, int64_t ctrl, int64_t ldp, int64_t rank,
                       int64_t two_shot_rows) {
  using namespace gemm;
  const int world = int(part.size());
  TORCH_CHECK(world >= 1 && world <= kMaxRanks && int(gath.size()) == world && int(flags.size()) == world,
              "gemm_allreduce: 1..8 ranks");
  const int N = w.size(0);
  TORCH_CHECK(N % 8 == 0 && N <= ldp && (N + kTileM - 1) / kTileM <= kTpTiles, "gemm_allreduce: N too large");
  TORCH_CHECK(ldp % 8 == 0, "gemm_allreduce: peer row stride must be a multiple of 8");
  TORCH_CHECK(residual.size(0) == x.size(0) && residual.size(1) == N && y.size(0) == x.size(0) && y.size(1) == N,
              "gemm_allreduce: residual / output shape");
  TORCH_CHECK(residual.stride(1) == 1 && y.stride(1) == 1 && residual.stride(0) % 8 == 0 && y.stride(0) % 8 == 0 &&
              reinterpret_cast<uintptr_t>(residual.data_ptr()) % 16 == 0 &&
              reinterpret_cast<uintptr_t>(y.data_ptr()) % 16 == 0, "gemm_allreduce: 16-byte aligned rows expected");
  return launch_chunks(x, w, kAllReduce, [&](Params& p, int t0) {
    for (int r = 0; r < world; ++r) {
      p.tp_part[r] = reinterpret_cast<__nv_bfloat16*>(part[r]);
      p.tp_gath[r] = reinterpret_cast<__nv_bfloat16*>(gath[r]);
      p.tp_flag[r] = reinterpret_cast<unsigned*>(flags[r]);
    }
    p.tp_calls = reinterpret_cast<unsigned*>(ctrl);
    p.tp_done = reinterpret_cast<unsigned*>(ctrl) + 1;
    p.ldp = int(ldp);
    p.world = world;
    p.rank = int(rank);
    p.two_shot = (world > 1 && p.T > two_shot_rows) ? 1 : 0;
    p.y = reinterpret_cast<__nv_bfloat16*>(y.data_ptr()) + size_t(t0) * y.stride(0);
    p.ldy = int(y.stride(0));
    p.res = reinterpret_cast<const __nv_bfloat16*>(residual.data_ptr()) + size_t(t0) * residual.stride(0);
    p.ldr = int(residual.stride(0));
  });
}

}  // namespace e4

// =====================================================================================================================
// Allocation-free GEMM entry point (declared in e4_noalloc.h, which states its callers, limits and sharing rules).
// This has no counterpart in the reference.
//
// The stream-K workspace of the regular entry point (partial tiles, per-tile arrival counters, error word) lives here
// in one file-scope device array. Host code only ever sees the array's host-side stand-in symbol; the kernel gets the
// device address that cudaGetSymbolAddress returns for the current device at the first call on that device.
// =====================================================================================================================
#include "e4_noalloc.h"

namespace e4 {
namespace noalloc {

constexpr int kMaxTokens = E4_NOALLOC_MAX_TOKENS;
constexpr int kMaxGrid = 160;   // CTAs (one per SM, B200 has 148)
constexpr int kMaxTiles = E4_NOALLOC_MAX_TILES;
constexpr size_t kWsFloats = size_t(2) * kMaxGrid * kMaxTokens * gemm::kTileM;
constexpr size_t kCountersOffset = kWsFloats * sizeof(float);
constexpr size_t kErrOffset = kCountersOffset + size_t(kMaxTiles) * sizeof(int);
constexpr size_t kBytes = kErrOffset + 256;
static_assert(kBytes == E4_NOALLOC_SCRATCH_BYTES, "e4_noalloc.h states the array's size");

static __device__ __align__(256) unsigned char scratch[kBytes];

constexpr int kMaxDevices = 64;
std::mutex setup_mu;
void* scratch_addr[kMaxDevices] = {};

// Device address of the array on ``dev`` (the current device), looked up once per device.
int setup(int dev, void** out) {
  std::lock_guard<std::mutex> g(setup_mu);
  if (!scratch_addr[dev]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, scratch) != cudaSuccess || !ptr) return E4_NOALLOC_CUDA_ERROR;
    if (cudaFuncSetAttribute(gemm::gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess)
      return E4_NOALLOC_CUDA_ERROR;
    scratch_addr[dev] = ptr;
  }
  *out = scratch_addr[dev];
  return E4_NOALLOC_OK;
}

int current(void** base) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return E4_NOALLOC_CUDA_ERROR;
  return setup(dev, base);
}

}  // namespace noalloc
}  // namespace e4

extern "C" int e4_gemm_bf16_noalloc(const void* x, int ldx, const void* w, int ldw, void* y, int ldy, int T, int N,
                                    int K, void* stream) {
  using namespace e4;
  using namespace e4::gemm;
  if (!x || !w || !y || T <= 0 || T > noalloc::kMaxTokens || N <= 0 || K <= 0) return E4_NOALLOC_BAD_ARGS;
  if (ldx < K || ldw < K || ldy < N || (ldx * 2) % 16 || (ldw * 2) % 16) return E4_NOALLOC_BAD_ARGS;
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(w) % 16) return E4_NOALLOC_BAD_ARGS;
  const int n_tiles = (N + kTileM - 1) / kTileM;
  if (n_tiles > noalloc::kMaxTiles) return E4_NOALLOC_BAD_ARGS;
  void* base = nullptr;
  if (const int rc = noalloc::current(&base)) return rc;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return E4_NOALLOC_CUDA_ERROR;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return E4_NOALLOC_CUDA_ERROR;
  const int kb_total = (K + kTileK - 1) / kTileK;
  const long total = long(n_tiles) * kb_total;
  // the regular entry point's grid and pipeline (same stream-K cut points, so the same reduction order)
  const int grid = gemm::gemm_grid(total, std::min(sms, noalloc::kMaxGrid));
  Params p{};
  p.T = T;
  p.N = N;
  p.K = K;
  p.nt = std::max(16, (T + 15) / 16 * 16);
  p.n_tiles = n_tiles;
  p.kb_total = kb_total;
  p.chunks = 1;
  p.units = n_tiles;
  p.total = total;
  p.epi = kPlain;
  p.stages = stage_count(p.nt);
  unsigned char* b = reinterpret_cast<unsigned char*>(base);
  p.ws = reinterpret_cast<float*>(b);
  p.counters = reinterpret_cast<int*>(b + noalloc::kCountersOffset);
  p.err = reinterpret_cast<int*>(b + noalloc::kErrOffset);
  p.y = reinterpret_cast<__nv_bfloat16*>(y);
  p.ldy = ldy;
  set_vector_epilogue(p);
  CUtensorMap wmap, xmap;
  try {
    wmap = make_map(w, N, K, ldw, kTileM);
    xmap = make_map(x, T, K, ldx, p.nt);
  } catch (...) {
    return E4_NOALLOC_CUDA_ERROR;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // the counters this call's tiles use, and the error word (the last call's contents are still in the array)
  if (cudaMemsetAsync(p.counters, 0, sizeof(int) * n_tiles, st) != cudaSuccess) return E4_NOALLOC_CUDA_ERROR;
  if (cudaMemsetAsync(p.err, 0, sizeof(int), st) != cudaSuccess) return E4_NOALLOC_CUDA_ERROR;
  if (launch_pdl(gemm_kernel, grid, kThreads, smem_bytes(p.stages, p.nt), st, wmap, xmap, p) != cudaSuccess)
    return E4_NOALLOC_CUDA_ERROR;
  return E4_NOALLOC_OK;
}

extern "C" int e4_gemm_noalloc_status(int* kernel_error, void* stream) {
  using namespace e4;
  if (!kernel_error) return E4_NOALLOC_BAD_ARGS;
  void* base = nullptr;
  if (const int rc = noalloc::current(&base)) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const void* err = reinterpret_cast<unsigned char*>(base) + noalloc::kErrOffset;
  if (cudaMemcpyAsync(kernel_error, err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return E4_NOALLOC_CUDA_ERROR;
  if (cudaStreamSynchronize(st) != cudaSuccess) return E4_NOALLOC_CUDA_ERROR;
  return E4_NOALLOC_OK;
}
