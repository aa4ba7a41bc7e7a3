// The plan of a small call formed by one block in shared memory, shared by
// the small-call route/plan/quantise kernel (wm_bs_sm100.cu).  The plan is the
// one the plan kernels of wm_plan.cu write (stable (token, k) order within an
// expert, the shared expert last).
#pragma once

#include <type_traits>

#include "wm_kernels.h"

namespace wm {
namespace {

constexpr int kMaxSmallPairs = 1024;   // T * K of the calls small_plan_block takes
constexpr int kMaxSmallTokens = 64;    // T of those calls (one bit per token)
constexpr int kMaxSmallExperts = 512;

// Shared-memory state of small_plan_block for calls of up to MAXT tokens and
// MAXP pairs (the few-token form keeps a byte of token bits per expert and is
// 6x smaller, which its one-block-per-token launch measured faster).  ids
// (the pairs' expert ids, in (token, k) order) is the input; pos (each pair's
// sorted row, -1 for an id outside [0, E)), shared_row0 and total are the
// results every block needs.
template <int MAXT, int MAXP>
struct SmallPlan {
  static_assert(MAXT <= kMaxSmallTokens && MAXP <= kMaxSmallPairs, "small plan limits");
  static constexpr int kMaxT = MAXT, kMaxP = MAXP;
  static constexpr int kMaxU = MAXP < kMaxSmallExperts ? MAXP : kMaxSmallExperts;  // distinct experts
  using Mask = typename std::conditional<(MAXT <= 8), uint32_t, unsigned long long>::type;
  static constexpr int kMaskWords = MAXT <= 8 ? kMaxSmallExperts / 4 : kMaxSmallExperts;
  int ids[MAXP];
  int pos[MAXP];
  uint32_t used[kMaxSmallExperts / 32];  // bit e: some pair names expert e
  int wpre[kMaxSmallExperts / 32];       // set bits in the words before
  Mask tmask[kMaskWords];                // the tokens that name expert e (a byte or a word per expert)
  int ucnt[kMaxU + 1];                   // per distinct expert, ascending (the shared expert last)
  int uexp[kMaxU + 1];
  int uoff[kMaxU + 2];                   // first sorted row; uoff[n_u + 1] = rows used
  int utile[kMaxU + 2];                  // first tile
  int wsum[2][32];                       // per-warp sums of the scan
  int n_u;                               // distinct routed experts
  int repeated;                          // a token names an expert twice
  int shared_row0;                       // first row of the shared expert (-1 without it)
  int total;                             // rows used

  __device__ __forceinline__ void mark(int e, int t) {
    if constexpr (MAXT <= 8)
      atomicOr(&tmask[e >> 2], 1u << ((e & 3) * 8 + t));
    else
      atomicOr(&tmask[e], 1ull << t);
  }
  __device__ __forceinline__ unsigned long long tokens(int e) const {
    if constexpr (MAXT <= 8)
      return (tmask[e >> 2] >> ((e & 3) * 8)) & 0xFFu;
    else
      return tmask[e];
  }
  // Place of expert e among the distinct experts named (set bits below it).
  __device__ __forceinline__ int slot(int e) const {
    return wpre[e >> 5] + __popc(used[e >> 5] & ((1u << (e & 31)) - 1u));
  }
};

// The plan of a call of T <= kMaxSmallTokens tokens, P = T * K <=
// kMaxSmallPairs pairs and E <= kMaxSmallExperts experts: the same plan as
// the plan kernels (rows of an expert in (token, k) order, groups padded to
// `align` rows, tiles of `align` rows when align > 1, else p.tile_rows or 16)
// with no sort.  A bitmap of the experts named gives each expert its place
// among the distinct ones (the set bits below it), a 64-bit mask per expert of
// the tokens naming it gives each pair its row within the expert (the tokens
// below it), and a block scan orders the distinct experts' padded counts.  A
// token that names an expert twice (never from the router) takes a
// pair-by-pair count instead.  With write = false only the shared-memory
// results are formed (a block that needs the rows but leaves the plan arrays
// to another block).  Every thread of the block calls it; blockDim.x is a
// multiple of 32 and at least 64.
template <class SP>
__device__ void small_plan_block(SP& sp, int T, int K, int E, int has_shared, int align, Plan p,
                                 int max_rows, int max_mtiles, uint32_t* status, bool write) {
  const int P = T * K;
  const int tile = align > 1 ? align : (p.tile_rows > 0 ? p.tile_rows : 16);
  const int words = (E + 31) / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (int w = threadIdx.x; w < SP::kMaskWords; w += blockDim.x) {
    sp.tmask[w] = 0;
    if (w < kMaxSmallExperts / 32) sp.used[w] = 0u;
  }
  if (threadIdx.x == 0) sp.repeated = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    const int e = sp.ids[i], t = i / K;
    if (e >= 0 && e < E) {
      atomicOr(&sp.used[e >> 5], 1u << (e & 31));
      sp.mark(e, t);
      for (int j = t * K; j < i; ++j)
        if (sp.ids[j] == e) sp.repeated = 1;
    } else if (write && (e >= 0 || !p.skip_negative)) {
      report_status(status, kStatusBadExpert, (uint32_t)i);
    }
  }
  __syncthreads();
  if (warp == 0) {  // set bits before each bitmap word
    const int c = lane < words ? __popc(sp.used[lane]) : 0;
    int x = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane < words) sp.wpre[lane] = x - c;
    if (lane == 31) sp.n_u = x;
  }
  __syncthreads();
  const bool rep = sp.repeated != 0;
  // each pair's row within its expert (in pos for now); the first pair of an
  // expert records the expert and its count at the expert's place
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    const int e = sp.ids[i], t = i / K;
    if (e < 0 || e >= E) {
      sp.pos[i] = -1;
      continue;
    }
    int rank = 0, cnt = 0;
    if (!rep) {
      const unsigned long long tm = sp.tokens(e);
      rank = __popcll(tm & ((1ull << t) - 1ull));
      cnt = __popcll(tm);
    } else {
      for (int j = 0; j < P; ++j) {
        if (sp.ids[j] != e) continue;
        ++cnt;
        if (j < i) ++rank;
      }
    }
    sp.pos[i] = rank;
    if (rank == 0) {
      const int slot = sp.slot(e);
      sp.uexp[slot] = e;
      sp.ucnt[slot] = cnt;
    }
  }
  __syncthreads();
  const int U = sp.n_u;
  const int n = U + 1;  // the distinct routed experts, then the shared expert
  // padded rows and tiles of each distinct expert -> offsets and first tiles:
  // one warp's scan when they fit it (no block barrier), else a block scan
  int carry_r = 0, carry_t = 0;
  if (n <= 32) {
    if (warp == 0) {
      const int c = lane < U ? sp.ucnt[lane] : (lane == U && has_shared ? T : 0);
      const int rows = lane < n ? (c + align - 1) / align * align : 0;
      const int tiles = lane < n ? (c + tile - 1) / tile : 0;
      int rs = rows, ts = tiles;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int r2 = __shfl_up_sync(0xffffffffu, rs, o), t2 = __shfl_up_sync(0xffffffffu, ts, o);
        if (lane >= o) {
          rs += r2;
          ts += t2;
        }
      }
      if (lane < n) {
        sp.uoff[lane] = rs - rows;
        sp.utile[lane] = ts - tiles;
        if (lane == U) sp.ucnt[U] = c;
      }
      carry_r = __shfl_sync(0xffffffffu, rs, 31);
      carry_t = __shfl_sync(0xffffffffu, ts, 31);
    }
  }
  for (int b = 0; n > 32 && b < n; b += blockDim.x) {
    const int u = b + threadIdx.x;
    const int c = u < U ? sp.ucnt[u] : (u == U && has_shared ? T : 0);
    const int rows = u < n ? (c + align - 1) / align * align : 0;
    const int tiles = u < n ? (c + tile - 1) / tile : 0;
    int rs = rows, ts = tiles;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int r2 = __shfl_up_sync(0xffffffffu, rs, o), t2 = __shfl_up_sync(0xffffffffu, ts, o);
      if (lane >= o) {
        rs += r2;
        ts += t2;
      }
    }
    if (lane == 31) {
      sp.wsum[0][warp] = rs;
      sp.wsum[1][warp] = ts;
    }
    __syncthreads();
    if (warp == 0) {
      int a0 = lane < nwarps ? sp.wsum[0][lane] : 0, a1 = lane < nwarps ? sp.wsum[1][lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y0 = __shfl_up_sync(0xffffffffu, a0, o), y1 = __shfl_up_sync(0xffffffffu, a1, o);
        if (lane >= o) {
          a0 += y0;
          a1 += y1;
        }
      }
      if (lane < nwarps) {
        sp.wsum[0][lane] = a0;
        sp.wsum[1][lane] = a1;
      }
    }
    __syncthreads();
    const int pre_r = carry_r + (warp > 0 ? sp.wsum[0][warp - 1] : 0) + rs - rows;
    const int pre_t = carry_t + (warp > 0 ? sp.wsum[1][warp - 1] : 0) + ts - tiles;
    if (u < n) {
      sp.uoff[u] = pre_r;
      sp.utile[u] = pre_t;
      if (u == U) sp.ucnt[U] = c;
    }
    carry_r += sp.wsum[0][nwarps - 1];
    carry_t += sp.wsum[1][nwarps - 1];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    sp.uoff[n] = carry_r;
    sp.utile[n] = carry_t;
    sp.total = carry_r;
    sp.shared_row0 = has_shared ? sp.uoff[U] : -1;
    if (write && carry_r > max_rows) report_status(status, kStatusOverflow, (uint32_t)carry_r);
    if (write && carry_t > max_mtiles) report_status(status, kStatusOverflow, (uint32_t)carry_t);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < P; i += blockDim.x)
    if (sp.pos[i] >= 0) sp.pos[i] += sp.uoff[sp.slot(sp.ids[i])];
  if (!write) return;
  const int total = sp.total, n_tiles = sp.utile[U + 1];
  // per-expert arrays: an expert's place among the distinct ones from the bitmap
  for (int x = threadIdx.x; x <= E + 1; x += blockDim.x) {
    if (x < E) {
      const int s = sp.slot(x);
      p.counts[x] = (sp.used[x >> 5] >> (x & 31)) & 1u ? sp.ucnt[s] : 0;
      p.offsets[x] = sp.uoff[s];
    } else if (x == E) {
      p.counts[E] = sp.ucnt[U];
      p.offsets[E] = sp.uoff[U];
    } else {
      p.offsets[E + 1] = total;
    }
  }
  const int n_unique = U + (sp.ucnt[U] > 0 ? 1 : 0);
  for (int u = threadIdx.x; u < n_unique; u += blockDim.x) p.unique[u] = u < U ? sp.uexp[u] : E;
  if (threadIdx.x == 0) {
    *p.n_unique = n_unique;
    *p.n_mtiles = min(n_tiles, max_mtiles);
  }
  for (int u = threadIdx.x; u <= U; u += blockDim.x) {
    const int ue = u < U ? sp.uexp[u] : E;
    const int c = sp.ucnt[u];
    const int m_tiles = (c + tile - 1) / tile;
    for (int m = 0; m < m_tiles && sp.utile[u] + m < max_mtiles; ++m) {
      p.mtiles[2 * (sp.utile[u] + m)] = ue;
      p.mtiles[2 * (sp.utile[u] + m) + 1] = sp.uoff[u] + tile * m;
    }
  }
  if (total > max_rows) return;
  for (int u = threadIdx.x; u <= U; u += blockDim.x)
    for (int r = sp.uoff[u] + sp.ucnt[u]; r < sp.uoff[u + 1]; ++r) p.row_token[r] = -1;
  if (p.rowmax != nullptr)
    for (int r = threadIdx.x; r < total; r += blockDim.x) p.rowmax[r] = 0u;
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    p.pair_pos[i] = sp.pos[i];
    if (sp.pos[i] >= 0) p.row_token[sp.pos[i]] = i / K;
  }
  if (has_shared)
    for (int t = threadIdx.x; t < T; t += blockDim.x) p.row_token[sp.shared_row0 + t] = t;
}

}  // namespace
}  // namespace wm
