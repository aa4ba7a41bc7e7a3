// The plan of a small call formed by one block in shared memory, shared by
// the small-call route/plan/quantise kernel (wm_bs_sm100.cu).  The plan is the
// one the plan kernels of wm_plan.cu write (stable (token, k) order within an
// expert, the shared expert last).
#pragma once

#include "wm_kernels.h"

namespace wm {
namespace {

constexpr int kMaxSmallPairs = 128;  // T * K of the calls small_plan_block takes
constexpr int kMaxSmallTokens = 8;   // T of those calls (one bit per token)
constexpr int kMaxSmallExperts = 512;

// Shared-memory state of small_plan_block.  ids (the pairs' expert ids, in
// (token, k) order) is the input; pos (each pair's sorted row, -1 for an id
// outside [0, E)), shared_row0 and total are the results every block needs.
struct SmallPlan {
  int ids[kMaxSmallPairs];
  int pos[kMaxSmallPairs];
  uint32_t used[kMaxSmallExperts / 32];   // bit e: some pair names expert e
  int wpre[kMaxSmallExperts / 32];        // set bits in the words before
  uint32_t tmask[kMaxSmallExperts / 4];   // byte e: the tokens that name expert e
  int ucnt[kMaxSmallPairs + 1];           // per distinct expert, ascending (the shared expert last)
  int uexp[kMaxSmallPairs + 1];
  int uoff[kMaxSmallPairs + 2];           // first sorted row; uoff[n_u + 1] = rows used
  int utile[kMaxSmallPairs + 2];          // first tile
  int n_u;                                // distinct routed experts
  int repeated;                           // a token names an expert twice
  int shared_row0;                        // first row of the shared expert (-1 without it)
  int total;                              // rows used
};

// The plan of a call of T <= kMaxSmallTokens tokens, P = T * K <=
// kMaxSmallPairs pairs (P <= blockDim.x) and E <= kMaxSmallExperts experts:
// the same plan as the single-block plan kernel (rows of an expert in
// (token, k) order, groups padded to `align` rows, tiles of `align` rows when
// align > 1, else p.tile_rows or 16) with no scan over the E + 1 experts.  A
// bitmap of the experts named gives each expert its place among the distinct
// ones (the set bits below it), a byte per expert of the tokens naming it
// gives each pair its row within the expert (the tokens below it), and one
// warp scans the distinct experts' padded counts.  A token that names an
// expert twice (never from the router) takes a pair-by-pair count instead.
// With write = false only the shared-memory results are formed (a block that
// needs the rows but leaves the plan arrays to another block).  Every thread
// of the block calls it.
__device__ void small_plan_block(SmallPlan& sp, int T, int K, int E, int has_shared, int align, Plan p,
                                 int max_rows, int max_mtiles, uint32_t* status, bool write) {
  const int P = T * K;
  const int tile = align > 1 ? align : (p.tile_rows > 0 ? p.tile_rows : 16);
  const int words = (E + 31) / 32;
  for (int w = threadIdx.x; w < kMaxSmallExperts / 4; w += blockDim.x) {
    sp.tmask[w] = 0u;
    if (w < kMaxSmallExperts / 32) sp.used[w] = 0u;
  }
  if (threadIdx.x == 0) sp.repeated = 0;
  __syncthreads();
  const int i = threadIdx.x;  // one pair per thread
  int e = -1, t = 0;
  if (i < P) {
    e = sp.ids[i];
    t = i / K;
    if (e >= 0 && e < E) {
      atomicOr(&sp.used[e >> 5], 1u << (e & 31));
      atomicOr(&sp.tmask[e >> 2], 1u << ((e & 3) * 8 + t));
      for (int j = t * K; j < i; ++j)
        if (sp.ids[j] == e) sp.repeated = 1;
    } else {
      if (write && (e >= 0 || !p.skip_negative)) report_status(status, kStatusBadExpert, (uint32_t)i);
      e = -1;
    }
  }
  __syncthreads();
  if (threadIdx.x < 32) {  // set bits before each bitmap word
    const int lane = threadIdx.x;
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
  int slot = -1, rank = 0;
  if (e >= 0) {
    slot = sp.wpre[e >> 5] + __popc(sp.used[e >> 5] & ((1u << (e & 31)) - 1u));
    if (!rep) {
      const uint32_t tm = (sp.tmask[e >> 2] >> ((e & 3) * 8)) & 0xFFu;
      rank = __popc(tm & ((1u << t) - 1u));
      if (rank == 0) {
        sp.uexp[slot] = e;
        sp.ucnt[slot] = __popc(tm);
      }
    } else {  // pair by pair
      int cnt = 0;
      bool first = true;
      for (int j = 0; j < P; ++j) {
        if (sp.ids[j] != e) continue;
        ++cnt;
        if (j < i) {
          ++rank;
          first = false;
        }
      }
      if (first) {
        sp.uexp[slot] = e;
        sp.ucnt[slot] = cnt;
      }
    }
  }
  __syncthreads();
  const int U = sp.n_u;
  if (threadIdx.x < 32) {  // offsets and first tiles: a scan over the distinct experts (+ the shared one)
    const int lane = threadIdx.x;
    const int n = U + 1;
    int row_carry = 0, tile_carry = 0;
    for (int b = 0; b < n; b += 32) {
      const int u = b + lane;
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
      if (u < n) {
        sp.uoff[u] = row_carry + rs - rows;
        sp.utile[u] = tile_carry + ts - tiles;
        if (u == U) sp.ucnt[U] = c;
      }
      row_carry += __shfl_sync(0xffffffffu, rs, 31);
      tile_carry += __shfl_sync(0xffffffffu, ts, 31);
    }
    if (lane == 0) {
      sp.uoff[n] = row_carry;
      sp.utile[n] = tile_carry;
      sp.total = row_carry;
      sp.shared_row0 = has_shared ? sp.uoff[U] : -1;
      if (write && row_carry > max_rows) report_status(status, kStatusOverflow, (uint32_t)row_carry);
      if (write && tile_carry > max_mtiles) report_status(status, kStatusOverflow, (uint32_t)tile_carry);
    }
  }
  __syncthreads();
  if (i < P) sp.pos[i] = e < 0 ? -1 : sp.uoff[slot] + rank;
  if (!write) return;
  const int total = sp.total, n_tiles = sp.utile[U + 1];
  // per-expert arrays: an expert's place among the distinct ones from the bitmap
  for (int x = threadIdx.x; x <= E + 1; x += blockDim.x) {
    if (x < E) {
      const uint32_t wv = sp.used[x >> 5], bit = 1u << (x & 31);
      const int s = sp.wpre[x >> 5] + __popc(wv & (bit - 1u));
      p.counts[x] = (wv & bit) ? sp.ucnt[s] : 0;
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
  if (i < P) {
    p.pair_pos[i] = sp.pos[i];
    if (sp.pos[i] >= 0) p.row_token[sp.pos[i]] = t;
  }
  if (has_shared)
    for (int tt = threadIdx.x; tt < T; tt += blockDim.x) p.row_token[sp.shared_row0 + tt] = tt;
}

}  // namespace
}  // namespace wm
