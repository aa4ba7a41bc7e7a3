// Token sort / permute / unpermute on the device.
//
// The reference groups the flattened (token, k) pairs by expert with a stable
// sort (np.argsort(kind="stable"), qwen_expert_waves.py:39-51;
// std::stable_sort, Native/QwenNative/engine.mm:2105-2127) and gathers the rows
// of each group (gather_rows16, QwenNative/kernels.metal:691-700).  Here the
// same stable grouping is a counting sort: per-expert counts, an exclusive
// scan into row offsets, then a scatter that walks the tokens in order, so a
// group's rows stay in ascending (token, k) order.  The shared expert is
// expert index E with one row per token.  Nothing here synchronises with the
// host: routes never leave the GPU (the reference waits for them on the CPU,
// qwen4_exp.py:899-902).
#include "wm_kernels.h"

namespace wm {

namespace {

__device__ __forceinline__ int round_up(int v, int a) { return (v + a - 1) / a * a; }

// Exclusive scan over n values given by value(i); store(i, prefix) for each.
// Returns the total.  Every thread of the block must call it.
template <typename F, typename G>
__device__ int block_exclusive_scan(int n, F value, G store) {
  __shared__ int warp_sums[32];
  __shared__ int carry;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = (blockDim.x + 31) >> 5;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < n; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const int v = i < n ? value(i) : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int s = lane < nwarps ? warp_sums[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      warp_sums[lane] = s;
    }
    __syncthreads();
    const int prefix = carry + (warp > 0 ? warp_sums[warp - 1] : 0) + x - v;
    if (i < n) store(i, prefix);
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = prefix + v;
    __syncthreads();
  }
  return carry;
}

// From per-expert counts in shared memory: offsets, unique list, row-tile
// list and padding rows.  `cnt` holds E + 1 counts (index E = shared expert).
// Tiles are `align` rows (the GEMM's 128-row tiles) when the groups are
// padded, else p.tile_rows rows (the decode kernels' token chunks; 16 when 0).
__device__ void finish_plan(const int* cnt, int* off, int E, int align, Plan p, int max_rows, int max_mtiles,
                            uint32_t* status) {
  const int total = block_exclusive_scan(
      E + 1, [&](int i) { return round_up(cnt[i], align); }, [&](int i, int v) { off[i] = v; });
  if (threadIdx.x == 0) {
    off[E + 1] = total;
    if (total > max_rows) report_status(status, kStatusOverflow, (uint32_t)total);
  }
  __syncthreads();
  for (int i = threadIdx.x; i <= E; i += blockDim.x) {
    p.counts[i] = cnt[i];
    p.offsets[i] = off[i];
  }
  if (threadIdx.x == 0) p.offsets[E + 1] = total;
  const int nu = block_exclusive_scan(
      E + 1, [&](int i) { return cnt[i] > 0 ? 1 : 0; },
      [&](int i, int v) {
        if (cnt[i] > 0) p.unique[v] = i;
      });
  const int tile = align > 1 ? align : (p.tile_rows > 0 ? p.tile_rows : 16);
  const int nm = block_exclusive_scan(
      E + 1, [&](int i) { return (cnt[i] + tile - 1) / tile; },
      [&](int i, int v) {
        const int m_tiles = (cnt[i] + tile - 1) / tile;
        for (int m = 0; m < m_tiles && v + m < max_mtiles; ++m) {
          p.mtiles[2 * (v + m)] = i;
          p.mtiles[2 * (v + m) + 1] = off[i] + tile * m;
        }
      });
  if (threadIdx.x == 0) {
    *p.n_unique = nu;
    *p.n_mtiles = min(nm, max_mtiles);
    if (nm > max_mtiles) report_status(status, kStatusOverflow, (uint32_t)nm);
  }
  if (total > max_rows) return;
  for (int e = threadIdx.x; e <= E; e += blockDim.x)
    for (int r = off[e] + cnt[e]; r < off[e + 1]; ++r) p.row_token[r] = -1;
  if (p.rowmax != nullptr)
    for (int r = threadIdx.x; r < total; r += blockDim.x) p.rowmax[r] = 0u;
}

// Warp 0 assigns sorted rows to the pairs of tokens [t_begin, t_end), in
// (token, k) order.  run[e] holds the next free row of expert e.  Repeated
// experts within a token keep k order (ranked with __match_any_sync).
__device__ void scatter_pairs(const int32_t* idx, int t_begin, int t_end, int K, int E, int* run, Plan p,
                              uint32_t* status) {
  // Pairs in flat (t, k) order, 32 per step: a pair's slot is its expert's
  // running count plus the number of earlier lanes naming the same expert,
  // so the order within an expert stays the flat pair order.
  const int lane = threadIdx.x & 31;
  const unsigned lt_mask = (1u << lane) - 1u;
  const int i_end = t_end * K;
  for (int i0 = t_begin * K; i0 < i_end; i0 += 32) {
    const int i = i0 + lane;
    int e = -1;
    if (i < i_end) {
      e = idx[i];
      if (e < 0 || e >= E) {
        if (e >= 0 || !p.skip_negative) report_status(status, kStatusBadExpert, (uint32_t)i);
        p.pair_pos[i] = -1;
        e = -1;
      }
    }
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(same & lt_mask);
    const int base = e >= 0 ? run[e] : 0;
    if (e >= 0) {
      const int pos = base + rank;
      p.pair_pos[i] = pos;
      p.row_token[pos] = i / K;
    }
    __syncwarp();
    if (e >= 0 && rank == 0) run[e] = base + __popc(same);
    __syncwarp();
  }
}

}  // namespace

// Single-block plan for small calls (decode).  1024 threads.
__global__ void __launch_bounds__(1024) plan_small_kernel(const int32_t* __restrict__ idx, int T, int K, int E,
                                                          int has_shared, int align, Plan p, int max_rows,
                                                          int max_mtiles, uint32_t* status) {
  extern __shared__ int sm[];
  int* cnt = sm;            // E + 1
  int* off = cnt + E + 1;   // E + 2
  int* run = off + E + 2;   // E + 1
  for (int i = threadIdx.x; i <= E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < T * K; i += blockDim.x) {
    const int e = idx[i];
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) cnt[E] = has_shared ? T : 0;
  __syncthreads();
  finish_plan(cnt, off, E, align, p, max_rows, max_mtiles, status);
  __syncthreads();
  if (off[E + 1] > max_rows) return;
  for (int i = threadIdx.x; i <= E; i += blockDim.x) run[i] = off[i];
  if (has_shared)
    for (int t = threadIdx.x; t < T; t += blockDim.x) p.row_token[off[E] + t] = t;
  if (T <= 64) {
    // Every pair at once: a pair's rank within its expert is the number of
    // earlier tokens that chose the expert (a 64-bit token mask per expert),
    // valid when no token names an expert twice.
    unsigned long long* mask =
        reinterpret_cast<unsigned long long*>((reinterpret_cast<uintptr_t>(run + E + 2) + 7) & ~uintptr_t(7));
    __shared__ int repeated;
    if (threadIdx.x == 0) repeated = 0;
    for (int i = threadIdx.x; i <= E; i += blockDim.x) mask[i] = 0ull;
    __syncthreads();
    for (int i = threadIdx.x; i < T * K; i += blockDim.x) {
      const int e = idx[i], t = i / K;
      if (e < 0 || e >= E) continue;
      atomicOr(&mask[e], 1ull << t);
      for (int j = t * K; j < i; ++j)
        if (idx[j] == e) repeated = 1;
    }
    __syncthreads();
    if (!repeated) {
      for (int i = threadIdx.x; i < T * K; i += blockDim.x) {
        const int e = idx[i], t = i / K;
        if (e < 0 || e >= E) {
          if (e >= 0 || !p.skip_negative) report_status(status, kStatusBadExpert, (uint32_t)i);
          p.pair_pos[i] = -1;
          continue;
        }
        const int pos = off[e] + __popcll(mask[e] & ((1ull << t) - 1ull));
        p.pair_pos[i] = pos;
        p.row_token[pos] = t;
      }
      return;
    }
  }
  __syncthreads();
  if (threadIdx.x < 32) scatter_pairs(idx, 0, T, K, E, run, p, status);
}

// Large calls: per-chunk counts ...
__global__ void __launch_bounds__(256) plan_count_kernel(const int32_t* __restrict__ idx, int T, int K, int E,
                                                         int chunk_tokens, Plan p) {
  extern __shared__ int cnt[];  // E + 1
  const int c = blockIdx.x;
  const int t0 = c * chunk_tokens, t1 = min(T, t0 + chunk_tokens);
  for (int i = threadIdx.x; i <= E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  for (int i = t0 * K + threadIdx.x; i < t1 * K; i += blockDim.x) {
    const int e = idx[i];
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i <= E; i += blockDim.x) p.hist[(int64_t)c * (E + 1) + i] = cnt[i];
}

// ... one block turns them into per-chunk start rows and the expert offsets ...
__global__ void __launch_bounds__(1024) plan_scan_kernel(int T, int E, int chunks, int has_shared, int align, Plan p,
                                                         int max_rows, int max_mtiles, uint32_t* status) {
  extern __shared__ int sm[];
  int* cnt = sm;           // E + 1
  int* off = cnt + E + 1;  // E + 2
  constexpr int kBatch = 16;  // chunk counts loaded together: one L2 round trip per batch, not per chunk
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int running = 0;
    for (int c0 = 0; c0 < chunks; c0 += kBatch) {
      int h[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) h[j] = c0 + j < chunks ? p.hist[(int64_t)(c0 + j) * (E + 1) + e] : 0;
#pragma unroll
      for (int j = 0; j < kBatch; ++j)
        if (c0 + j < chunks) {
          p.hist[(int64_t)(c0 + j) * (E + 1) + e] = running;
          running += h[j];
        }
    }
    cnt[e] = running;
  }
  if (threadIdx.x == 0) cnt[E] = has_shared ? T : 0;
  __syncthreads();
  finish_plan(cnt, off, E, align, p, max_rows, max_mtiles, status);
}

// ... and each chunk scatters its pairs (and its shared-expert rows).
__global__ void __launch_bounds__(256) plan_scatter_kernel(const int32_t* __restrict__ idx, int T, int K, int E,
                                                           int chunk_tokens, int has_shared, Plan p, int max_rows,
                                                           uint32_t* status) {
  extern __shared__ int run[];  // E + 1
  const int c = blockIdx.x;
  const int t0 = c * chunk_tokens, t1 = min(T, t0 + chunk_tokens);
  if (p.offsets[E + 1] > max_rows) return;
  for (int e = threadIdx.x; e < E; e += blockDim.x) run[e] = p.offsets[e] + p.hist[(int64_t)c * (E + 1) + e];
  if (has_shared) {
    const int base = p.offsets[E];
    for (int t = t0 + threadIdx.x; t < t1; t += blockDim.x) p.row_token[base + t] = t;
  }
  __syncthreads();
  if (threadIdx.x < 32) scatter_pairs(idx, t0, t1, K, E, run, p, status);
}

// The owner's plan of an expert-parallel step: chunk c covers slots
// [j0, j1) of recv block r = c / per_block, clipped to the block's real pairs
// (counts[r]); the pairs are single routes (K = 1) in slot order.
__device__ __forceinline__ void block_chunk(const int32_t* counts, int capacity, int chunk_slots, int per_block,
                                            int c, int* first, int* last) {
  const int r = c / per_block, cc = c - r * per_block;
  const int n = max(0, min(counts[r], capacity));
  const int j0 = cc * chunk_slots, j1 = min(j0 + chunk_slots, n);
  *first = r * capacity + j0;
  *last = r * capacity + max(j0, j1);
}

__global__ void __launch_bounds__(256) plan_blocks_count_kernel(const int32_t* __restrict__ ids,
                                                                const int32_t* __restrict__ counts, int capacity,
                                                                int chunk_slots, int per_block, int E, Plan p) {
  extern __shared__ int cnt[];  // E + 1
  int s0, s1;
  block_chunk(counts, capacity, chunk_slots, per_block, blockIdx.x, &s0, &s1);
  for (int i = threadIdx.x; i <= E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  for (int i = s0 + threadIdx.x; i < s1; i += blockDim.x) {
    const int e = ids[i];
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i <= E; i += blockDim.x) p.hist[(int64_t)blockIdx.x * (E + 1) + i] = cnt[i];
}

__global__ void __launch_bounds__(256) plan_blocks_scatter_kernel(const int32_t* __restrict__ ids,
                                                                  const int32_t* __restrict__ counts, int capacity,
                                                                  int chunk_slots, int per_block, int E, Plan p,
                                                                  int max_rows, uint32_t* status) {
  extern __shared__ int run[];  // E + 1
  const int c = blockIdx.x;
  if (p.offsets[E + 1] > max_rows) return;
  int s0, s1;
  block_chunk(counts, capacity, chunk_slots, per_block, c, &s0, &s1);
  for (int e = threadIdx.x; e < E; e += blockDim.x) run[e] = p.offsets[e] + p.hist[(int64_t)c * (E + 1) + e];
  __syncthreads();
  if (threadIdx.x < 32) scatter_pairs(ids, s0, s1, 1, E, run, p, status);
}

// The owner's plan of a small exchange (world * capacity <= 4096 slots) in
// one block: counts over the real slots, finish_plan, then warp 0 walks each
// sender's block in slot order (row_token[row] = slot, pair_pos[slot] = row).
__global__ void __launch_bounds__(1024) plan_blocks_small_kernel(const int32_t* __restrict__ ids,
                                                                 const int32_t* __restrict__ counts, int world,
                                                                 int capacity, int E, int align, Plan p, int max_rows,
                                                                 int max_mtiles, uint32_t* status) {
  extern __shared__ int sm[];
  int* cnt = sm;            // E + 1
  int* off = cnt + E + 1;   // E + 2
  int* run = off + E + 2;   // E + 1
  for (int i = threadIdx.x; i <= E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  for (int r = 0; r < world; ++r) {
    const int n = min(counts[r], capacity);
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
      const int e = ids[int64_t(r) * capacity + j];
      if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    }
  }
  __syncthreads();
  finish_plan(cnt, off, E, align, p, max_rows, max_mtiles, status);
  __syncthreads();
  if (off[E + 1] > max_rows) return;
  for (int i = threadIdx.x; i <= E; i += blockDim.x) run[i] = off[i];
  __syncthreads();
  if (threadIdx.x < 32)
    for (int r = 0; r < world; ++r)
      scatter_pairs(ids, r * capacity, r * capacity + min(counts[r], capacity), 1, E, run, p, status);
}

// x_sorted[r] = x[row_token[r]] (zeros for padding rows).  One warp per row.
__global__ void __launch_bounds__(256) gather_rows_kernel(const uint16_t* __restrict__ x, Plan p, int E, int H,
                                                          uint16_t* __restrict__ xs) {
  const int rows = p.offsets[E + 1];
  const int lane = threadIdx.x & 31;
  const int pieces = H / 8;
  for (int r = blockIdx.x * 8 + (threadIdx.x >> 5); r < rows; r += gridDim.x * 8) {
    const int t = p.row_token[r];
    uint4* dst = reinterpret_cast<uint4*>(xs + (int64_t)r * H);
    if (t >= 0) {
      const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)t * H);
      for (int i = lane; i < pieces; i += 32) dst[i] = src[i];
    } else {
      for (int i = lane; i < pieces; i += 32) dst[i] = make_uint4(0, 0, 0, 0);
    }
  }
}

// out[t] = sum_k w[t, k] * routed[pair_pos[t, k]] + g(t) * routed[offsets[E] + t],
// an fp32 sum in k order, rounded once to bf16 (qwen4_exp.py:1049-1051,
// deepseek_v41/moe.py:110-112, QwenNative/kernels.metal:185-194).
// g(t) = sg[t] (sigmoid gate) or 1.  Eight columns per thread.
// DENSE: `routed` holds the pairs -- pair (t, k) at row p.pair_pos[t * K + k]
// when p.pair_pos is set, else at row t * K + k -- and `shared_rows` the
// shared expert's rows; otherwise both come from the plan's sorted rows.
template <bool DENSE>
__global__ void __launch_bounds__(256) combine_kernel(const uint16_t* __restrict__ routed, Plan p,
                                                      const float* __restrict__ w, const float* __restrict__ sg,
                                                      int shared_kind, int T, int H, int E, int K,
                                                      const uint16_t* __restrict__ shared_rows,
                                                      uint16_t* __restrict__ out) {
  const int t = blockIdx.y;
  const int h0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (h0 >= H) return;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
  // the shared expert's row is loaded first (it depends on no pair) and added last
  uint4 sv = make_uint4(0, 0, 0, 0);
  float g = 0.0f;
  if (shared_kind != WM_SHARED_NONE) {
    g = shared_kind == WM_SHARED_SIGMOID_GATE ? sg[t] : 1.0f;
    const uint16_t* srow = DENSE ? shared_rows + (int64_t)t * H : routed + (int64_t)(p.offsets[E] + t) * H;
    sv = *reinterpret_cast<const uint4*>(srow + h0);
  }
  // eight pairs' loads in flight at a time; the sum keeps k order
  for (int k0 = 0; k0 < K; k0 += 8) {
    int pos[8];
    float wk[8];
    uint4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k = k0 + j;
      pos[j] = k < K ? ((DENSE && p.pair_pos == nullptr) ? t * K + k : p.pair_pos[(int64_t)t * K + k]) : -1;
      wk[j] = k < K ? w[(int64_t)t * K + k] : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      v[j] = pos[j] >= 0 ? *reinterpret_cast<const uint4*>(routed + (int64_t)pos[j] * H + h0) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (pos[j] < 0) continue;
      float2 f;
      f = unpack_bf16x2(v[j].x); acc[0] = fmaf(wk[j], f.x, acc[0]); acc[1] = fmaf(wk[j], f.y, acc[1]);
      f = unpack_bf16x2(v[j].y); acc[2] = fmaf(wk[j], f.x, acc[2]); acc[3] = fmaf(wk[j], f.y, acc[3]);
      f = unpack_bf16x2(v[j].z); acc[4] = fmaf(wk[j], f.x, acc[4]); acc[5] = fmaf(wk[j], f.y, acc[5]);
      f = unpack_bf16x2(v[j].w); acc[6] = fmaf(wk[j], f.x, acc[6]); acc[7] = fmaf(wk[j], f.y, acc[7]);
    }
  }
  if (shared_kind != WM_SHARED_NONE) {
    const uint4 v = sv;
    float2 f;
    f = unpack_bf16x2(v.x); acc[0] = fmaf(g, f.x, acc[0]); acc[1] = fmaf(g, f.y, acc[1]);
    f = unpack_bf16x2(v.y); acc[2] = fmaf(g, f.x, acc[2]); acc[3] = fmaf(g, f.y, acc[3]);
    f = unpack_bf16x2(v.z); acc[4] = fmaf(g, f.x, acc[4]); acc[5] = fmaf(g, f.y, acc[5]);
    f = unpack_bf16x2(v.w); acc[6] = fmaf(g, f.x, acc[6]); acc[7] = fmaf(g, f.y, acc[7]);
  }
  uint4 o;
  o.x = pack_bf16x2(acc[0], acc[1]);
  o.y = pack_bf16x2(acc[2], acc[3]);
  o.z = pack_bf16x2(acc[4], acc[5]);
  o.w = pack_bf16x2(acc[6], acc[7]);
  *reinterpret_cast<uint4*>(out + (int64_t)t * H + h0) = o;
}

// routed_out[t, k] = routed[pair_pos[t, k]] (the [T, K, H] layout of
// StreamingExperts.__call__).  One warp per pair.
__global__ void __launch_bounds__(256) unpermute_kernel(const uint16_t* __restrict__ routed, Plan p, int TK, int H,
                                                        uint16_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  for (int i = blockIdx.x * 8 + (threadIdx.x >> 5); i < TK; i += gridDim.x * 8) {
    const int pos = p.pair_pos[i];
    uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)i * H);
    if (pos < 0) {
      for (int j = lane; j < H / 8; j += 32) dst[j] = make_uint4(0, 0, 0, 0);
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(routed + (int64_t)pos * H);
    for (int j = lane; j < H / 8; j += 32) dst[j] = src[j];
  }
}

// ------------------------------------------------------------------ launchers

void launch_plan(const int32_t* idx, int T, int K, int E, bool has_shared, int align, const Plan& p, int max_rows,
                 int max_mtiles, int max_chunks, uint32_t* status, cudaStream_t stream, int* launches) {
  if (T * K <= 8192) {
    const size_t smem = size_t(3 * (E + 2)) * sizeof(int) + size_t(E + 2) * sizeof(unsigned long long);
    plan_small_kernel<<<1, 1024, smem, stream>>>(idx, T, K, E, has_shared ? 1 : 0, align, p, max_rows, max_mtiles,
                                                  status);
    *launches += 1;
    return;
  }
  int chunk_tokens = 64;
  while ((T + chunk_tokens - 1) / chunk_tokens > max_chunks) chunk_tokens *= 2;
  const int chunks = (T + chunk_tokens - 1) / chunk_tokens;
  const size_t smem1 = size_t(E + 1) * sizeof(int);
  plan_count_kernel<<<chunks, 256, smem1, stream>>>(idx, T, K, E, chunk_tokens, p);
  const size_t smem2 = size_t(2 * (E + 2)) * sizeof(int);
  plan_scan_kernel<<<1, 1024, smem2, stream>>>(T, E, chunks, has_shared ? 1 : 0, align, p, max_rows, max_mtiles,
                                               status);
  plan_scatter_kernel<<<chunks, 256, smem1, stream>>>(idx, T, K, E, chunk_tokens, has_shared ? 1 : 0, p, max_rows,
                                                      status);
  *launches += 3;
}

void launch_plan_blocks(const int32_t* ids, const int32_t* counts, int world, int capacity, int E, int align,
                        const Plan& p, int max_rows, int max_mtiles, int max_chunks, uint32_t* status,
                        cudaStream_t stream, int* launches) {
  if (int64_t(world) * capacity <= 4096) {  // decode-sized exchanges: one block
    const size_t smem = size_t(3 * (E + 2)) * sizeof(int);
    plan_blocks_small_kernel<<<1, 1024, smem, stream>>>(ids, counts, world, capacity, E, align, p, max_rows, max_mtiles,
                                                        status);
    *launches += 1;
    return;
  }
  int chunk_slots = 64;
  while (int64_t(world) * ((capacity + chunk_slots - 1) / chunk_slots) > max_chunks) chunk_slots *= 2;
  const int per_block = (capacity + chunk_slots - 1) / chunk_slots;
  const int chunks = world * per_block;
  const size_t smem1 = size_t(E + 1) * sizeof(int);
  plan_blocks_count_kernel<<<chunks, 256, smem1, stream>>>(ids, counts, capacity, chunk_slots, per_block, E, p);
  const size_t smem2 = size_t(2 * (E + 2)) * sizeof(int);
  plan_scan_kernel<<<1, 1024, smem2, stream>>>(0, E, chunks, 0, align, p, max_rows, max_mtiles, status);
  plan_blocks_scatter_kernel<<<chunks, 256, smem1, stream>>>(ids, counts, capacity, chunk_slots, per_block, E, p,
                                                             max_rows, status);
  *launches += 3;
}

void launch_gather_rows(const uint16_t* x, const Plan& p, int E, int H, uint16_t* xs, int num_sms,
                        cudaStream_t stream) {
  gather_rows_kernel<<<num_sms * 8, 256, 0, stream>>>(x, p, E, H, xs);
}

void launch_combine(const uint16_t* routed, const Plan& p, const float* w, const float* sg, int shared_kind, int T,
                    int H, int E, int K, uint16_t* out, cudaStream_t stream) {
  dim3 grid((H / 8 + 255) / 256, T);
  combine_kernel<false><<<grid, 256, 0, stream>>>(routed, p, w, sg, shared_kind, T, H, E, K, nullptr, out);
}

void launch_combine_dense(const uint16_t* pairs, const int32_t* pair_pos, const float* w, const float* sg,
                          int shared_kind, int T, int H, int K, const uint16_t* shared_rows, uint16_t* out,
                          cudaStream_t stream) {
  dim3 grid((H / 8 + 255) / 256, T);
  Plan p{};
  p.pair_pos = const_cast<int32_t*>(pair_pos);
  combine_kernel<true><<<grid, 256, 0, stream>>>(pairs, p, w, sg, shared_kind, T, H, 0, K, shared_rows, out);
}

// owner[i] = idx[i] / per_rank (the rank that holds expert idx[i]).
__global__ void ep_owner_kernel(const int32_t* __restrict__ idx, int P, int per_rank, int world,
                                int32_t* __restrict__ owner, uint32_t* status) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < P; i += gridDim.x * blockDim.x) {
    const int e = idx[i];
    if (e < 0 || e >= per_rank * world) {
      report_status(status, kStatusBadExpert, (uint32_t)i);
      owner[i] = -1;
    } else {
      owner[i] = e / per_rank;
    }
  }
}

// After the plan over owners: each pair's slot in send order, its expert id
// local to the owner at that slot, and the per-owner counts.  With
// capacity > 0 owner r's pairs take slots [r * capacity, r * capacity +
// count_r), the other slots get expert id -1 (padding), and the x rows are
// copied here (one warp per pair); with capacity 0 the slots are packed.
__global__ void ep_finish_kernel(const int32_t* __restrict__ idx, Plan p, int T, int K, int per_rank, int world,
                                 int capacity, int32_t* __restrict__ send_counts, int32_t* __restrict__ pair_pos,
                                 int32_t* __restrict__ send_eid, const uint16_t* __restrict__ x, int H,
                                 uint16_t* __restrict__ send_x) {
  const int P = T * K;
  const int gtid = blockIdx.x * blockDim.x + threadIdx.x, nthreads = gridDim.x * blockDim.x;
  if (capacity > 0)
    for (int i = gtid; i < world * capacity; i += nthreads) {
      const int r = i / capacity, j = i - r * capacity;
      if (j >= p.counts[r]) send_eid[i] = -1;
    }
  for (int i = gtid; i < P; i += nthreads) {
    const int pos = p.pair_pos[i];
    if (pos < 0) {
      pair_pos[i] = -1;
      continue;
    }
    const int e = idx[i], r = e / per_rank;
    const int slot = capacity > 0 ? r * capacity + (pos - p.offsets[r]) : pos;
    pair_pos[i] = slot;
    send_eid[slot] = e - r * per_rank;
  }
  if (blockIdx.x == 0)
    for (int r = threadIdx.x; r < world; r += blockDim.x) send_counts[r] = p.counts[r];
  if (capacity > 0) {
    const int lane = threadIdx.x & 31, warps = nthreads >> 5;
    for (int i = gtid >> 5; i < P; i += warps) {
      const int pos = p.pair_pos[i];
      if (pos < 0) continue;
      const int r = idx[i] / per_rank;
      const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)(i / K) * H);
      uint4* dst = reinterpret_cast<uint4*>(send_x + (int64_t)(r * capacity + (pos - p.offsets[r])) * H);
      for (int j = lane; j < H / 8; j += 32) dst[j] = src[j];
    }
  }
}

void launch_ep_owner(const int32_t* idx, int P, int per_rank, int world, int32_t* owner, uint32_t* status,
                     int num_sms, cudaStream_t stream) {
  ep_owner_kernel<<<num_sms, 256, 0, stream>>>(idx, P, per_rank, world, owner, status);
}

void launch_ep_finish(const int32_t* idx, const Plan& p, int T, int K, int per_rank, int world, int capacity,
                      int32_t* send_counts, int32_t* pair_pos, int32_t* send_eid, const uint16_t* x, int H,
                      uint16_t* send_x, int num_sms, cudaStream_t stream) {
  ep_finish_kernel<<<num_sms, 256, 0, stream>>>(idx, p, T, K, per_rank, world, capacity, send_counts, pair_pos,
                                                send_eid, x, H, send_x);
}

void launch_unpermute(const uint16_t* routed, const Plan& p, int TK, int H, uint16_t* out, int num_sms,
                      cudaStream_t stream) {
  unpermute_kernel<<<num_sms * 4, 256, 0, stream>>>(routed, p, TK, H, out);
}


// ------------------------------------------------------------------ f16 row copies
// The prescaled f16 copies of the sorted rows that the register-direct decode
// kernel and the MXFP4 grouped GEMM multiply (exact: a power-of-two scale per row).

// 2^k for a row whose largest magnitude has float bits `maxbits`: the scaled
// row's largest element lands in [2^14, 2^15).
__device__ __forceinline__ float row_prescale(uint32_t maxbits) {
  if (maxbits == 0u || maxbits >= 0x7f800000u) return 1.0f;
  const int e = int(maxbits >> 23) - 127;  // floor(log2(max)) for normal values
  const int k = min(max(14 - e, -100), 100);
  return exp2f(float(k));
}

// One row of bf16 pieces (16 bytes) -> f16 pieces scaled by k2.
__device__ __forceinline__ uint4 f16_piece(const uint4 v, float k2) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t q[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = unpack_bf16x2(w[j]);
    const __half2 hh = __floats2half2_rn(f.x * k2, f.y * k2);
    q[j] = *reinterpret_cast<const uint32_t*>(&hh);
  }
  return make_uint4(q[0], q[1], q[2], q[3]);
}

// Largest |bf16| of a piece, as ordered bits (a positive float's bits order like its value).
__device__ __forceinline__ uint32_t piece_absmax_bits(const uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t m = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) m = max(m, max((w[j] & 0x7fffu) << 16, w[j] & 0x7fff0000u));
  return m;
}

// Sorted f16 copy of the activation rows: out[r] = x[row_token[r]] * 2^k,
// scale[r] = 2^k (largest magnitude of the row lands in [2^14, 2^15)).
// One warp per sorted row; with NV > 0 (rows of at most 256 NV bf16) the row
// stays in registers, so it is read once with all its loads in flight.
// Padding rows (row_token < 0) only get scale 1: their data is left as the
// workspace holds it (zero from creation, or an earlier call's finite f16
// row).  Every product and epilogue of the expert kernels is row-local (a row
// of A gives a row of D, a token column gives a column), and no padding row is
// read by the combine, so what a padding row holds never reaches an output.
template <int NV>
__global__ void __launch_bounds__(256) gather_f16_kernel(const uint16_t* __restrict__ x, Plan p, int E, int H,
                                                         uint16_t* __restrict__ out, float* __restrict__ scale) {
  constexpr int kRowPieces = NV > 0 ? NV : 1;
  const int rows = p.offsets[E + 1];
  const int lane = threadIdx.x & 31;
  const int pieces = H / 8, per_lane = (pieces + 31) / 32;
  for (int r = blockIdx.x * 8 + (threadIdx.x >> 5); r < rows; r += gridDim.x * 8) {
    const int t = p.row_token[r];
    if (t < 0) {
      if (lane == 0) scale[r] = 1.0f;
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(x + int64_t(t) * H);
    uint4* dst = reinterpret_cast<uint4*>(out + int64_t(r) * H);
    if (NV > 0) {
      // the whole row in registers: one read of it, all loads in flight at once
      uint4 v[kRowPieces];
      uint32_t m = 0;
#pragma unroll
      for (int j = 0; j < kRowPieces; ++j) {
        const int i = lane + 32 * j;
        v[j] = (t >= 0 && j < per_lane && i < pieces) ? src[i] : make_uint4(0, 0, 0, 0);
        m = max(m, piece_absmax_bits(v[j]));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float k2 = row_prescale(m);
#pragma unroll
      for (int j = 0; j < kRowPieces; ++j) {
        const int i = lane + 32 * j;
        if (j < per_lane && i < pieces) dst[i] = t >= 0 ? f16_piece(v[j], k2) : make_uint4(0, 0, 0, 0);
      }
      if (lane == 0) scale[r] = k2;
      continue;
    }
    uint32_t m = 0;
    if (t >= 0)
      for (int i = lane; i < pieces; i += 32) m = max(m, piece_absmax_bits(src[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float k2 = row_prescale(m);
    for (int i = lane; i < pieces; i += 32) dst[i] = t >= 0 ? f16_piece(src[i], k2) : make_uint4(0, 0, 0, 0);
    if (lane == 0) scale[r] = k2;
  }
}

// act rows -> f16 with the prescale of their |act| maxima; a warp takes two
// rows per step (four when a row is at most 64 pieces) so their loads overlap.
__global__ void __launch_bounds__(256) act_f16_kernel(const uint16_t* __restrict__ act, Plan p, int E, int I,
                                                      uint16_t* __restrict__ out, float* __restrict__ scale) {
  constexpr int R = 4;
  const int rows = p.offsets[E + 1];
  const int lane = threadIdx.x & 31;
  const int pieces = I / 8;
  const int warps = gridDim.x * 8;
  for (int r0 = (blockIdx.x * 8 + (threadIdx.x >> 5)) * R; r0 < rows; r0 += warps * R) {
    float k2[R];
#pragma unroll
    for (int q = 0; q < R; ++q) k2[q] = r0 + q < rows ? row_prescale(p.rowmax[r0 + q]) : 1.0f;
    for (int i0 = lane; i0 < pieces; i0 += 32 * 2) {
      uint4 v[R][2];
#pragma unroll
      for (int q = 0; q < R; ++q)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int i = i0 + 32 * h;
          v[q][h] = (r0 + q < rows && i < pieces) ? reinterpret_cast<const uint4*>(act + int64_t(r0 + q) * I)[i]
                                                  : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
      for (int q = 0; q < R; ++q)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int i = i0 + 32 * h;
          if (r0 + q < rows && i < pieces)
            reinterpret_cast<uint4*>(out + int64_t(r0 + q) * I)[i] = f16_piece(v[q][h], k2[q]);
        }
    }
    if (lane < R && r0 + lane < rows) {
      float k = 1.0f;
#pragma unroll
      for (int q = 0; q < R; ++q)
        if (q == lane) k = k2[q];
      scale[r0 + lane] = k;
    }
  }
}

// Tiles of 128 weight rows and 64 K; a row's E8M0 bytes (a multiple of 16)
// come as one TMA box; the two scale slots fit shared memory up to K = 7168.
bool decode_shape_ok(int H, int I) { return H % 512 == 0 && I % 512 == 0 && H <= 7168 && I <= 7168; }


void launch_gather_f16(const uint16_t* x, const Plan& p, int E, int H, uint16_t* out, float* scale, int num_sms,
                       cudaStream_t stream) {
  const int per_lane = (H / 8 + 31) / 32;
  if (per_lane <= 8)
    gather_f16_kernel<8><<<num_sms * 4, 256, 0, stream>>>(x, p, E, H, out, scale);
  else if (per_lane <= 16)
    gather_f16_kernel<16><<<num_sms * 4, 256, 0, stream>>>(x, p, E, H, out, scale);
  else
    gather_f16_kernel<0><<<num_sms * 4, 256, 0, stream>>>(x, p, E, H, out, scale);
}

void launch_act_f16(const uint16_t* act, const Plan& p, int E, int I, uint16_t* out, float* scale, int num_sms,
                    cudaStream_t stream) {
  act_f16_kernel<<<num_sms * 4, 256, 0, stream>>>(act, p, E, I, out, scale);
}

}  // namespace wm
