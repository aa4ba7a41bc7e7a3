// Expert-parallel exchanges over NVLink peer memory (no collective library).
//
// Every rank owns one exchange buffer (recv_x, recv_e, back, flags), mapped
// into its peers' address spaces through CUDA IPC.  One layer step:
//
//   dispatch  ep_send_kernel stores each (token, k) pair's x row and
//             owner-local expert id straight into the owner's recv block for
//             this rank (slot rank * capacity + j), marks the block's unused
//             slots with id -1, and -- after every CTA's stores are fenced at
//             system scope -- the last CTA raises this rank's dispatch flag on
//             every peer to the step number;
//   wait      ep_wait_kernel: one lane per peer polls the local flag (bounded:
//             after 2 s it records a timeout in the status word and returns);
//   experts   the owner runs its experts on recv_x (padding ids skipped);
//   return    ep_return_kernel stores each valid result row into the source
//             rank's `back` buffer at the slot the pair was sent from, then
//             raises the return flags the same way; after a wait the source
//             rank combines, reading pair (t, k) at its slot.
//
// Only real pairs cross NVLink (the fixed-capacity all-to-all of the
// collective path moves every padded slot), and nothing waits on the host,
// so a step can be captured in one CUDA graph.  The step number lives on the
// device (ep_begin_kernel increments it), so graph replays signal fresh
// values.  The reference runs its experts on one device; this is the
// B200-native counterpart of the expert-parallel plan, not a port.
#include <algorithm>

#include "wm_kernels.h"

namespace wm {

namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// After this CTA's stores to peer memory: fence them at system scope, take a
// ticket, and let the last CTA of the grid raise the flags (one per peer) to
// the step number and reset the ticket for the next exchange.
__device__ __forceinline__ void signal_peers(const EpPeers& pe, int world) {
  __shared__ int last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(pe.ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence_system();
  const uint32_t step = *pe.epoch;
  if (threadIdx.x < world) st_release_sys(pe.flag[threadIdx.x], step);
  if (threadIdx.x == 0) *pe.ticket = 0u;
}

// One row of H bf16 from src to dst (either may be a peer's memory) by one
// warp: four 16-byte loads in flight per lane before their stores, so a warp
// is not bound by one load's latency per 512 bytes.
__device__ __forceinline__ void copy_row(uint4* __restrict__ dst, const uint4* __restrict__ src, int H, int lane) {
  const int n = H / 8;
  int c = lane;
  for (; c + 96 < n; c += 128) {
    const uint4 v0 = src[c], v1 = src[c + 32], v2 = src[c + 64], v3 = src[c + 96];
    dst[c] = v0;
    dst[c + 32] = v1;
    dst[c + 64] = v2;
    dst[c + 96] = v3;
  }
  for (; c < n; c += 32) dst[c] = src[c];
}

}  // namespace

__global__ void ep_begin_kernel(uint32_t* epoch) { epoch[0] += 1u; }

// Dispatch of the pairs after the plan over owners (as ep_finish_kernel with a
// capacity, but into the owners' buffers).
constexpr int kCopyThreads = 512;  // exchange kernels: 2 CTAs of 16 warps per SM

__global__ void __launch_bounds__(kCopyThreads) ep_send_kernel(const int32_t* __restrict__ idx, Plan p, int T, int K,
                                                      int per_rank, int world, int capacity,
                                                      int32_t* __restrict__ pair_pos, const uint16_t* __restrict__ x,
                                                      int H, const EpPeers pe) {
  const int P = T * K;
  const int gtid = blockIdx.x * blockDim.x + threadIdx.x, nthreads = gridDim.x * blockDim.x;
  for (int i = gtid; i < world * capacity; i += nthreads) {
    const int r = i / capacity, j = i - r * capacity;
    if (j >= p.counts[r]) pe.ids[r][j] = -1;
  }
  if (gtid < world) pe.count[gtid][0] = p.counts[gtid];  // the owner plans over real pairs only
  for (int i = gtid; i < P; i += nthreads) {
    const int pos = p.pair_pos[i];
    if (pos < 0) {
      pair_pos[i] = -1;
      continue;
    }
    const int e = idx[i], r = e / per_rank, j = pos - p.offsets[r];
    pair_pos[i] = r * capacity + j;
    pe.ids[r][j] = e - r * per_rank;
  }
  const int lane = threadIdx.x & 31, warps = nthreads >> 5;
  for (int i = gtid >> 5; i < P; i += warps) {
    const int pos = p.pair_pos[i];
    if (pos < 0) continue;
    const int r = idx[i] / per_rank;
    copy_row(reinterpret_cast<uint4*>(pe.rows[r] + int64_t(pos - p.offsets[r]) * H),
             reinterpret_cast<const uint4*>(x + int64_t(i / K) * H), H, lane);
  }
  signal_peers(pe, world);
}

// The whole dispatch of a small call (P = T * K <= kSmallPairs pairs) in one
// launch: every CTA ranks all pairs by owner in shared memory (warp 0, 32
// pairs a step, a pair's slot = its owner's running count plus the earlier
// lanes naming the same owner: the (token, k) order of the plan over owners),
// then the CTAs share the row copies, ids and padding ids; CTA 0 advances the
// step number first (the last CTA's flags carry it) and writes the counts.
constexpr int kSmallPairs = 4096;

__global__ void __launch_bounds__(kCopyThreads) ep_dispatch_small_kernel(
    const int32_t* __restrict__ idx, int T, int K, int per_rank, int world, int capacity, int32_t* __restrict__ pair_pos,
    const uint16_t* __restrict__ x, int H, const EpPeers pe, uint32_t* epoch, uint32_t* status) {
  __shared__ int16_t slot[kSmallPairs];  // pair -> slot within its owner's block (-1: bad id)
  __shared__ int8_t own[kSmallPairs];
  __shared__ int count[kMaxEpRanks];
  const int P = T * K;
  if (blockIdx.x == 0 && threadIdx.x == 0) epoch[0] += 1u;
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    const int e = idx[i];
    const bool ok = e >= 0 && e < per_rank * world;
    own[i] = ok ? int8_t(e / per_rank) : int8_t(-1);
    if (!ok && blockIdx.x == 0) report_status(status, kStatusBadExpert, uint32_t(i));
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int run = 0;  // lane r < world: owner r's running count
    const unsigned lt_mask = (1u << lane) - 1u;
    for (int i0 = 0; i0 < P; i0 += 32) {
      const int i = i0 + lane;
      const int r = i < P ? own[i] : -1;
      const unsigned same = __match_any_sync(0xffffffffu, r);
      const int base = __shfl_sync(0xffffffffu, run, r < 0 ? 0 : r);
      if (i < P) slot[i] = r < 0 ? int16_t(-1) : int16_t(base + __popc(same & lt_mask));
      // owner q's lane adds the pairs of this step that name it
      for (int q = 0; q < world; ++q) {
        const unsigned hits = __ballot_sync(0xffffffffu, r == q);
        if (lane == q) run += __popc(hits);
      }
    }
    if (lane < world) count[lane] = run;
  }
  __syncthreads();
  const int gtid = blockIdx.x * blockDim.x + threadIdx.x, nthreads = gridDim.x * blockDim.x;
  if (gtid < world) pe.count[gtid][0] = count[gtid];  // the owner plans over real pairs only
  for (int i = gtid; i < world * capacity; i += nthreads) {
    const int r = i / capacity, j = i - r * capacity;
    if (j >= count[r]) pe.ids[r][j] = -1;
  }
  for (int i = gtid; i < P; i += nthreads) {
    const int r = own[i];
    if (r < 0) {
      pair_pos[i] = -1;
      continue;
    }
    pair_pos[i] = r * capacity + slot[i];
    pe.ids[r][slot[i]] = idx[i] - r * per_rank;
  }
  const int lane = threadIdx.x & 31, warps = nthreads >> 5;
  for (int i = gtid >> 5; i < P; i += warps) {
    const int r = own[i];
    if (r < 0) continue;
    copy_row(reinterpret_cast<uint4*>(pe.rows[r] + int64_t(slot[i]) * H),
             reinterpret_cast<const uint4*>(x + int64_t(i / K) * H), H, lane);
  }
  signal_peers(pe, world);
}

// Result rows back to the ranks that sent the pairs: slot s of recv block r
// (valid when its expert id is >= 0) goes to slot j of rank r's back block
// for this rank.
__global__ void __launch_bounds__(kCopyThreads) ep_return_kernel(const uint16_t* __restrict__ y,
                                                        const int32_t* __restrict__ recv_e, int world, int capacity,
                                                        int H, const EpPeers pe) {
  const int lane = threadIdx.x & 31, warps = gridDim.x * blockDim.x >> 5;
  for (int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; s < world * capacity; s += warps) {
    if (recv_e[s] < 0) continue;
    const int r = s / capacity, j = s - r * capacity;
    copy_row(reinterpret_cast<uint4*>(pe.rows[r] + int64_t(j) * H), reinterpret_cast<const uint4*>(y + int64_t(s) * H),
             H, lane);
  }
  signal_peers(pe, world);
}

// Result rows back to their senders straight from the owner's sorted rows:
// slot j < counts[r] of recv block r is row pair_pos[r * capacity + j] of
// `routed`, and goes to slot j of rank r's back block for this rank.  Fuses
// the unpermute of the owner's rows with the return.
__global__ void __launch_bounds__(kCopyThreads) ep_return_sorted_kernel(const uint16_t* __restrict__ routed,
                                                               const int32_t* __restrict__ pair_pos,
                                                               const int32_t* __restrict__ counts, int world,
                                                               int capacity, int H, const EpPeers pe) {
  const int lane = threadIdx.x & 31, warps = gridDim.x * blockDim.x >> 5;
  for (int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; s < world * capacity; s += warps) {
    const int r = s / capacity, j = s - r * capacity;
    if (j >= min(counts[r], capacity)) continue;
    const int row = pair_pos[s];
    if (row < 0) continue;
    copy_row(reinterpret_cast<uint4*>(pe.rows[r] + int64_t(j) * H),
             reinterpret_cast<const uint4*>(routed + int64_t(row) * H), H, lane);
  }
  signal_peers(pe, world);
}

// Bounded wait until every peer's flag has reached this step.
__global__ void ep_wait_kernel(const uint32_t* flags, int world, const uint32_t* epoch, uint32_t* status, int code) {
  const int r = threadIdx.x;
  if (r >= world) return;
  const uint32_t step = *epoch;
  const uint64_t start = global_timer_ns();
  for (uint32_t spin = 0; ld_acquire_sys(flags + r) < step; ++spin) {
    __nanosleep(64);
    if ((spin & 63u) == 63u && global_timer_ns() - start > 2000000000ull) {
      report_status(status, kStatusWaitTimeout, uint32_t(code * 16 + r));
      return;
    }
  }
}

void launch_ep_begin(uint32_t* epoch, cudaStream_t stream) { ep_begin_kernel<<<1, 1, 0, stream>>>(epoch); }

void launch_ep_send(const int32_t* idx, const Plan& p, int T, int K, int per_rank, int world, int capacity,
                    int32_t* pair_pos, const uint16_t* x, int H, const EpPeers& pe, int num_sms,
                    cudaStream_t stream) {
  ep_send_kernel<<<2 * num_sms, kCopyThreads, 0, stream>>>(idx, p, T, K, per_rank, world, capacity, pair_pos, x, H, pe);
}

bool ep_dispatch_small_ok(int P, int world, int capacity) {
  return P <= kSmallPairs && world <= kMaxEpRanks && capacity <= 32767;
}

void launch_ep_dispatch_small(const int32_t* idx, int T, int K, int per_rank, int world, int capacity,
                              int32_t* pair_pos, const uint16_t* x, int H, const EpPeers& pe, uint32_t* epoch,
                              uint32_t* status, int num_sms, cudaStream_t stream) {
  const int P = T * K;
  const int grid = std::max(1, std::min(2 * num_sms, (P + 15) / 16));  // 16 rows per CTA at least
  ep_dispatch_small_kernel<<<grid, kCopyThreads, 0, stream>>>(idx, T, K, per_rank, world, capacity, pair_pos, x, H, pe,
                                                              epoch, status);
}

void launch_ep_return(const uint16_t* y, const int32_t* recv_e, int world, int capacity, int H, const EpPeers& pe,
                      int num_sms, cudaStream_t stream) {
  ep_return_kernel<<<2 * num_sms, kCopyThreads, 0, stream>>>(y, recv_e, world, capacity, H, pe);
}

// Raises this rank's return flag on every peer to the step number.
__global__ void ep_signal_kernel(const EpPeers pe, int world) {
  __threadfence_system();
  const uint32_t step = *pe.epoch;
  if (threadIdx.x < world) st_release_sys(pe.flag[threadIdx.x], step);
}

void launch_ep_signal(const EpPeers& pe, int world, cudaStream_t stream) {
  ep_signal_kernel<<<1, 32, 0, stream>>>(pe, world);
}

void launch_ep_return_sorted(const uint16_t* routed, const int32_t* pair_pos, const int32_t* counts, int world,
                             int capacity, int H, const EpPeers& pe, int num_sms, cudaStream_t stream) {
  ep_return_sorted_kernel<<<2 * num_sms, kCopyThreads, 0, stream>>>(routed, pair_pos, counts, world, capacity, H, pe);
}

void launch_ep_wait(const uint32_t* flags, int world, const uint32_t* epoch, uint32_t* status, int code,
                    cudaStream_t stream) {
  ep_wait_kernel<<<1, 32, 0, stream>>>(flags, world, epoch, status, code);
}

}  // namespace wm
