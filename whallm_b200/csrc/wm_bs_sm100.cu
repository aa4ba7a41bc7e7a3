// Decode path on tcgen05 block-scaled MMA (kind::mxf8f6f4): the MXFP4 expert
// weights go from the blob to shared memory by TMA and into the tensor cores
// as they are -- E2M1 elements with their E8M0 group scales applied by the
// MMA itself -- so no CUDA core touches a weight.
//
// Reference arithmetic: the decode GEMVs expert_linear4 / expert_group<R, K>
// (QwenNative/kernels.metal:1186-1219, DeepSeekNative/kernels.metal:933-987)
// and mx.quantized_matmul(mode="mxfp4", group_size=32) (model.py:504-513):
// exact dequantised weights times the activation rows, fp32 accumulation.
//
// Operands of one MMA (M = 128 weight rows, N = 32, K = 32):
//   A  weights: E2M1 nibbles straight from the blob (the TMA type
//      16U4_ALIGN16B spreads every 8 packed bytes over 16 bytes of shared
//      memory, the layout kind::mxf8f6f4 reads), K-major, 128-byte swizzle;
//      scale factors = the blob's E8M0 bytes (UE8M0), one per row and 32 K.
//   B  token rows as two E4M3 parts: hi = e4m3(x / s_hi) and lo =
//      e4m3((x - hi * s_hi) / s_lo) with power-of-two scales per row and 32 K
//      (UE8M0, chosen so no element saturates), hi rows in N 0..15, lo rows
//      in N 16..31, so one MMA multiplies the weights by both parts and the
//      epilogue adds the two column halves.  x = hi * s_hi + lo * s_lo + r
//      with |r| <= 2^-8 |x| per element: the layer outputs stay within
//      ~1e-3 of the exact products (measured on the CPU against exact
//      arithmetic at the config-2 and config-4 shapes: 8.5e-4 and 8.8e-4 of
//      max|y|; one E4M3 part alone gives 4-5e-2).
//   D  fp32 in TMEM, 128 lanes (weight rows) x 32 columns.
// Scale factors reach TMEM with tcgen05.cp (32x128b, copied to the four lane
// quarters): a 512-byte atom per stage in which row r (16 bytes) holds, for
// the M rows r, r + 32, r + 64, r + 96, the four UE8M0 bytes of the stage's
// four 32-K blocks; the MMA of block kk reads byte kk (the scale-factor id).
//
// Work: an item is (16-token tile of one expert, 128 weight rows); for
// gate/up the 128 rows are 64 gate and the 64 up rows of the same features
// (one 4-D TMA box over both halves of w13), so SwiGLU runs in the epilogue, which also quantises the
// act rows (hi / lo E4M3 + UE8M0, 32 features per warp = one scale block) for
// the down kernel.  One persistent CTA per SM; warp roles:
//   warp 0     TMA producer, two copies per stage: the A box (gate and up
//              rows in one 4-D box) and the B tile image with its scale atom;
//              every fourth stage the raw E8M0 rows of the next four stages
//   warp 1     scale warp: raw E8M0 rows -> the stage's scale-factor atom
//   warp 2     TMEM owner and MMA issuer (one elected lane)
//   warps 4-7  epilogue (TMEM lane quarters 0..3)
// Every mbarrier wait is bounded (2 s); on a timeout the kernel records the
// status, the other roles unwind and TMEM is freed.
#include <cuda.h>

#include <algorithm>
#include <type_traits>

#include "wm_bs_common.cuh"
#include "wm_kernels.h"
#include "wm_plan.cuh"
#include "wm_route.cuh"

namespace wm {

namespace {

constexpr int kBM = 128;         // weight rows per item (MMA M)
constexpr int kBK = 128;         // K per stage (four 32-K scale blocks)
constexpr int kTokTile = 16;     // tokens per item; N = 2 x 16 (hi and lo parts)
constexpr int kN = 2 * kTokTile;
constexpr int kThreads = 256;
constexpr int kEpiWarp0 = 4;
constexpr int kRawSlots = 3;     // raw E8M0 slots, four stages each
constexpr int kAccCols = kN;     // TMEM columns per accumulator
constexpr uint32_t kTmemCols = 128;
constexpr uint32_t kSfCol0 = 2 * kAccCols;  // scale factors after the two accumulators
constexpr int kMaxStages = 8;               // ring slots, 4 SFA + 4 SFB columns each
static_assert(kSfCol0 + 8 * kMaxStages <= kTmemCols, "scale factors exceed the TMEM allocation");

// Transaction bytes of one 128 x 128 E2M1 box loaded as 16U4_ALIGN16B.
constexpr uint32_t kATxBytes = kBM * kBK / 2;
constexpr int kASmem = kBM * kBK;          // unpacked: 16 bytes per 16 elements + 8-byte gaps
constexpr int kBSmem = kN * kBK;           // 32 rows x 128 bytes
constexpr int kAtom = 512;
constexpr int kStageBytes = kASmem + kBSmem + 2 * kAtom;  // A, B, SFB atom, SFA atom
constexpr int kImage = kBSmem + kAtom;     // a token tile image: 32 part rows + their scale atom
constexpr int kRawBytes = kBM * 16;        // 128 rows x 16 E8M0 bytes (four stages)

struct BsShared {
  uint64_t full[16];
  uint64_t empty[16];
  uint64_t raw_full[kRawSlots];
  uint64_t raw_empty[kRawSlots];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t xch_full[2];   // gate/up: the up warps wrote xch[b]
  uint64_t xch_empty[2];  // the gate warps read it
  uint64_t mma_done;      // every MMA of this CTA has completed (before TMEM is freed)
  uint32_t tmem_base;
  int abort;
  float xch[2][64][kTokTile];  // gate/up: the up rows' sums for the gate warps
};

int bs_stages(int) { return kMaxStages; }

size_t bs_smem_bytes(int stages) {
  return size_t(stages) * kStageBytes + size_t(kRawSlots) * kRawBytes + sizeof(BsShared) + 1024;
}

// kind::mxf8f6f4 instruction descriptor: A E2M1, B E4M3, both K-major,
// UE8M0 scales, M = 128, N = kN, scale-factor ids kk for A and B.
__device__ __forceinline__ uint32_t bs_idesc(uint32_t kk) {
  return (kk << 4) | (5u << 7) | (0u << 10) | (uint32_t(kN >> 3) << 17) | (1u << 23) | (uint32_t(kBM >> 4) << 24) |
         (kk << 29);
}

// One 32-value block of a token row -> its hi / lo E4M3 parts and UE8M0
// bytes, stored into the tile image of sorted row r (tile j = r / 16, row n =
// r % 16, stage s = g / 4, block kk = g % 4 of the stage).
__device__ __forceinline__ void store_block(uint8_t* __restrict__ img, int S, int r, int g, const uint32_t* hi,
                                            const uint32_t* lo, uint32_t bh, uint32_t bl) {
  const int j = r / kTokTile, n = r % kTokTile;
  const int s = g / 4, kk = g % 4;
  uint8_t* base = img + (int64_t(j) * S + s) * kImage;
  *reinterpret_cast<uint4*>(base + image_off(n, 2 * kk)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  *reinterpret_cast<uint4*>(base + image_off(n, 2 * kk + 1)) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
  *reinterpret_cast<uint4*>(base + image_off(kTokTile + n, 2 * kk)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  *reinterpret_cast<uint4*>(base + image_off(kTokTile + n, 2 * kk + 1)) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
  uint8_t* sa = base + kBSmem;
  sa[n * 16 + kk] = uint8_t(bh);
  sa[(kTokTile + n) * 16 + kk] = uint8_t(bl);
}

// Block g (32 values) of bf16 row `src` -> hi / lo parts.
__device__ __forceinline__ void split_row_block(const uint16_t* __restrict__ src, int g, uint32_t* hi, uint32_t* lo,
                                                uint32_t* bh, uint32_t* bl) {
  float v[32];
  const uint4* s4 = reinterpret_cast<const uint4*>(src + g * 32);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 u = s4[q];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16x2(w[i]);
      v[8 * q + 2 * i] = f.x;
      v[8 * q + 2 * i + 1] = f.y;
    }
  }
  split_block(v, hi, lo, bh, bl);
}

}  // namespace

// x rows (sorted by the plan, 16-row tiles) -> tile images: for tile j and
// stage s, 4608 bytes = hi rows 0..15 then lo rows 16..31 of K [128 s, 128 s +
// 128) in the swizzled layout, then a 512-byte scale atom (row n: bytes 0..3 =
// the four 32-K blocks' UE8M0 of part row n), so one copy brings both.  One warp per row, one 32-K
// block per lane step; padding rows are skipped (their MMA columns are never
// read).
__global__ void __launch_bounds__(256) bs_quant_rows_kernel(const uint16_t* __restrict__ x, Plan p, int E, int K,
                                                            uint8_t* __restrict__ img) {
  const int rows = p.offsets[E + 1];
  const int lane = threadIdx.x & 31;
  const int S = K / kBK;
  for (int r = blockIdx.x * 8 + (threadIdx.x >> 5); r < rows; r += gridDim.x * 8) {
    const int t = p.row_token[r];
    if (t < 0) continue;
    const uint16_t* src = x + int64_t(t) * K;
    for (int g = lane; g < K / 32; g += 32) {
      uint32_t hi[8], lo[8], bh, bl;
      split_row_block(src, g, hi, lo, &bh, &bl);
      store_block(img, S, r, g, hi, lo, bh, bl);
    }
  }
}

// Calls of up to 64 tokens in one launch of T blocks.  Every block forms the
// plan of the sorted rows (groups padded to 16 rows) in shared memory -- for
// router calls of up to kSmallCallTokens tokens (EPL > 0) after selecting the
// top-k of every token itself (a group of four warps per token, the short-call
// top-k kernel's own code), else
// from the given routes -- which is short, so repeating it in every block
// costs no time; then block t quantises token t: each 32-value block of the
// row is split into hi / lo parts once and stored to every sorted row that
// holds the token (its K pairs and the shared expert's row).  Block 0 also
// writes the routes and the plan arrays.  The routes, plan and images are the
// bytes the top-k, plan and quantise kernels write one after another.
template <int EPL>
__global__ void __launch_bounds__(kSmallCallThreads) bs_route_plan_quant_kernel(
    const float* __restrict__ logits, const int32_t* __restrict__ routes, int T, int E, const TopkArgs tk,
    int has_shared, Plan p, int max_rows, int max_mtiles, uint32_t* status, const uint16_t* __restrict__ x, int H,
    uint8_t* __restrict__ img) {
  using SP = typename std::conditional<(EPL > 0), SmallPlan<8, kSmallCallTokens * 32>,
                                       SmallPlan<kMaxSmallTokens, kMaxSmallPairs>>::type;
  __shared__ SP sp;
  const int warp = threadIdx.x >> 5;
  const bool lead = blockIdx.x == 0;
  if constexpr (EPL > 0) {
    // token t: warps 4t .. 4t + 3 select from a quarter of the experts each,
    // then warp 4t from their candidates
    __shared__ float sw[kSmallCallTokens * 32];
    __shared__ TopkCands cands[kSmallCallTokens];
    const int tt = warp / kTopkGroupWarps, g = warp % kTopkGroupWarps;
    if (tt < T) topk_group_local<EPL>(logits + int64_t(tt) * E, tk, E, g, threadIdx.x & 31, cands[tt]);
    __syncthreads();
    if (tt < T && g == 0) {
      TopkArgs st = tk;
      st.idx = sp.ids;
      st.w = sw;
      topk_group_merge(cands[tt], st, tt, threadIdx.x & 31, lead ? tk.idx : nullptr, lead ? tk.w : nullptr);
    }
  } else {
    for (int i = threadIdx.x; i < T * tk.K; i += blockDim.x) sp.ids[i] = routes[i];
  }
  __syncthreads();
  small_plan_block(sp, T, tk.K, E, has_shared, kTokTile, p, max_rows, max_mtiles, status, lead);
  __syncthreads();
  if (sp.total > max_rows) return;  // reported by block 0
  const int t = blockIdx.x, K = tk.K, blocks = H / 32, S = H / kBK;
  const int nrows = K + (has_shared ? 1 : 0);
  const int split = max(1, min(nrows, int(blockDim.x) / blocks));  // threads sharing one value block's rows
  const uint16_t* src = x + int64_t(t) * H;
  for (int q = threadIdx.x; q < blocks * split; q += blockDim.x) {
    const int g = q % blocks, part = q / blocks;
    uint32_t hi[8], lo[8], bh, bl;
    split_row_block(src, g, hi, lo, &bh, &bl);
    for (int k = part; k < nrows; k += split) {
      const int r = k < K ? sp.pos[t * K + k] : sp.shared_row0 + t;
      if (r >= 0) store_block(img, S, r, g, hi, lo, bh, bl);
    }
  }
}

// ------------------------------------------------------------------ the expert kernel

// KIND 0: gate/up + SwiGLU -> act tile images (hi / lo E4M3 + scale atoms) for
// KIND 1; KIND 1: down -> routed [rows, H] bf16.
template <int KIND>
__global__ void __launch_bounds__(kThreads, 1) bs_decode_kernel(const __grid_constant__ CUtensorMap tm_w,
                                                                const __grid_constant__ CUtensorMap tm_ws,
                                                                const __grid_constant__ CUtensorMap tm_s,
                                                                const __grid_constant__ CUtensorMap tm_ss,
                                                                const BsArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const int K = KIND == 0 ? a.H : a.I;
  const int S = K / kBK;  // stages per item
  const int nb = KIND == 0 ? a.I / 64 : a.H / kBM;
  const int NS = a.stages;
  const int n_items = *a.plan.n_mtiles * nb;
  const uint32_t raw0 = smem_u32(smem_raw);
  const uint32_t base = (raw0 + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw0);
  BsShared& sh = *reinterpret_cast<BsShared*>(gbase + NS * kStageBytes + kRawSlots * kRawBytes);
  const uint32_t raw_base = base + NS * kStageBytes;
  auto a_addr = [&](int slot) { return base + slot * kStageBytes; };
  auto b_addr = [&](int slot) { return base + slot * kStageBytes + kASmem; };
  auto sfb_addr = [&](int slot) { return base + slot * kStageBytes + kASmem + kBSmem; };
  auto sfa_addr = [&](int slot) { return base + slot * kStageBytes + kASmem + kBSmem + kAtom; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&sh.full[i], 2);  // the TMA producer (with bytes) and the scale warp
      mbar_init(&sh.empty[i], 1);
    }
    for (int i = 0; i < kRawSlots; ++i) {
      mbar_init(&sh.raw_full[i], 1);
      mbar_init(&sh.raw_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh.tmem_full[i], 1);
      mbar_init(&sh.tmem_empty[i], 4);
      mbar_init(&sh.xch_full[i], 2);
      mbar_init(&sh.xch_empty[i], 2);
    }
    mbar_init(&sh.mma_done, 1);
    sh.abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 2) {
    tmem_alloc(&sh.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  volatile int* abort = &sh.abort;
  auto fail = [&](uint32_t role) {
    if (atomicExch(&sh.abort, 1) == 0) report_status(a.status, kStatusWaitTimeout, role);
  };
  auto item = [&](int q, int* e, int* row0, int* blk) {
    const int tile = q / nb;
    *blk = q - tile * nb;
    *e = a.plan.mtiles[2 * tile];
    *row0 = a.plan.mtiles[2 * tile + 1];
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_w);
      tma_prefetch_desc(&tm_s);
      int st = 0, ph = 0, rs = 0, rph = 0;
      // item metadata is read two items ahead, so no TMA issue waits on a load
      int ce = 0, crow0 = 0, cblk = 0, ne = 0, nrow0 = 0, nblk = 0;
      if (int(blockIdx.x) < n_items) item(blockIdx.x, &ce, &crow0, &cblk);
      if (int(blockIdx.x + gridDim.x) < n_items) item(blockIdx.x + gridDim.x, &ne, &nrow0, &nblk);
      for (int q = blockIdx.x; q < n_items && !*abort; q += gridDim.x) {
        const int e = ce, row0 = crow0, blk = cblk;
        int n2e = 0, n2row0 = 0, n2blk = 0;
        if (q + 2 * int(gridDim.x) < n_items) item(q + 2 * gridDim.x, &n2e, &n2row0, &n2blk);
        const bool shared_e = e == a.wts.E;
        const void* mw = shared_e ? &tm_ws : &tm_w;
        const void* ms = shared_e ? &tm_ss : &tm_s;
        const int ez = shared_e ? 0 : e;
        const int tile = row0 / kTokTile;
        for (int s = 0; s < S; ++s) {
          if ((s & 3) == 0) {
            if (!mbar_wait(&sh.raw_empty[rs], rph ^ 1, abort)) { fail(70 + KIND); break; }
            const uint32_t dst = raw_base + rs * kRawBytes;
            mbar_arrive_expect_tx(&sh.raw_full[rs], kRawBytes);
            if (KIND == 0) {  // rows blk * 64 .. + 63 of both halves of w13 (one 4-D box)
              tma_load_4d(dst, ms, 16 * (s >> 2), blk * 64, 0, ez, &sh.raw_full[rs]);
            } else {
              tma_load_3d(dst, ms, 16 * (s >> 2), blk * kBM, ez, &sh.raw_full[rs]);
            }
            if (++rs == kRawSlots) { rs = 0; rph ^= 1; }
          }
          if (!mbar_wait(&sh.empty[st], ph ^ 1, abort)) { fail(72 + KIND); break; }
          mbar_arrive_expect_tx(&sh.full[st], kATxBytes + uint32_t(kImage));
          if (KIND == 0)
            tma_load_4d(a_addr(st), mw, s * kBK, blk * 64, 0, ez, &sh.full[st]);
          else
            tma_load_3d(a_addr(st), mw, s * kBK, blk * kBM, ez, &sh.full[st]);
          // the token tile image and its scale atom in one copy
          bulk_g2s(b_addr(st), a.img + (int64_t(tile) * S + s) * kImage, uint32_t(kImage), &sh.full[st]);
          if (++st == NS) { st = 0; ph ^= 1; }
        }
        ce = ne, crow0 = nrow0, cblk = nblk;
        ne = n2e, nrow0 = n2row0, nblk = n2blk;
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- scale warp
    int st = 0, ph = 0, rs = 0, rph = 0;
    for (int q = blockIdx.x; q < n_items; q += gridDim.x) {
      if (warp_aborted(abort)) break;
      bool ok = true;
      // four stages per raw slot: their atoms, then one proxy fence and four arrivals
      for (int s0 = 0; s0 < S && ok; s0 += 4) {
        if (!warp_wait(&sh.raw_full[rs], rph, abort)) { ok = false; break; }
        int st_g[4];
        for (int j = 0; j < 4; ++j) {
          if (!warp_wait(&sh.empty[st], ph ^ 1, abort)) { ok = false; break; }
          // row lane + 32 m1 of the tile, bytes of the stage's four 32-K blocks
          const uint32_t rb = raw_base + rs * kRawBytes + 4 * j;
          const uint32_t w0 = lds_b32(rb + (lane)*16), w1 = lds_b32(rb + (lane + 32) * 16),
                         w2 = lds_b32(rb + (lane + 64) * 16), w3 = lds_b32(rb + (lane + 96) * 16);
          sts_v4(sfa_addr(st) + lane * 16, w0, w1, w2, w3);
          st_g[j] = st;
          if (++st == NS) { st = 0; ph ^= 1; }
        }
        if (!ok) break;
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          for (int j = 0; j < 4; ++j) mbar_arrive(&sh.full[st_g[j]]);
          mbar_arrive(&sh.raw_empty[rs]);
        }
        if (++rs == kRawSlots) { rs = 0; rph ^= 1; }
      }
      if (!ok) {
        if (lane == 0) fail(74 + KIND);
        break;
      }
    }
  } else if (warp == 2) {
    // ---------------------------------------------------------------- MMA issuer
    int st = 0, ph = 0, li = 0;
    for (int q = blockIdx.x; q < n_items; q += gridDim.x, ++li) {
      if (warp_aborted(abort)) break;
      const int acc = li & 1;
      if (!warp_wait(&sh.tmem_empty[acc], ((li >> 1) & 1) ^ 1, abort)) {
        if (lane == 0) fail(76 + KIND);
        break;
      }
      tc_fence_after();
      const uint32_t d = tmem + acc * kAccCols;
      bool ok = true;
      for (int s = 0; s < S; ++s) {
        if (!warp_wait(&sh.full[st], ph, abort)) { ok = false; break; }
        tc_fence_after();
        // four SFA and four SFB columns per ring slot (the MMA's scale-factor
        // operands start on 4-column boundaries)
        const uint32_t sfa_t = tmem + kSfCol0 + st * 8, sfb_t = sfa_t + 4;
        sf_copy_elect(sfa_t, sf_desc(sfa_addr(st)));
        sf_copy_elect(sfb_t, sf_desc(sfb_addr(st)));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          bs_mma_elect(d, umma_desc_sw128(a_addr(st) + 32 * kk), umma_desc_sw128(b_addr(st) + 32 * kk),
                       bs_idesc(uint32_t(kk)), sfa_t | (uint32_t(kk) << 30), sfb_t | (uint32_t(kk) << 30),
                       (s > 0 || kk > 0) ? 1u : 0u);
        umma_commit_elect(&sh.empty[st]);
        __syncwarp();
        if (++st == NS) { st = 0; ph ^= 1; }
      }
      if (!ok) {
        if (lane == 0) fail(78 + KIND);
        break;
      }
      umma_commit_elect(&sh.tmem_full[acc]);
      __syncwarp();
    }
    // every MMA issued here has completed before TMEM is freed (bounded wait)
    umma_commit_elect(&sh.mma_done);
    __syncwarp();
    volatile int keep_waiting = 0;  // this wait ignores the abort flag (0.2 s bound)
    mbar_wait(&sh.mma_done, 0, &keep_waiting, 0, 200000000ull);
  } else if (warp >= kEpiWarp0) {
    // ---------------------------------------------------------------- epilogue
    const int quarter = warp - kEpiWarp0;  // TMEM lanes 32 quarter .. 32 quarter + 31
    int li = 0;
    // item metadata read ahead (the tile entry two items early, the expert's
    // row count one item early), off the path from one accumulator to the next
    int ce = 0, crow0 = 0, cblk = 0, cvalid = 0, ne = 0, nrow0 = 0, nblk = 0;
    if (int(blockIdx.x) < n_items) {
      item(blockIdx.x, &ce, &crow0, &cblk);
      cvalid = min(kTokTile, a.plan.counts[ce] - (crow0 - a.plan.offsets[ce]));
    }
    if (int(blockIdx.x + gridDim.x) < n_items) item(blockIdx.x + gridDim.x, &ne, &nrow0, &nblk);
    for (int q = blockIdx.x; q < n_items; q += gridDim.x, ++li) {
      if (warp_aborted(abort)) break;
      const int e = ce, row0 = crow0, blk = cblk, valid = cvalid;
      int n2e = 0, n2row0 = 0, n2blk = 0, ncount = 0, noff = 0;
      if (q + 2 * int(gridDim.x) < n_items) item(q + 2 * gridDim.x, &n2e, &n2row0, &n2blk);
      if (q + int(gridDim.x) < n_items) {
        ncount = a.plan.counts[ne];
        noff = a.plan.offsets[ne];
      }
      (void)e;
      const int acc = li & 1;
      if (!warp_wait(&sh.tmem_full[acc], (li >> 1) & 1, abort)) {
        if (lane == 0) fail(80 + KIND);
        break;
      }
      tc_fence_after();
      uint32_t r[32];
      tmem_ld_32cols(tmem + acc * kAccCols + (uint32_t(quarter * 32) << 16), r);
      tmem_ld_wait();
      float y[kTokTile];
#pragma unroll
      for (int n = 0; n < kTokTile; ++n) y[n] = __uint_as_float(r[n]) + __uint_as_float(r[kTokTile + n]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.tmem_empty[acc]);
      if (KIND == 1) {
        const int h = blk * kBM + quarter * 32 + lane;
        if (a.ret.rows[0] != nullptr) {  // expert-parallel owner: straight into the senders' back blocks
          for (int n = 0; n < valid; ++n) {
            const int slot = a.plan.row_token[row0 + n];
            if (slot >= 0)
              a.ret.rows[slot / a.ret.capacity][int64_t(slot % a.ret.capacity) * a.H + h] = f32_to_bf16_bits(y[n]);
          }
        } else {
          for (int n = 0; n < valid; ++n) a.routed[int64_t(row0 + n) * a.H + h] = f32_to_bf16_bits(y[n]);
        }
      } else {
        // tile rows 0..63 are w13 rows blk * 64 .. of the first half (gate for
        // the Qwen layout, up for w13 = [w3; w1]), rows 64..127 the same rows of
        // the second half: the up rows' sums go to the gate warps
        const int xb = li & 1;
        const uint32_t xph = (li >> 1) & 1;
        const bool up_warp = a.gate_first ? quarter >= 2 : quarter < 2;
        const int pair = quarter & 1;  // features blk * 64 + 32 pair .. + 31
        if (up_warp) {
          if (!warp_wait(&sh.xch_empty[xb], xph ^ 1, abort)) {
            if (lane == 0) fail(82);
            break;
          }
#pragma unroll
          for (int n = 0; n < kTokTile; ++n) sh.xch[xb][pair * 32 + lane][n] = y[n];
          __syncwarp();
          if (lane == 0) mbar_arrive(&sh.xch_full[xb]);
        } else {
          if (!warp_wait(&sh.xch_full[xb], xph, abort)) {
            if (lane == 0) fail(83);
            break;
          }
          const int f = blk * 64 + pair * 32 + lane;  // feature (act column)
          const int Sd = a.I / kBK, sd = f / kBK, kk = (f % kBK) / 32;
          const int tile = row0 / kTokTile;
          uint8_t* img = a.act_img + (int64_t(tile) * Sd + sd) * kImage;
          uint8_t* sfb = img + kBSmem;
          const int c = (f % kBK) / 16, byte = f % 16;
          for (int n = 0; n < valid; ++n) {
            const float gv = bf16_round(y[n]), uv = bf16_round(sh.xch[xb][pair * 32 + lane][n]);
            const float act = bf16_round(swiglu_f32(gv, uv, a.limit));
            // hi / lo parts of this token's 32 features (one scale block per warp)
            float amax = fabsf(act);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const uint32_t bh = e4m3_block_scale(amax);
            const uint32_t hb = to_e4m3x2(act * __uint_as_float((254u - bh) << 23), 0.0f) & 0xFFu;
            float hv[4];
            e4m3x4_to_f32(hb, hv);
            const float res = act - hv[0] * __uint_as_float(bh << 23);
            float rmax = fabsf(res);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, o));
            const uint32_t bl = e4m3_block_scale(rmax);
            const uint32_t lb = to_e4m3x2(res * __uint_as_float((254u - bl) << 23), 0.0f) & 0xFFu;
            img[image_off(n, c) + byte] = uint8_t(hb);
            img[image_off(kTokTile + n, c) + byte] = uint8_t(lb);
            if (lane == 0) {
              sfb[n * 16 + kk] = uint8_t(bh);
              sfb[(kTokTile + n) * 16 + kk] = uint8_t(bl);
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&sh.xch_empty[xb]);  // xch[xb] is free again
        }
      }
      ce = ne, crow0 = nrow0, cblk = nblk;
      cvalid = min(kTokTile, ncount - (nrow0 - noff));
      ne = n2e, nrow0 = n2row0, nblk = n2blk;
    }
    // rows stored into other GPUs' memory: one system-scope fence per thread,
    // after its last store (a fence per item would wait out NVLink each time)
    if (KIND == 1 && a.ret.rows[0] != nullptr) __threadfence_system();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ gate/up and down in one launch

__device__ __forceinline__ uint32_t ld_acquire_gpu_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_gpu_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Orders generic-proxy global accesses and async-proxy (bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Both expert kernels of the block-scaled decode path in one persistent
// launch: items [0, n0) are the gate/up items of bs_decode_kernel<0> (tile
// q / nb0, 64 features), items [n0, n0 + n1) the down items of
// bs_decode_kernel<1> (tile, 128 output rows), each CTA taking items
// blockIdx.x, blockIdx.x + gridDim.x, ... in order, with the same stage ring,
// MMAs and epilogues.  A down item reads its tile's act images, which the
// gate warps of that tile's nb0 gate/up items write: each gate warp, after its
// bytes, fences them toward the async proxy and adds 1 to the tile's count
// (release); the down item's producer waits (acquire, bounded: 2 s, then the
// status word and unwinding) for 2 nb0 before the act-image copy.  The down
// weights stream while the last gate/up items finish, instead of after the
// first launch's tail.  No wait can close a cycle: every CTA's gate/up items
// precede its down items, and gate/up items wait for nothing.  The CTA that
// finishes last clears the counts for the next launch.
__global__ void __launch_bounds__(kThreads, 1) bs_decode_fused_kernel(
    const __grid_constant__ CUtensorMap gu_w, const __grid_constant__ CUtensorMap gu_ws,
    const __grid_constant__ CUtensorMap gu_s, const __grid_constant__ CUtensorMap gu_ss,
    const __grid_constant__ CUtensorMap dn_w, const __grid_constant__ CUtensorMap dn_ws,
    const __grid_constant__ CUtensorMap dn_s, const __grid_constant__ CUtensorMap dn_ss, const BsArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const int S0 = a.H / kBK, S1 = a.I / kBK;  // stages of a gate/up and of a down item
  const int nb0 = a.I / 64, nb1 = a.H / kBM;
  const int NS = a.stages;
  const int n_tiles = *a.plan.n_mtiles;
  const int n0 = n_tiles * nb0, n_items = n0 + n_tiles * nb1;
  const uint32_t done_target = 2u * uint32_t(nb0);  // two gate warps per gate/up item
  const uint32_t raw0 = smem_u32(smem_raw);
  const uint32_t base = (raw0 + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw0);
  BsShared& sh = *reinterpret_cast<BsShared*>(gbase + NS * kStageBytes + kRawSlots * kRawBytes);
  const uint32_t raw_base = base + NS * kStageBytes;
  auto a_addr = [&](int slot) { return base + slot * kStageBytes; };
  auto b_addr = [&](int slot) { return base + slot * kStageBytes + kASmem; };
  auto sfb_addr = [&](int slot) { return base + slot * kStageBytes + kASmem + kBSmem; };
  auto sfa_addr = [&](int slot) { return base + slot * kStageBytes + kASmem + kBSmem + kAtom; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&sh.full[i], 2);  // the TMA producer (with bytes) and the scale warp
      mbar_init(&sh.empty[i], 1);
    }
    for (int i = 0; i < kRawSlots; ++i) {
      mbar_init(&sh.raw_full[i], 1);
      mbar_init(&sh.raw_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh.tmem_full[i], 1);
      mbar_init(&sh.tmem_empty[i], 4);
      mbar_init(&sh.xch_full[i], 2);
      mbar_init(&sh.xch_empty[i], 2);
    }
    mbar_init(&sh.mma_done, 1);
    sh.abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 2) {
    tmem_alloc(&sh.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  volatile int* abort = &sh.abort;
  auto fail = [&](uint32_t role) {
    if (atomicExch(&sh.abort, 1) == 0) report_status(a.status, kStatusWaitTimeout, role);
  };
  // item q: kind (0 gate/up, 1 down), expert, first row, block
  auto item = [&](int q, int* kind, int* e, int* row0, int* blk) {
    const int down = q >= n0 ? 1 : 0;
    const int r = q - down * n0, nb = down ? nb1 : nb0;
    const int tile = r / nb;
    *kind = down;
    *blk = r - tile * nb;
    *e = a.plan.mtiles[2 * tile];
    *row0 = a.plan.mtiles[2 * tile + 1];
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&gu_w);
      tma_prefetch_desc(&gu_s);
      tma_prefetch_desc(&dn_w);
      tma_prefetch_desc(&dn_s);
      int st = 0, ph = 0, rs = 0, rph = 0;
      int ck = 0, ce = 0, crow0 = 0, cblk = 0, nk = 0, ne = 0, nrow0 = 0, nblk = 0;
      if (int(blockIdx.x) < n_items) item(blockIdx.x, &ck, &ce, &crow0, &cblk);
      if (int(blockIdx.x + gridDim.x) < n_items) item(blockIdx.x + gridDim.x, &nk, &ne, &nrow0, &nblk);
      for (int q = blockIdx.x; q < n_items && !*abort; q += gridDim.x) {
        const int kind = ck, e = ce, row0 = crow0, blk = cblk;
        int n2k = 0, n2e = 0, n2row0 = 0, n2blk = 0;
        if (q + 2 * int(gridDim.x) < n_items) item(q + 2 * gridDim.x, &n2k, &n2e, &n2row0, &n2blk);
        const bool shared_e = e == a.wts.E;
        const void* mw = kind ? (shared_e ? &dn_ws : &dn_w) : (shared_e ? &gu_ws : &gu_w);
        const void* ms = kind ? (shared_e ? &dn_ss : &dn_s) : (shared_e ? &gu_ss : &gu_s);
        const int ez = shared_e ? 0 : e;
        const int tile = row0 / kTokTile;
        const int S = kind ? S1 : S0;
        const uint8_t* img = kind ? a.act_img : a.img;
        bool ok = true;
        for (int s = 0; s < S; ++s) {
          if ((s & 3) == 0) {
            if (!mbar_wait(&sh.raw_empty[rs], rph ^ 1, abort)) { fail(90); ok = false; break; }
            const uint32_t dst = raw_base + rs * kRawBytes;
            mbar_arrive_expect_tx(&sh.raw_full[rs], kRawBytes);
            if (kind == 0)  // rows blk * 64 .. + 63 of both halves of w13 (one 4-D box)
              tma_load_4d(dst, ms, 16 * (s >> 2), blk * 64, 0, ez, &sh.raw_full[rs]);
            else
              tma_load_3d(dst, ms, 16 * (s >> 2), blk * kBM, ez, &sh.raw_full[rs]);
            if (++rs == kRawSlots) { rs = 0; rph ^= 1; }
          }
          if (!mbar_wait(&sh.empty[st], ph ^ 1, abort)) { fail(91); ok = false; break; }
          mbar_arrive_expect_tx(&sh.full[st], kATxBytes + uint32_t(kImage));
          if (kind == 0)
            tma_load_4d(a_addr(st), mw, s * kBK, blk * 64, 0, ez, &sh.full[st]);
          else
            tma_load_3d(a_addr(st), mw, s * kBK, blk * kBM, ez, &sh.full[st]);
          if (kind == 1 && s == 0) {
            // the tile's act images: every gate warp of its gate/up items has written them
            const uint64_t t0 = global_timer_ns();
            for (uint32_t spin = 0; ld_acquire_gpu_u32(a.tile_done + tile) < done_target; ++spin) {
              if ((spin & 15u) == 15u && (*abort || global_timer_ns() - t0 > 2000000000ull)) {
                ok = false;
                break;
              }
              __nanosleep(64);
            }
            fence_proxy_async_global();
            if (!ok) {
              fail(92);
              // complete the stage's transaction so no wait on it is left pending
              bulk_g2s(b_addr(st), img + (int64_t(tile) * S + s) * kImage, uint32_t(kImage), &sh.full[st]);
              break;
            }
          }
          // the token (or act) tile image and its scale atom in one copy
          bulk_g2s(b_addr(st), img + (int64_t(tile) * S + s) * kImage, uint32_t(kImage), &sh.full[st]);
          if (++st == NS) { st = 0; ph ^= 1; }
        }
        if (!ok) break;
        ck = nk, ce = ne, crow0 = nrow0, cblk = nblk;
        nk = n2k, ne = n2e, nrow0 = n2row0, nblk = n2blk;
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- scale warp
    int st = 0, ph = 0, rs = 0, rph = 0;
    for (int q = blockIdx.x; q < n_items; q += gridDim.x) {
      if (warp_aborted(abort)) break;
      const int S = q >= n0 ? S1 : S0;
      bool ok = true;
      for (int s0 = 0; s0 < S && ok; s0 += 4) {
        if (!warp_wait(&sh.raw_full[rs], rph, abort)) { ok = false; break; }
        int st_g[4];
        for (int j = 0; j < 4; ++j) {
          if (!warp_wait(&sh.empty[st], ph ^ 1, abort)) { ok = false; break; }
          const uint32_t rb = raw_base + rs * kRawBytes + 4 * j;
          const uint32_t w0 = lds_b32(rb + (lane)*16), w1 = lds_b32(rb + (lane + 32) * 16),
                         w2 = lds_b32(rb + (lane + 64) * 16), w3 = lds_b32(rb + (lane + 96) * 16);
          sts_v4(sfa_addr(st) + lane * 16, w0, w1, w2, w3);
          st_g[j] = st;
          if (++st == NS) { st = 0; ph ^= 1; }
        }
        if (!ok) break;
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          for (int j = 0; j < 4; ++j) mbar_arrive(&sh.full[st_g[j]]);
          mbar_arrive(&sh.raw_empty[rs]);
        }
        if (++rs == kRawSlots) { rs = 0; rph ^= 1; }
      }
      if (!ok) {
        if (lane == 0) fail(93);
        break;
      }
    }
  } else if (warp == 2) {
    // ---------------------------------------------------------------- MMA issuer
    int st = 0, ph = 0, li = 0;
    for (int q = blockIdx.x; q < n_items; q += gridDim.x, ++li) {
      if (warp_aborted(abort)) break;
      const int S = q >= n0 ? S1 : S0;
      const int acc = li & 1;
      if (!warp_wait(&sh.tmem_empty[acc], ((li >> 1) & 1) ^ 1, abort)) {
        if (lane == 0) fail(94);
        break;
      }
      tc_fence_after();
      const uint32_t d = tmem + acc * kAccCols;
      bool ok = true;
      for (int s = 0; s < S; ++s) {
        if (!warp_wait(&sh.full[st], ph, abort)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sfa_t = tmem + kSfCol0 + st * 8, sfb_t = sfa_t + 4;
        sf_copy_elect(sfa_t, sf_desc(sfa_addr(st)));
        sf_copy_elect(sfb_t, sf_desc(sfb_addr(st)));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          bs_mma_elect(d, umma_desc_sw128(a_addr(st) + 32 * kk), umma_desc_sw128(b_addr(st) + 32 * kk),
                       bs_idesc(uint32_t(kk)), sfa_t | (uint32_t(kk) << 30), sfb_t | (uint32_t(kk) << 30),
                       (s > 0 || kk > 0) ? 1u : 0u);
        umma_commit_elect(&sh.empty[st]);
        __syncwarp();
        if (++st == NS) { st = 0; ph ^= 1; }
      }
      if (!ok) {
        if (lane == 0) fail(95);
        break;
      }
      umma_commit_elect(&sh.tmem_full[acc]);
      __syncwarp();
    }
    umma_commit_elect(&sh.mma_done);
    __syncwarp();
    volatile int keep_waiting = 0;  // this wait ignores the abort flag (0.2 s bound)
    mbar_wait(&sh.mma_done, 0, &keep_waiting, 0, 200000000ull);
  } else if (warp >= kEpiWarp0) {
    // ---------------------------------------------------------------- epilogue
    const int quarter = warp - kEpiWarp0;
    int li = 0;
    int ck = 0, ce = 0, crow0 = 0, cblk = 0, cvalid = 0, nk = 0, ne = 0, nrow0 = 0, nblk = 0;
    if (int(blockIdx.x) < n_items) {
      item(blockIdx.x, &ck, &ce, &crow0, &cblk);
      cvalid = min(kTokTile, a.plan.counts[ce] - (crow0 - a.plan.offsets[ce]));
    }
    if (int(blockIdx.x + gridDim.x) < n_items) item(blockIdx.x + gridDim.x, &nk, &ne, &nrow0, &nblk);
    for (int q = blockIdx.x; q < n_items; q += gridDim.x, ++li) {
      if (warp_aborted(abort)) break;
      const int kind = ck, row0 = crow0, blk = cblk, valid = cvalid;
      int n2k = 0, n2e = 0, n2row0 = 0, n2blk = 0, ncount = 0, noff = 0;
      if (q + 2 * int(gridDim.x) < n_items) item(q + 2 * gridDim.x, &n2k, &n2e, &n2row0, &n2blk);
      if (q + int(gridDim.x) < n_items) {
        ncount = a.plan.counts[ne];
        noff = a.plan.offsets[ne];
      }
      const int acc = li & 1;
      if (!warp_wait(&sh.tmem_full[acc], (li >> 1) & 1, abort)) {
        if (lane == 0) fail(96);
        break;
      }
      tc_fence_after();
      uint32_t r[32];
      tmem_ld_32cols(tmem + acc * kAccCols + (uint32_t(quarter * 32) << 16), r);
      tmem_ld_wait();
      float y[kTokTile];
#pragma unroll
      for (int n = 0; n < kTokTile; ++n) y[n] = __uint_as_float(r[n]) + __uint_as_float(r[kTokTile + n]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.tmem_empty[acc]);
      if (kind == 1) {
        const int h = blk * kBM + quarter * 32 + lane;
        if (a.ret.rows[0] != nullptr) {
          for (int n = 0; n < valid; ++n) {
            const int slot = a.plan.row_token[row0 + n];
            if (slot >= 0)
              a.ret.rows[slot / a.ret.capacity][int64_t(slot % a.ret.capacity) * a.H + h] = f32_to_bf16_bits(y[n]);
          }
        } else {
          for (int n = 0; n < valid; ++n) a.routed[int64_t(row0 + n) * a.H + h] = f32_to_bf16_bits(y[n]);
        }
      } else {
        const int xb = li & 1;
        const uint32_t xph = (li >> 1) & 1;
        const bool up_warp = a.gate_first ? quarter >= 2 : quarter < 2;
        const int pair = quarter & 1;
        if (up_warp) {
          if (!warp_wait(&sh.xch_empty[xb], xph ^ 1, abort)) {
            if (lane == 0) fail(97);
            break;
          }
#pragma unroll
          for (int n = 0; n < kTokTile; ++n) sh.xch[xb][pair * 32 + lane][n] = y[n];
          __syncwarp();
          if (lane == 0) mbar_arrive(&sh.xch_full[xb]);
        } else {
          if (!warp_wait(&sh.xch_full[xb], xph, abort)) {
            if (lane == 0) fail(98);
            break;
          }
          const int f = blk * 64 + pair * 32 + lane;
          const int sd = f / kBK, kk = (f % kBK) / 32;
          const int tile = row0 / kTokTile;
          uint8_t* img = a.act_img + (int64_t(tile) * S1 + sd) * kImage;
          uint8_t* sfb = img + kBSmem;
          const int c = (f % kBK) / 16, byte = f % 16;
          for (int n = 0; n < valid; ++n) {
            const float gv = bf16_round(y[n]), uv = bf16_round(sh.xch[xb][pair * 32 + lane][n]);
            const float act = bf16_round(swiglu_f32(gv, uv, a.limit));
            float amax = fabsf(act);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const uint32_t bh = e4m3_block_scale(amax);
            const uint32_t hb = to_e4m3x2(act * __uint_as_float((254u - bh) << 23), 0.0f) & 0xFFu;
            float hv[4];
            e4m3x4_to_f32(hb, hv);
            const float res = act - hv[0] * __uint_as_float(bh << 23);
            float rmax = fabsf(res);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, o));
            const uint32_t bl = e4m3_block_scale(rmax);
            const uint32_t lb = to_e4m3x2(res * __uint_as_float((254u - bl) << 23), 0.0f) & 0xFFu;
            img[image_off(n, c) + byte] = uint8_t(hb);
            img[image_off(kTokTile + n, c) + byte] = uint8_t(lb);
            if (lane == 0) {
              sfb[n * 16 + kk] = uint8_t(bh);
              sfb[(kTokTile + n) * 16 + kk] = uint8_t(bl);
            }
          }
          // this warp's act bytes, then its count for the tile's down items
          fence_proxy_async_global();
          __threadfence();
          __syncwarp();
          if (lane == 0) {
            red_release_gpu_add(a.tile_done + tile, 1u);
            mbar_arrive(&sh.xch_empty[xb]);
          }
        }
      }
      ck = nk, ce = ne, crow0 = nrow0, cblk = nblk;
      cvalid = min(kTokTile, ncount - (nrow0 - noff));
      nk = n2k, ne = n2e, nrow0 = n2row0, nblk = n2blk;
    }
    if (a.ret.rows[0] != nullptr) __threadfence_system();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  // the last CTA to finish clears the tile counts for the next launch
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(a.tile_done + a.max_tiles, 1u) == gridDim.x - 1) {
      for (int t = 0; t < n_tiles; ++t) a.tile_done[t] = 0u;
      a.tile_done[a.max_tiles] = 0u;
      __threadfence();
    }
  }
}

void bs_init_attributes() {
  const int bytes = int(bs_smem_bytes(bs_stages(0)));
  cudaFuncSetAttribute(bs_decode_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  cudaFuncSetAttribute(bs_decode_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  cudaFuncSetAttribute(bs_decode_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

bool bs_shape_ok(int H, int I) { return H % 512 == 0 && I % 512 == 0 && H >= 512 && I >= 512; }

void launch_bs_quant_rows(const uint16_t* x, const Plan& p, int E, int K, uint8_t* img, int num_sms,
                          cudaStream_t stream) {
  bs_quant_rows_kernel<<<num_sms * 4, 256, 0, stream>>>(x, p, E, K, img);
}

bool bs_plan_quant_ok(int T, int K, int E) {
  return T >= 1 && T <= kMaxSmallTokens && K >= 1 && T * K <= kMaxSmallPairs && E <= kMaxSmallExperts;
}

bool bs_route_plan_quant_ok(int T, int K, int E, int kind) {
  static_assert(kSmallCallTokens * kTopkGroupWarps * 32 <= kSmallCallThreads, "a warp group per token");
  return bs_plan_quant_ok(T, K, E) && T <= kSmallCallTokens && K <= kTopkGroupMaxK && E <= kTopkGroupWarps * 128 &&
         kind != WM_ROUTER_SIGMOID_GROUPED;
}

void launch_bs_route_plan_quant(const float* logits, int T, int E, const TopkArgs& tk, bool has_shared, const Plan& p,
                                int max_rows, int max_mtiles, uint32_t* status, const uint16_t* x, int H,
                                uint8_t* img, cudaStream_t stream) {
  if (E <= kTopkGroupWarps * 64)
    bs_route_plan_quant_kernel<2><<<T, kSmallCallThreads, 0, stream>>>(
        logits, nullptr, T, E, tk, has_shared ? 1 : 0, p, max_rows, max_mtiles, status, x, H, img);
  else
    bs_route_plan_quant_kernel<4><<<T, kSmallCallThreads, 0, stream>>>(
        logits, nullptr, T, E, tk, has_shared ? 1 : 0, p, max_rows, max_mtiles, status, x, H, img);
}

void launch_bs_plan_quant(const int32_t* routes, int T, int K, int E, bool has_shared, const Plan& p, int max_rows,
                          int max_mtiles, uint32_t* status, const uint16_t* x, int H, uint8_t* img,
                          cudaStream_t stream) {
  TopkArgs tk{};
  tk.K = K;
  bs_route_plan_quant_kernel<0><<<T, kSmallCallThreads, 0, stream>>>(
      nullptr, routes, T, E, tk, has_shared ? 1 : 0, p, max_rows, max_mtiles, status, x, H, img);
}

void launch_bs_decode_fused(const BsArgs& args, const void* const* maps, int num_sms, cudaStream_t stream) {
  BsArgs a = args;
  a.stages = bs_stages(a.H);
  const size_t smem = bs_smem_bytes(a.stages);
  const CUtensorMap* m[8];
  for (int i = 0; i < 8; ++i) m[i] = static_cast<const CUtensorMap*>(maps[i]);
  bs_decode_fused_kernel<<<num_sms, kThreads, smem, stream>>>(*m[0], *m[1], *m[2], *m[3], *m[4], *m[5], *m[6], *m[7],
                                                               a);
}

void launch_bs_decode(const BsArgs& args, int kind, const void* const* maps, int num_sms, cudaStream_t stream) {
  BsArgs a = args;
  a.stages = bs_stages(kind == 0 ? a.H : a.I);
  const size_t smem = bs_smem_bytes(a.stages);
  const CUtensorMap* m = static_cast<const CUtensorMap*>(maps[0]);
  const CUtensorMap* ms = static_cast<const CUtensorMap*>(maps[1]);
  const CUtensorMap* s = static_cast<const CUtensorMap*>(maps[2]);
  const CUtensorMap* ss = static_cast<const CUtensorMap*>(maps[3]);
  if (kind == 0)
    bs_decode_kernel<0><<<num_sms, kThreads, smem, stream>>>(*m, *ms, *s, *ss, a);
  else
    bs_decode_kernel<1><<<num_sms, kThreads, smem, stream>>>(*m, *ms, *s, *ss, a);
}

}  // namespace wm
