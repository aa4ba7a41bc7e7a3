// Prefill path on tcgen05 block-scaled MMA (kind::mxf8f6f4): a grouped GEMM
// over expert-sorted rows in which the MXFP4 expert weights go from the blob
// to the tensor cores by TMA as they are -- E2M1 elements, E8M0 group scales
// applied by the MMA as UE8M0 scale factors -- so no CUDA core touches a
// weight.
//
// Reference arithmetic: mx.gather_qmm(..., mode="mxfp4", group_size=32,
// sorted_indices=True) over expert-sorted rows (model.py:435-501,
// qwen4_exp.py:853-904) and the tiled Metal kernels expert_gemm_sg /
// tops_expert (QwenNative/kernels.metal:706-752, kernels_tensorops.metal:49-87):
// per expert Y = X_e W_e^T with exact dequantised weights and fp32
// accumulation; SwiGLU on the bf16 gate/up product (the reference's
// expert_act dispatch), bf16 rows out of the down product.
//
// Operands of one MMA (M = 128 token rows, N = 256 weight rows, K = 32):
//   A  token rows as two E4M3 parts, hi = e4m3(x / s_hi) and lo =
//      e4m3((x - hi * s_hi) / s_lo), power-of-two scales per row and 32 K
//      (the decode kernel's split: within 2^-8 of every element); the hi and
//      the lo MMA of a K step accumulate into the same TMEM columns, so the
//      tensor core adds the parts.
//   B  weights: E2M1 nibbles by TMA (16U4_ALIGN16B: 16 bytes of shared memory
//      per 16 elements, the layout kind::mxf8f6f4 reads), K-major, 128-byte
//      swizzle; gate/up tiles are two 4-D boxes of 64 gate + the 64 matching
//      up rows, so SwiGLU runs in the epilogue.
//   D  fp32, TMEM lanes = token rows, 256 columns.
//
// Token rows reach shared memory two ways.  Gate/up: bsg_quant_scatter
// quantises each x row once and writes its parts to every sorted row that
// holds it (hi, lo [rows][H] E4M3, shi, slo [rows][H / 32] UE8M0, plan
// order), and the producer loads a stage's 128 x 128-byte hi and lo tiles by
// TMA (128-byte swizzle) and, every fourth stage, the rows' scale bytes for
// the scale warp, which builds the A scale atoms beside the weight atoms.
// Down: the gate/up epilogue writes act tile images -- for the plan's
// 128-row tile j and 128-K stage s one 33,792-byte block at (j * S + s) *
// 33,792: hi rows (16 KB) and lo rows (16 KB) in the swizzled layout, then
// the hi and the lo scale atoms -- and one bulk copy brings a stage's A
// operands and scale factors.  (Measured and dropped: gathering the x rows
// inside the GEMM with TMA tile::gather4, 64 requests of 4 rows per stage,
// 3x slower; quantising per row and copying into images, 250 us against
// ~150 for the scatter at config 2.)
//
// One persistent CTA per SM walks the (128-row tile, 256-row weight tile)
// work list; 12 warps:
//   warp 0      TMA producer: per stage the token rows (two tiles, or the
//               act image) and two weight boxes; every fourth stage the raw
//               scale rows of the next four stages
//   warp 1      scale warp: raw scale rows -> the stage's scale atoms
//   warp 2      TMEM owner and MMA issuer (one elected lane, warp-wide)
//   warps 4-11  epilogue: lane quarter warp % 4, column half (warp - 4) / 4;
//               each thread loads its 128 columns into registers and frees
//               the accumulator before the SwiGLU / quantisation / stores
// Three 66 KB stages; one 256-column accumulator (the other TMEM columns hold
// the scale factors).  Every mbarrier wait is bounded (2 s); on a timeout the
// kernel records the status, the other roles unwind and TMEM is freed.
#include "wm_bs_common.cuh"
#include "wm_kernels.h"

namespace wm {

namespace {

constexpr int kTM = 128;                       // token rows per tile (MMA M)
constexpr int kTN = 256;                       // weight rows per tile (MMA N)
constexpr int kBK = 128;                       // K per stage: four 32-K scale blocks
constexpr int kStages = 3;
constexpr int kThreads = 384;
constexpr int kEpiWarp0 = 4, kEpiWarps = 8;
constexpr int kPart = kTM * kBK;               // one part's 128 rows of 128 bytes
constexpr int kAtom = 512;
constexpr int kImg = 2 * kPart + 2 * kAtom;    // tile image: hi rows, lo rows, hi atom, lo atom
constexpr int kBBytes = kTN * kBK;             // 256 weight rows, unpacked
constexpr uint32_t kBTx = kTN * kBK / 2;       // their packed bytes (TMA transaction count)
constexpr int kStageBytes = kImg + kBBytes + 2 * kAtom;
constexpr int kRawSlots = 2;
constexpr int kRawW = kTN * 16;                // 256 weight rows x 16 E8M0 bytes (four stages)
constexpr int kRawX = 2 * kTM * 16;            // gate/up: 128 token rows x 16 bytes, hi then lo
constexpr int kRawBytes = kRawW + kRawX;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSfCol0 = kTN;              // scale factors after the accumulator
constexpr uint32_t kSfStage = 16;              // SFA hi 4, SFA lo 4, SFB 8 columns
static_assert(kSfCol0 + kSfStage * kStages <= kTmemCols, "scale factors exceed the TMEM allocation");
static_assert(kImg % 1024 == 0 && kStageBytes % 1024 == 0, "swizzled operands need 1024-byte alignment");
static_assert(kPart % 128 == 0 && kRawW % 128 == 0 && kRawX % 256 == 0 && kRawBytes % 128 == 0,
              "every TMA destination in shared memory must be 128-byte aligned");

struct GShared {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t raw_full[kRawSlots];
  uint64_t raw_empty[kRawSlots];
  uint64_t tmem_full;
  uint64_t tmem_empty;
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};

constexpr size_t kSmemBytes = size_t(kStages) * kStageBytes + size_t(kRawSlots) * kRawBytes + sizeof(GShared) + 1024;
static_assert(kSmemBytes <= 232448, "more shared memory than a B200 CTA may have");

// kind::mxf8f6f4 instruction descriptor: A E4M3, B E2M1, both K-major, UE8M0
// scales, M = 128, N = 256, scale-factor ids kk for A and B.
__device__ __forceinline__ uint32_t g_idesc(uint32_t kk) {
  return (kk << 4) | (0u << 7) | (5u << 10) | (uint32_t(kTN >> 3) << 17) | (1u << 23) | (uint32_t(kTM >> 4) << 24) |
         (kk << 29);
}

// Byte of (part row n, 32-K block kk of the stage) in a scale atom.
__device__ __forceinline__ int atom_off(int n, int kk) { return (n & 31) * 16 + (n >> 5) * 4 + kk; }

}  // namespace

// x rows -> their hi / lo E4M3 parts and UE8M0 scales, written to every
// sorted row that holds them: hi, lo [rows][K], shi, slo [rows][K / 32] in
// plan order.  Source row t goes to rows pair_pos[t * topk + k] (k < topk;
// none when < 0) and, with has_shared, offsets[E] + t.  With `counts` the
// source rows are expert-parallel slots (block r = t / capacity holds
// counts[r]) and the others are skipped.  One warp per source row; per pass
// each lane splits two 32-K blocks once and stores them to every destination
// (a warp writes 1 KB of a row per store, coalesced).
__global__ void __launch_bounds__(256) bsg_quant_scatter_kernel(const uint16_t* __restrict__ x, int rows, int K,
                                                                Plan p, int topk, int has_shared, int E,
                                                                const int32_t* __restrict__ counts, int capacity,
                                                                uint8_t* __restrict__ hi, uint8_t* __restrict__ lo,
                                                                uint8_t* __restrict__ shi, uint8_t* __restrict__ slo) {
  const int lane = threadIdx.x & 31;
  const int nblk = K / 32;
  for (int t = blockIdx.x * 8 + (threadIdx.x >> 5); t < rows; t += gridDim.x * 8) {
    if (counts != nullptr && t % capacity >= counts[t / capacity]) continue;
    // destination rows: lane j holds pair_pos[t * topk + j] and [.. + 32 + j]
    const int pp0 = lane < topk ? p.pair_pos[int64_t(t) * topk + lane] : -1;
    const int pp1 = lane + 32 < topk ? p.pair_pos[int64_t(t) * topk + 32 + lane] : -1;
    const int ndst = topk + (has_shared ? 1 : 0);
    const int shared_row = has_shared ? p.offsets[E] + t : -1;
    const uint16_t* src = x + int64_t(t) * K;
    for (int g0 = 0; g0 < nblk; g0 += 64) {
      uint32_t h[2][8], l[2][8], bh[2], bl[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int g = g0 + 32 * j + lane;
        if (g < nblk) {
          float v[32];
          const uint4* s4 = reinterpret_cast<const uint4*>(src + g * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 u = __ldg(s4 + q);
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float2 f = unpack_bf16x2(w[i]);
              v[8 * q + 2 * i] = f.x;
              v[8 * q + 2 * i + 1] = f.y;
            }
          }
          split_block(v, h[j], l[j], &bh[j], &bl[j]);
        }
      }
      for (int k = 0; k < ndst; ++k) {
        const int rk = __shfl_sync(0xffffffffu, k < 32 ? pp0 : pp1, k & 31);
        const int r = k < topk ? rk : shared_row;
        if (r < 0) continue;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int g = g0 + 32 * j + lane;
          if (g < nblk) {
            uint4* hd = reinterpret_cast<uint4*>(hi + int64_t(r) * K + g * 32);
            uint4* ld = reinterpret_cast<uint4*>(lo + int64_t(r) * K + g * 32);
            hd[0] = make_uint4(h[j][0], h[j][1], h[j][2], h[j][3]);
            hd[1] = make_uint4(h[j][4], h[j][5], h[j][6], h[j][7]);
            ld[0] = make_uint4(l[j][0], l[j][1], l[j][2], l[j][3]);
            ld[1] = make_uint4(l[j][4], l[j][5], l[j][6], l[j][7]);
            shi[int64_t(r) * nblk + g] = uint8_t(bh[j]);
            slo[int64_t(r) * nblk + g] = uint8_t(bl[j]);
          }
        }
      }
    }
  }
}

// KIND 0: gate/up + SwiGLU -> act tile images for KIND 1 (a.act_img);
// KIND 1: down -> routed [rows, H] bf16, or with a.ret.rows[0] set the
// senders' back blocks (expert-parallel owner).
template <int KIND>
__global__ void __launch_bounds__(kThreads, 1) bsg_kernel(const __grid_constant__ CUtensorMap tm_w,
                                                          const __grid_constant__ CUtensorMap tm_ws,
                                                          const __grid_constant__ CUtensorMap tm_s,
                                                          const __grid_constant__ CUtensorMap tm_ss,
                                                          const __grid_constant__ CUtensorMap tm_xh,
                                                          const __grid_constant__ CUtensorMap tm_xl,
                                                          const __grid_constant__ CUtensorMap tm_xsh,
                                                          const __grid_constant__ CUtensorMap tm_xsl,
                                                          const BsArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const int K = KIND == 0 ? a.H : a.I;
  const int S = K / kBK;                           // stages per item (a multiple of 4)
  const int n_nt = KIND == 0 ? a.I / (kTN / 2) : a.H / kTN;
  const int n_items = *a.plan.n_mtiles * n_nt;
  const uint32_t raw0 = smem_u32(smem_raw);
  const uint32_t base = (raw0 + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw0);
  GShared& sh = *reinterpret_cast<GShared*>(gbase + kStages * kStageBytes + kRawSlots * kRawBytes);
  const uint32_t raw_base = base + kStages * kStageBytes;
  auto img_addr = [&](int slot) { return base + slot * kStageBytes; };
  auto b_addr = [&](int slot) { return base + slot * kStageBytes + kImg; };
  auto sfb_addr = [&](int slot) { return base + slot * kStageBytes + kImg + kBBytes; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sh.full[i], 2);  // the TMA producer (with bytes) and the scale warp
      mbar_init(&sh.empty[i], 1);
    }
    for (int i = 0; i < kRawSlots; ++i) {
      mbar_init(&sh.raw_full[i], 1);
      mbar_init(&sh.raw_empty[i], 1);
    }
    mbar_init(&sh.tmem_full, 1);
    mbar_init(&sh.tmem_empty, kEpiWarps);
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

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_w);
      tma_prefetch_desc(&tm_s);
      if (KIND == 0) {
        tma_prefetch_desc(&tm_xh);
        tma_prefetch_desc(&tm_xsh);
      }
      int st = 0, ph = 0, rs = 0, rph = 0;
      for (int q = blockIdx.x; q < n_items && !*abort; q += gridDim.x) {
        const int tile = q / n_nt, nt = q - tile * n_nt;
        const int e = a.plan.mtiles[2 * tile], row0 = a.plan.mtiles[2 * tile + 1];
        const bool shared_e = e == a.wts.E;
        const void* mw = shared_e ? &tm_ws : &tm_w;
        const void* ms = shared_e ? &tm_ss : &tm_s;
        const int ez = shared_e ? 0 : e;
        const uint8_t* src = a.img + int64_t(tile) * S * kImg;  // down: image (tile, s) at (tile * S + s) * kImg
        for (int s = 0; s < S; ++s) {
          if ((s & 3) == 0) {
            if (!mbar_wait(&sh.raw_empty[rs], rph ^ 1, abort)) { fail(90 + KIND); break; }
            const uint32_t dst = raw_base + rs * kRawBytes;
            mbar_arrive_expect_tx(&sh.raw_full[rs], KIND == 0 ? uint32_t(kRawBytes) : uint32_t(kRawW));
            if (KIND == 0) {  // tile rows 0..127: E8M0 rows nt * 128 .. + 63 of both halves; 128..255: the next 64
              tma_load_4d(dst, ms, 16 * (s >> 2), nt * 128, 0, ez, &sh.raw_full[rs]);
              tma_load_4d(dst + kRawW / 2, ms, 16 * (s >> 2), nt * 128 + 64, 0, ez, &sh.raw_full[rs]);
              // the token rows' scale bytes, hi then lo
              tma_load_2d_s(dst + kRawW, &tm_xsh, 16 * (s >> 2), row0, &sh.raw_full[rs]);
              tma_load_2d_s(dst + kRawW + kRawX / 2, &tm_xsl, 16 * (s >> 2), row0, &sh.raw_full[rs]);
            } else {
              tma_load_3d(dst, ms, 16 * (s >> 2), nt * kTN, ez, &sh.raw_full[rs]);
              tma_load_3d(dst + kRawW / 2, ms, 16 * (s >> 2), nt * kTN + 128, ez, &sh.raw_full[rs]);
            }
            if (++rs == kRawSlots) { rs = 0; rph ^= 1; }
          }
          if (!mbar_wait(&sh.empty[st], ph ^ 1, abort)) { fail(92 + KIND); break; }
          mbar_arrive_expect_tx(&sh.full[st], (KIND == 0 ? uint32_t(2 * kPart) : uint32_t(kImg)) + kBTx);
          if (KIND == 0) {  // the tile's hi and lo rows of this stage's 128 K
            tma_load_2d_s(img_addr(st), &tm_xh, s * kBK, row0, &sh.full[st]);
            tma_load_2d_s(img_addr(st) + kPart, &tm_xl, s * kBK, row0, &sh.full[st]);
          } else {
            bulk_g2s(img_addr(st), src + int64_t(s) * kImg, uint32_t(kImg), &sh.full[st]);
          }
          if (KIND == 0) {
            tma_load_4d(b_addr(st), mw, s * kBK, nt * 128, 0, ez, &sh.full[st]);
            tma_load_4d(b_addr(st) + kBBytes / 2, mw, s * kBK, nt * 128 + 64, 0, ez, &sh.full[st]);
          } else {
            tma_load_3d(b_addr(st), mw, s * kBK, nt * kTN, ez, &sh.full[st]);
            tma_load_3d(b_addr(st) + kBBytes / 2, mw, s * kBK, nt * kTN + 128, ez, &sh.full[st]);
          }
          if (++st == kStages) { st = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- scale warp
    int st = 0, ph = 0, rs = 0, rph = 0;
    for (int q = blockIdx.x; q < n_items; q += gridDim.x) {
      if (warp_aborted(abort)) break;
      bool ok = true;
      for (int s = 0; s < S; ++s) {
        if ((s & 3) == 0 && !warp_wait(&sh.raw_full[rs], rph, abort)) { ok = false; break; }
        if (!warp_wait(&sh.empty[st], ph ^ 1, abort)) { ok = false; break; }
        // atom h: rows 128 h + lane + 32 m of the tile, the stage's four 32-K blocks
        const uint32_t rb = raw_base + rs * kRawBytes + 4 * (s & 3);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t w0 = lds_b32(rb + (128 * h + lane) * 16), w1 = lds_b32(rb + (128 * h + lane + 32) * 16),
                         w2 = lds_b32(rb + (128 * h + lane + 64) * 16), w3 = lds_b32(rb + (128 * h + lane + 96) * 16);
          sts_v4(sfb_addr(st) + h * kAtom + lane * 16, w0, w1, w2, w3);
        }
        if (KIND == 0) {  // the token rows' scale bytes: hi atom, lo atom (the down images carry theirs)
          const uint32_t rx = raw_base + rs * kRawBytes + kRawW + 4 * (s & 3);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t w0 = lds_b32(rx + h * (kRawX / 2) + lane * 16),
                           w1 = lds_b32(rx + h * (kRawX / 2) + (lane + 32) * 16),
                           w2 = lds_b32(rx + h * (kRawX / 2) + (lane + 64) * 16),
                           w3 = lds_b32(rx + h * (kRawX / 2) + (lane + 96) * 16);
            sts_v4(img_addr(st) + 2 * kPart + h * kAtom + lane * 16, w0, w1, w2, w3);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sh.full[st]);
          if ((s & 3) == 3) mbar_arrive(&sh.raw_empty[rs]);
        }
        if (++st == kStages) { st = 0; ph ^= 1; }
        if ((s & 3) == 3 && ++rs == kRawSlots) { rs = 0; rph ^= 1; }
      }
      if (!ok) {
        if (lane == 0) fail(94 + KIND);
        break;
      }
    }
  } else if (warp == 2) {
    // ---------------------------------------------------------------- MMA issuer
    int st = 0, ph = 0, li = 0;
    for (int q = blockIdx.x; q < n_items; q += gridDim.x, ++li) {
      if (warp_aborted(abort)) break;
      if (!warp_wait(&sh.tmem_empty, (li & 1) ^ 1, abort)) {
        if (lane == 0) fail(96 + KIND);
        break;
      }
      tc_fence_after();
      bool ok = true;
      for (int s = 0; s < S; ++s) {
        if (!warp_wait(&sh.full[st], ph, abort)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sf = tmem + kSfCol0 + st * kSfStage;  // SFA hi, SFA lo, SFB (two atoms)
        const uint32_t ia = img_addr(st);
        sf_copy_elect(sf, sf_desc(ia + 2 * kPart));
        sf_copy_elect(sf + 4, sf_desc(ia + 2 * kPart + kAtom));
        sf_copy_elect(sf + 8, sf_desc(sfb_addr(st)));
        sf_copy_elect(sf + 12, sf_desc(sfb_addr(st) + kAtom));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t db = umma_desc_sw128(b_addr(st) + 32 * kk);
          const uint32_t sfb = (sf + 8) | (uint32_t(kk) << 30);
          bs_mma_elect(tmem, umma_desc_sw128(ia + 32 * kk), db, g_idesc(uint32_t(kk)), sf | (uint32_t(kk) << 30), sfb,
                       (s > 0 || kk > 0) ? 1u : 0u);
          bs_mma_elect(tmem, umma_desc_sw128(ia + kPart + 32 * kk), db, g_idesc(uint32_t(kk)),
                       (sf + 4) | (uint32_t(kk) << 30), sfb, 1u);
        }
        umma_commit_elect(&sh.empty[st]);
        __syncwarp();
        if (++st == kStages) { st = 0; ph ^= 1; }
      }
      if (!ok) {
        if (lane == 0) fail(98 + KIND);
        break;
      }
      umma_commit_elect(&sh.tmem_full);
      __syncwarp();
    }
    // every MMA issued here has completed before TMEM is freed (bounded wait)
    umma_commit_elect(&sh.mma_done);
    __syncwarp();
    volatile int keep_waiting = 0;  // this wait ignores the abort flag (0.2 s bound)
    mbar_wait(&sh.mma_done, 0, &keep_waiting, 0, 200000000ull);
  } else if (warp >= kEpiWarp0) {
    // ---------------------------------------------------------------- epilogue
    const int quarter = warp & 3;                 // TMEM lanes 32 quarter .. + 31
    const int half = (warp - kEpiWarp0) >> 2;     // accumulator columns 128 half .. + 127
    const int r = quarter * 32 + lane;            // token row of the tile
    int li = 0;
    for (int q = blockIdx.x; q < n_items; q += gridDim.x, ++li) {
      if (warp_aborted(abort)) break;
      const int tile = q / n_nt, nt = q - tile * n_nt;
      const int row0 = a.plan.mtiles[2 * tile + 1];
      if (!warp_wait(&sh.tmem_full, li & 1, abort)) {
        if (lane == 0) fail(100 + KIND);
        break;
      }
      tc_fence_after();
      uint32_t v[128];
      const uint32_t taddr = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(half * 128);
      tmem_ld_32cols(taddr, v);
      tmem_ld_32cols(taddr + 32, v + 32);
      tmem_ld_32cols(taddr + 64, v + 64);
      tmem_ld_32cols(taddr + 96, v + 96);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.tmem_empty);  // the next tile's MMAs may overwrite the columns
      if (KIND == 0) {
        // columns 0..63 of this half: w13 rows nt * 128 + 64 half + i of the
        // first half of w13 (gate for the Qwen layout, up for [w3; w1]),
        // columns 64..127 the same rows of the second half
        const bool gate_lo = a.gate_first != 0;
        uint8_t* dst = a.act_img + (int64_t(tile) * (a.I / kBK) + nt) * kImg;
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          float act[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float c0 = __uint_as_float(v[32 * b + i]), c1 = __uint_as_float(v[64 + 32 * b + i]);
            const float gv = bf16_round(gate_lo ? c0 : c1), uv = bf16_round(gate_lo ? c1 : c0);
            act[i] = bf16_round(swiglu_f32(gv, uv, a.limit));
          }
          uint32_t hi[8], lo[8], bh, bl;
          split_block(act, hi, lo, &bh, &bl);
          const int c = half * 4 + 2 * b, kk = half * 2 + b;  // 16-byte chunk and 32-K block of the down stage
          *reinterpret_cast<uint4*>(dst + image_off(r, c)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
          *reinterpret_cast<uint4*>(dst + image_off(r, c + 1)) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
          *reinterpret_cast<uint4*>(dst + kPart + image_off(r, c)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
          *reinterpret_cast<uint4*>(dst + kPart + image_off(r, c + 1)) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
          dst[2 * kPart + atom_off(r, kk)] = uint8_t(bh);
          dst[2 * kPart + kAtom + atom_off(r, kk)] = uint8_t(bl);
        }
      } else {
        const int row = row0 + r;
        const int col = nt * kTN + half * 128;
        // padding rows (row_token < 0) are not stored; with ret set (expert-parallel
        // owner) the rows go straight into the senders' back blocks
        const int slot = a.plan.row_token[row];
        uint16_t* dst = slot < 0 ? nullptr : a.routed + int64_t(row) * a.H + col;
        if (a.ret.rows[0] != nullptr && slot >= 0)
          dst = a.ret.rows[slot / a.ret.capacity] + int64_t(slot % a.ret.capacity) * a.H + col;
        if (dst != nullptr) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint32_t pk[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
              pk[i] = pack_bf16x2(__uint_as_float(v[16 * c + 2 * i]), __uint_as_float(v[16 * c + 2 * i + 1]));
            asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst + 16 * c), "r"(pk[0]),
                         "r"(pk[1]), "r"(pk[2]), "r"(pk[3]), "r"(pk[4]), "r"(pk[5]), "r"(pk[6]), "r"(pk[7])
                         : "memory");
          }
        }
      }
    }
    // rows stored into other GPUs' memory: one system-scope fence per thread
    // after its last store, before the next kernel raises the flags
    if (KIND == 1 && a.ret.rows[0] != nullptr) __threadfence_system();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

void bsg_init_attributes() {
  cudaFuncSetAttribute(bsg_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes));
  cudaFuncSetAttribute(bsg_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes));
}

size_t bsg_image_bytes(int64_t mtiles, int K) { return size_t(mtiles) * size_t(K / kBK) * kImg; }

void launch_bsg_quant_scatter(const uint16_t* x, int rows, int K, const Plan& p, int topk, bool has_shared, int E,
                               const int32_t* counts, int capacity, uint8_t* hi, uint8_t* lo, uint8_t* shi,
                               uint8_t* slo, int num_sms, cudaStream_t stream) {
  bsg_quant_scatter_kernel<<<num_sms * 8, 256, 0, stream>>>(x, rows, K, p, topk, has_shared ? 1 : 0, E, counts,
                                                            capacity, hi, lo, shi, slo);
}

void launch_bsg(const BsArgs& a, int kind, const void* const* maps, int num_sms, cudaStream_t stream) {
  const CUtensorMap* m[8];
  for (int i = 0; i < 8; ++i) m[i] = static_cast<const CUtensorMap*>(maps[kind == 0 || i < 4 ? i : 0]);
  if (kind == 0)
    bsg_kernel<0><<<num_sms, kThreads, kSmemBytes, stream>>>(*m[0], *m[1], *m[2], *m[3], *m[4], *m[5], *m[6], *m[7],
                                                             a);
  else
    bsg_kernel<1><<<num_sms, kThreads, kSmemBytes, stream>>>(*m[0], *m[1], *m[2], *m[3], *m[4], *m[5], *m[6], *m[7],
                                                             a);
}

}  // namespace wm
