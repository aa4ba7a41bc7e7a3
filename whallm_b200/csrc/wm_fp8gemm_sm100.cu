// Prefill path for FP8 experts with fp32 128 x 128 block scales (config 3) on
// tcgen05 block-scaled MMA (kind::mxf8f6f4): the E4M3 weights go from the
// blob to the tensor cores by TMA as they are, and each weight block's fp32
// scale is applied outside the MMA, per 128-K block, in fp32 registers.
//
// Reference arithmetic: the DeepSeek-style FP8 linears decode each weight as
// bf16(e4m3 * scale) (mimo/weights.py:38-41, Native/DeepSeekNative/
// kernels.metal:106-160 linear_fp8, kernels_tensorops.metal:30-76 tops_fp8)
// and multiply with fp32 accumulation.  Here a weight enters as its exact
// E4M3 value and the product of a 128-K block is scaled once by the block's
// fp32 scale: the weights are exact instead of rounded to bf16 (a 2^-9
// relative difference per weight at most, well inside the layer tolerance).
//
// Operands of one MMA (M = 128 token rows, N = 128 weight rows, K = 32):
//   A  token rows as hi / lo E4M3 parts with UE8M0 scales per 32 K (the
//      block-scaled MXFP4 GEMM's operand: the same sorted rows for gate/up,
//      the same act tile images for down); a hi and a lo MMA per K step.
//   B  E4M3 weights by TMA, K-major, 128-byte swizzle; their scale factors
//      are one constant atom of 2^0 (the weight scale is not a power of two).
//   D  a fresh fp32 partial per 128-K block in TMEM (two, alternating; a
//      third measured no faster).
// The 8 epilogue warps load each partial, multiply it by the block's weight
// scale and add it to fp32 accumulators in registers (64 per thread); at the
// tile's end they run the gate/up epilogue (bf16 gate / up, SwiGLU, the act
// rows' hi / lo split into act tile images) or store the down rows.
//
// Tiles: gate/up 128 tokens x (64 first-half + the 64 matching second-half
// rows of w13, one 4-D box), so a thread owns 32 gate and the 32 matching up
// columns; down 128 tokens x 128 rows of w2.  One persistent CTA per SM,
// 12 warps: warp 0 TMA producer, warp 1 scale warp (gate/up: token scale
// rows -> the stage's A atoms), warp 2 TMEM owner and MMA issuer, warps 4-11
// promotion and epilogue.  Four stages of 49 KB.  Every mbarrier wait is
// bounded (2 s); on a timeout the kernel records the status, the other roles
// unwind and TMEM is freed.
#include "wm_bs_common.cuh"
#include "wm_kernels.h"

namespace wm {

namespace {

constexpr int kTM = 128;                       // token rows per tile (MMA M)
constexpr int kTN = 128;                       // weight rows per tile (MMA N)
constexpr int kBK = 128;                       // K per stage = one weight-scale block
constexpr int kStages = 4;
constexpr int kThreads = 384;
constexpr int kEpiWarp0 = 4, kEpiWarps = 8;
constexpr int kPart = kTM * kBK;               // one part's 128 rows of 128 bytes
constexpr int kAtom = 512;
constexpr int kImg = 2 * kPart + 2 * kAtom;    // A: hi rows, lo rows, hi atom, lo atom
constexpr int kBBytes = kTN * kBK;             // 128 E4M3 weight rows
constexpr int kStageBytes = kImg + kBBytes;
constexpr int kRawSlots = 2;
constexpr int kRawBytes = 2 * kTM * 16;        // gate/up: 128 token rows x 16 scale bytes, hi then lo
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kPartCols = kTN;            // TMEM columns of one partial
constexpr int kParts = 2;                      // partials in flight between the MMAs and the promotion
constexpr uint32_t kSfaCol0 = kParts * kPartCols;  // SFA hi / lo: 8 columns per stage
constexpr uint32_t kSfbCol = kSfaCol0 + 8 * kStages;  // the constant SFB atom: 4 columns
static_assert(kSfbCol + 4 <= kTmemCols, "scale factors exceed the TMEM allocation");
static_assert(kImg % 1024 == 0 && kStageBytes % 1024 == 0, "swizzled operands need 1024-byte alignment");
static_assert(kRawBytes % 128 == 0, "TMA destinations in shared memory must be 128-byte aligned");

struct FShared {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t raw_full[kRawSlots];
  uint64_t raw_empty[kRawSlots];
  uint64_t pfull[kParts];   // partial p holds a finished 128-K block
  uint64_t pempty[kParts];  // the epilogue warps have loaded partial p
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
  alignas(128) uint8_t sfb[kAtom];  // 0x7F everywhere: UE8M0 2^0 (tcgen05.cp source)
};

constexpr size_t kSmemBytes = size_t(kStages) * kStageBytes + size_t(kRawSlots) * kRawBytes + sizeof(FShared) + 1024;
static_assert(kSmemBytes <= 232448, "more shared memory than a B200 CTA may have");

// kind::mxf8f6f4 instruction descriptor: A and B E4M3, both K-major, UE8M0
// scales, M = 128, N = 128, scale-factor ids kk for A and B.
__device__ __forceinline__ uint32_t f_idesc(uint32_t kk) {
  return (kk << 4) | (0u << 7) | (0u << 10) | (uint32_t(kTN >> 3) << 17) | (1u << 23) | (uint32_t(kTM >> 4) << 24) |
         (kk << 29);
}

// Byte of (part row n, 32-K block kk of the stage) in a scale atom.
__device__ __forceinline__ int atom_off(int n, int kk) { return (n & 31) * 16 + (n >> 5) * 4 + kk; }

}  // namespace

// KIND 0: gate/up + SwiGLU -> act tile images (a.act_img, the block-scaled
// down GEMM's layout); KIND 1: down -> routed [rows, H] bf16, or with
// a.ret.rows[0] set the senders' back blocks.  tm_w: the w13 (4-D [E][2][I][H],
// boxes 128 x 64 x 2) or w2 (3-D [E][H][I], boxes 128 x 128) E4M3 bytes of
// the routed experts, tm_ws the shared expert's; tm_xsh / tm_xsl / tm_xh /
// tm_xl (gate/up) the sorted rows' parts and scale rows.
template <int KIND>
__global__ void __launch_bounds__(kThreads, 1) fp8g_kernel(const __grid_constant__ CUtensorMap tm_w,
                                                           const __grid_constant__ CUtensorMap tm_ws,
                                                           const __grid_constant__ CUtensorMap tm_xh,
                                                           const __grid_constant__ CUtensorMap tm_xl,
                                                           const __grid_constant__ CUtensorMap tm_xsh,
                                                           const __grid_constant__ CUtensorMap tm_xsl,
                                                           const BsArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const int K = KIND == 0 ? a.H : a.I;
  const int S = K / kBK;  // stages (= weight-scale blocks) per tile, a multiple of 4
  const int n_nt = KIND == 0 ? a.I / 64 : a.H / kTN;
  const int n_items = *a.plan.n_mtiles * n_nt;
  const uint32_t raw0 = smem_u32(smem_raw);
  const uint32_t base = (raw0 + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw0);
  FShared& sh = *reinterpret_cast<FShared*>(gbase + kStages * kStageBytes + kRawSlots * kRawBytes);
  const uint32_t raw_base = base + kStages * kStageBytes;
  auto img_addr = [&](int slot) { return base + slot * kStageBytes; };
  auto b_addr = [&](int slot) { return base + slot * kStageBytes + kImg; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sh.full[i], KIND == 0 ? 2 : 1);  // the TMA producer (with bytes) and, for gate/up, the scale warp
      mbar_init(&sh.empty[i], 1);
    }
    for (int i = 0; i < kRawSlots; ++i) {
      mbar_init(&sh.raw_full[i], 1);
      mbar_init(&sh.raw_empty[i], 1);
    }
    for (int i = 0; i < kParts; ++i) {
      mbar_init(&sh.pfull[i], 1);
      mbar_init(&sh.pempty[i], kEpiWarps);
    }
    mbar_init(&sh.mma_done, 1);
    sh.abort = 0;
    fence_mbarrier_init();
  }
  for (int i = threadIdx.x; i < kAtom / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(sh.sfb)[i] = 0x7F7F7F7Fu;
  fence_proxy_async_smem();
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
        const int ez = shared_e ? 0 : e;
        const uint8_t* src = a.img + int64_t(tile) * S * kImg;  // down: image (tile, s) at (tile * S + s) * kImg
        for (int s = 0; s < S; ++s) {
          if (KIND == 0 && (s & 3) == 0) {  // the token rows' scale bytes of the next four stages, hi then lo
            if (!mbar_wait(&sh.raw_empty[rs], rph ^ 1, abort)) { fail(110); break; }
            const uint32_t dst = raw_base + rs * kRawBytes;
            mbar_arrive_expect_tx(&sh.raw_full[rs], uint32_t(kRawBytes));
            tma_load_2d_s(dst, &tm_xsh, 16 * (s >> 2), row0, &sh.raw_full[rs]);
            tma_load_2d_s(dst + kRawBytes / 2, &tm_xsl, 16 * (s >> 2), row0, &sh.raw_full[rs]);
            if (++rs == kRawSlots) { rs = 0; rph ^= 1; }
          }
          if (!mbar_wait(&sh.empty[st], ph ^ 1, abort)) { fail(112 + KIND); break; }
          if (KIND == 0) {
            mbar_arrive_expect_tx(&sh.full[st], uint32_t(2 * kPart + kBBytes));
            tma_load_2d_s(img_addr(st), &tm_xh, s * kBK, row0, &sh.full[st]);
            tma_load_2d_s(img_addr(st) + kPart, &tm_xl, s * kBK, row0, &sh.full[st]);
            tma_load_4d(b_addr(st), mw, s * kBK, nt * 64, 0, ez, &sh.full[st]);  // 64 rows of each half
          } else {
            mbar_arrive_expect_tx(&sh.full[st], uint32_t(kImg + kBBytes));
            bulk_g2s(img_addr(st), src + int64_t(s) * kImg, uint32_t(kImg), &sh.full[st]);
            tma_load_3d(b_addr(st), mw, s * kBK, nt * kTN, ez, &sh.full[st]);
          }
          if (++st == kStages) { st = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- scale warp (gate/up)
    if (KIND == 0) {
      int st = 0, ph = 0, rs = 0, rph = 0;
      for (int q = blockIdx.x; q < n_items; q += gridDim.x) {
        if (warp_aborted(abort)) break;
        bool ok = true;
        for (int s = 0; s < S; ++s) {
          if ((s & 3) == 0 && !warp_wait(&sh.raw_full[rs], rph, abort)) { ok = false; break; }
          if (!warp_wait(&sh.empty[st], ph ^ 1, abort)) { ok = false; break; }
          // atom h (hi, lo): token rows lane + 32 m, the stage's four 32-K blocks
          const uint32_t rx = raw_base + rs * kRawBytes + 4 * (s & 3);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t w0 = lds_b32(rx + h * (kRawBytes / 2) + lane * 16),
                           w1 = lds_b32(rx + h * (kRawBytes / 2) + (lane + 32) * 16),
                           w2 = lds_b32(rx + h * (kRawBytes / 2) + (lane + 64) * 16),
                           w3 = lds_b32(rx + h * (kRawBytes / 2) + (lane + 96) * 16);
            sts_v4(img_addr(st) + 2 * kPart + h * kAtom + lane * 16, w0, w1, w2, w3);
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
          if (lane == 0) fail(114);
          break;
        }
      }
    }
  } else if (warp == 2) {
    // ---------------------------------------------------------------- MMA issuer
    // the weights' scale factors, 2^0 for every row and block, once (the
    // tensor pipe runs this thread's copies and MMAs in order)
    sf_copy_elect(tmem + kSfbCol, sf_desc(smem_u32(sh.sfb)));
    int st = 0, ph = 0, pu = 0;  // pu: partials issued; partial pu % kParts
    for (int q = blockIdx.x; q < n_items; q += gridDim.x) {
      if (warp_aborted(abort)) break;
      bool ok = true;
      for (int s = 0; s < S; ++s, ++pu) {
        const int p = pu % kParts;
        if (!warp_wait(&sh.pempty[p], ((pu / kParts) & 1) ^ 1, abort)) { ok = false; break; }
        if (!warp_wait(&sh.full[st], ph, abort)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sfa = tmem + kSfaCol0 + st * 8;  // SFA hi, SFA lo
        const uint32_t ia = img_addr(st);
        sf_copy_elect(sfa, sf_desc(ia + 2 * kPart));
        sf_copy_elect(sfa + 4, sf_desc(ia + 2 * kPart + kAtom));
        const uint32_t d = tmem + uint32_t(p) * kPartCols;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t db = umma_desc_sw128(b_addr(st) + 32 * kk);
          const uint32_t sfb = (tmem + kSfbCol) | (uint32_t(kk) << 30);
          bs_mma_elect(d, umma_desc_sw128(ia + 32 * kk), db, f_idesc(uint32_t(kk)), sfa | (uint32_t(kk) << 30), sfb,
                       kk > 0 ? 1u : 0u);
          bs_mma_elect(d, umma_desc_sw128(ia + kPart + 32 * kk), db, f_idesc(uint32_t(kk)),
                       (sfa + 4) | (uint32_t(kk) << 30), sfb, 1u);
        }
        umma_commit_elect(&sh.empty[st]);
        umma_commit_elect(&sh.pfull[p]);
        __syncwarp();
        if (++st == kStages) { st = 0; ph ^= 1; }
      }
      if (!ok) {
        if (lane == 0) fail(116 + KIND);
        break;
      }
    }
    // every MMA issued here has completed before TMEM is freed (bounded wait)
    umma_commit_elect(&sh.mma_done);
    __syncwarp();
    volatile int keep_waiting = 0;  // this wait ignores the abort flag (0.2 s bound)
    mbar_wait(&sh.mma_done, 0, &keep_waiting, 0, 200000000ull);
  } else if (warp >= kEpiWarp0) {
    // ---------------------------------------------------------------- promotion and epilogue
    const int quarter = warp & 3;              // TMEM lanes 32 quarter .. + 31
    const int half = (warp - kEpiWarp0) >> 2;  // gate/up: columns 32 half .. and 64 + 32 half ..; down: 64 half ..
    const int r = quarter * 32 + lane;         // token row of the tile
    const int kb_rows = K / kBK;               // weight-scale blocks per row block
    int pu = 0;
    for (int q = blockIdx.x; q < n_items; q += gridDim.x) {
      if (warp_aborted(abort)) break;
      const int tile = q / n_nt, nt = q - tile * n_nt;
      const int e = a.plan.mtiles[2 * tile], row0 = a.plan.mtiles[2 * tile + 1];
      const bool shared_e = e == a.wts.E;
      // the fp32 block scales of this tile's rows: gate/up the first-half block
      // (rows nt * 64 ..) and the second-half block (rows I + nt * 64 ..), down block nt
      const float* sc = reinterpret_cast<const float*>(
          KIND == 0 ? (shared_e ? a.wts.sh_s13 : a.wts.s13 + int64_t(e) * a.wts.s13_stride)
                    : (shared_e ? a.wts.sh_s2 : a.wts.s2 + int64_t(e) * a.wts.s2_stride));
      const float* sc0 = sc + int64_t(KIND == 0 ? (nt * 64) / 128 : nt) * kb_rows;
      const float* sc1 = sc + int64_t(KIND == 0 ? (a.I + nt * 64) / 128 : nt) * kb_rows;
      float acc[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) acc[i] = 0.0f;
      bool ok = true;
      for (int s = 0; s < S; ++s, ++pu) {
        const int p = pu % kParts;
        const float s0 = __ldg(sc0 + s), s1 = __ldg(sc1 + s);
        if (!warp_wait(&sh.pfull[p], (pu / kParts) & 1, abort)) { ok = false; break; }
        tc_fence_after();
        uint32_t v[64];
        const uint32_t taddr = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(p) * kPartCols;
        if (KIND == 0) {
          tmem_ld_32cols(taddr + 32 * half, v);
          tmem_ld_32cols(taddr + 64 + 32 * half, v + 32);
        } else {
          tmem_ld_32cols(taddr + 64 * half, v);
          tmem_ld_32cols(taddr + 64 * half + 32, v + 32);
        }
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.pempty[p]);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          acc[i] = fmaf(s0, __uint_as_float(v[i]), acc[i]);
          acc[32 + i] = fmaf(KIND == 0 ? s1 : s0, __uint_as_float(v[32 + i]), acc[32 + i]);
        }
      }
      if (!ok) {
        if (lane == 0) fail(118 + KIND);
        break;
      }
      if (KIND == 0) {
        // features f = nt * 64 + 32 half + i: acc[i] from the first half of
        // w13 (gate for gate-first layouts, up for [w3; w1]), acc[32 + i] the
        // same rows of the second half; one 32-K block of a down stage
        const bool gate_lo = a.gate_first != 0;
        float act[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float gv = bf16_round(gate_lo ? acc[i] : acc[32 + i]);
          const float uv = bf16_round(gate_lo ? acc[32 + i] : acc[i]);
          act[i] = bf16_round(swiglu_f32(gv, uv, a.limit));
        }
        uint32_t hi[8], lo[8], bh, bl;
        split_block(act, hi, lo, &bh, &bl);
        const int f = nt * 64 + 32 * half;
        const int sd = f / kBK, kk = (f % kBK) / 32;  // down stage and its 32-K block
        uint8_t* dst = a.act_img + (int64_t(tile) * (a.I / kBK) + sd) * kImg;
        *reinterpret_cast<uint4*>(dst + image_off(r, 2 * kk)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(dst + image_off(r, 2 * kk + 1)) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
        *reinterpret_cast<uint4*>(dst + kPart + image_off(r, 2 * kk)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        *reinterpret_cast<uint4*>(dst + kPart + image_off(r, 2 * kk + 1)) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
        dst[2 * kPart + atom_off(r, kk)] = uint8_t(bh);
        dst[2 * kPart + kAtom + atom_off(r, kk)] = uint8_t(bl);
      } else {
        // padding rows (row_token < 0) are not stored; with ret set (expert-parallel
        // owner) the rows go straight into the senders' back blocks
        const int row = row0 + r;
        const int col = nt * kTN + 64 * half;
        const int slot = a.plan.row_token[row];
        uint16_t* dst = slot < 0 ? nullptr : a.routed + int64_t(row) * a.H + col;
        if (a.ret.rows[0] != nullptr && slot >= 0)
          dst = a.ret.rows[slot / a.ret.capacity] + int64_t(slot % a.ret.capacity) * a.H + col;
        if (dst != nullptr) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t pk[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) pk[i] = pack_bf16x2(acc[16 * c + 2 * i], acc[16 * c + 2 * i + 1]);
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

void fp8g_init_attributes() {
  cudaFuncSetAttribute(fp8g_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes));
  cudaFuncSetAttribute(fp8g_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes));
}

bool fp8g_shape_ok(int H, int I) { return H % 512 == 0 && I % 512 == 0 && H >= 512 && I >= 512; }

void launch_fp8g(const BsArgs& a, int kind, const void* const* maps, int num_sms, cudaStream_t stream) {
  const CUtensorMap* m[6];
  for (int i = 0; i < 6; ++i) m[i] = static_cast<const CUtensorMap*>(maps[kind == 0 || i < 2 ? i : 0]);
  if (kind == 0)
    fp8g_kernel<0><<<num_sms, kThreads, kSmemBytes, stream>>>(*m[0], *m[1], *m[2], *m[3], *m[4], *m[5], a);
  else
    fp8g_kernel<1><<<num_sms, kThreads, kSmemBytes, stream>>>(*m[0], *m[1], *m[2], *m[3], *m[4], *m[5], a);
}

}  // namespace wm
