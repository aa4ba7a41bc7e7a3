// Prefill path: grouped GEMM over expert-sorted rows on the 5th-generation
// tensor cores (tcgen05.mma, kind::f16, fp32 accumulators in TMEM), with the
// expert weights dequantised on the fly.  MXFP4 experts run with f16
// operands: the sorted activation rows are f16 copies scaled by 2^k per row
// (exact, as in the decode path) and a weight row enters as E2M1 * 2^(s -
// smax) with smax its largest E8M0 byte (exact in f16 for every group within
// 23 binades of it), one hardware conversion and one f16x2 multiply per two
// weights; the epilogue applies 2^(smax - 127) per column and 2^-k per row.
// FP8 experts run with bf16 operands (each weight rounded to bf16 after its
// fp32 128x128 block scale, as the reference decodes them, or after its
// UE8M0 32x32 block scale, two per 64-K block).
//
// Reference arithmetic: mx.gather_qmm(..., mode="mxfp4", group_size=32,
// sorted_indices=True) over expert-sorted rows (model.py:435-501,
// qwen4_exp.py:853-904) and the tiled Metal kernels expert_gemm_sg /
// tops_expert (QwenNative/kernels.metal:706-752, kernels_tensorops.metal:49-87,
// DeepSeekNative/kernels.metal:1018-1058): per expert, Y = X_e W_e^T with
// exact dequantised weights and fp32 accumulation.  The gate/up product is
// followed by SwiGLU in the epilogue (the reference's separate expert_act
// dispatch); the down product writes bf16 rows for the combine.
//
// One persistent CTA per SM walks the (128-row tile, 256-column tile) work
// list in a fixed order.  Warp roles:
//   warp 0      TMA producer: the 128 x 64 bf16 activation tile of each stage
//   warp 1      TMEM allocator and the single MMA-issuing thread
//   warps 2-9   weight producers: each thread loads one weight row's 64 K
//               values (MXFP4 nibbles + E8M0, or E4M3 + fp32 block scale),
//               dequantises them (f16 or bf16) and stores them in the
//               128-byte swizzled K-major layout the MMA reads
//   warps 10-13 epilogue: TMEM -> registers -> SwiGLU / bf16 -> global
// Four smem stages of (A 16 KB + B 32 KB); two 128 x 256 fp32 accumulators in
// TMEM (all 512 columns) so the epilogue of one tile overlaps the next tile's
// main loop.  Every mbarrier wait is bounded (2 s); on a timeout the kernel
// records the status, the other roles unwind, and TMEM is freed.
#include <cuda.h>

#include "wm_kernels.h"

namespace wm {

namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4, UMMA_K = 16;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int NUM_THREADS = 448;
constexpr int DQ_WARP0 = 2, DQ_WARPS = 8, EPI_WARP0 = 10;
constexpr uint32_t TMEM_COLS = 512;
// Column exponents of the MXFP4 path (each weight row's largest E8M0 byte),
// one set per tile in flight.  Producers run at most STAGES K blocks ahead of
// the MMA, and the MMA starts tile n + 2 only after the epilogue of tile n, so
// the set of tile n + CF_SETS is written after that epilogue whenever
// (CF_SETS - 2) * kblocks > STAGES: 5 sets cover two K blocks per tile (every
// K >= 128).  Kept as bytes: shared memory past ~195 KB per CTA shrinks the
// L1 carve-out, and on B200 that halved this kernel's speed.
constexpr int CF_SETS = 5;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + CF_SETS * BN + 256 /*barriers*/;

struct Shared {
  uint8_t colx[CF_SETS][BN];  // largest E8M0 byte of each weight row of the tile (MXFP4)
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t colf_full[CF_SETS];  // a tile's column factors are written (MXFP4)
  uint32_t tmem_base;
  int abort;
};

// Eight E4M3 bytes times the fp32 block scale, rounded to bf16 (fp32 product
// rounded once, then bf16: mimo/weights.py:38-41).
__device__ __forceinline__ uint4 dq_fp8_8(uint32_t lo, uint32_t hi, float scale) {
  float v[8];
  e4m3x4_to_f32(lo, v);
  e4m3x4_to_f32(hi, v + 4);
  uint4 o;
  o.x = pack_bf16x2(__fmul_rn(v[0], scale), __fmul_rn(v[1], scale));
  o.y = pack_bf16x2(__fmul_rn(v[2], scale), __fmul_rn(v[3], scale));
  o.z = pack_bf16x2(__fmul_rn(v[4], scale), __fmul_rn(v[5], scale));
  o.w = pack_bf16x2(__fmul_rn(v[6], scale), __fmul_rn(v[7], scale));
  return o;
}

// One word of E2M1 nibbles (8 values) times the f16x2 multiplier -> 4 f16x2.
__device__ __forceinline__ uint4 dq_mxfp4_word_f16(uint32_t w, uint32_t m2) {
  uint32_t h0, h1, h2, h3;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3)
      : "r"(w));
  uint4 o;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o.x) : "r"(h0), "r"(m2));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o.y) : "r"(h1), "r"(m2));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o.z) : "r"(h2), "r"(m2));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o.w) : "r"(h3), "r"(m2));
  return o;
}

// f16x2 holding 2^(s - smax) twice, given rinv = 2^(127 - smax): 0 for the
// E8M0 byte 0 (the Metal convention) and below f16's range; exact otherwise.
__device__ __forceinline__ uint32_t e8m0_mult_f16x2(uint32_t s, float rinv) {
  const float f = __uint_as_float(s << 23) * rinv;
  uint32_t h;
  asm("cvt.rn.f16x2.f32 %0, %1, %1;" : "=r"(h) : "f"(f));
  return h;
}

__device__ __forceinline__ void sts_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// 32 bytes per lane (one full sector): 256-bit global accesses (sm_100).
__device__ __forceinline__ void ldg_nc_v8(const void* p, uint4& lo, uint4& hi) {
  asm volatile("ld.global.nc.L1::no_allocate.v8.u32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(lo.x), "=r"(lo.y), "=r"(lo.z), "=r"(lo.w), "=r"(hi.x), "=r"(hi.y), "=r"(hi.z), "=r"(hi.w)
               : "l"(p));
}

__device__ __forceinline__ void stg_v8(void* p, const uint32_t* v) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(v[0]), "r"(v[1]), "r"(v[2]),
               "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}


__device__ __forceinline__ void fail(Shared& sh, uint32_t* status, uint32_t role) {
  report_status(status, kStatusWaitTimeout, role);
  sh.abort = 1;
}

}  // namespace

// KIND 0: gate/up + SwiGLU -> act [rows, I];  KIND 1: down -> routed [rows, H].
template <int FMT, int KIND>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* tiles = smem_raw + (base - raw);
  Shared& sh = *reinterpret_cast<Shared*>(tiles + STAGES * STAGE_BYTES);
  const uint32_t a_smem = base;                      // STAGES x A_BYTES
  const uint32_t b_smem = base + STAGES * A_BYTES;   // STAGES x B_BYTES

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles_n = KIND == 0 ? a.I / (BN / 2) : a.N / BN;
  const int kblocks = a.Kdim / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sh.full[s], 1 + DQ_WARPS);
      mbar_init(&sh.empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh.tmem_full[i], 1);
      mbar_init(&sh.tmem_empty[i], 4);
    }
    for (int i = 0; i < CF_SETS; ++i) mbar_init(&sh.colf_full[i], DQ_WARPS);
    sh.abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&sh.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tmap_a);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  volatile int* abort = &sh.abort;

  const int total = *a.plan.n_mtiles * n_tiles_n;

  if (warp == 0) {
    // ---------------------------------------------------------------- A producer (TMA)
    if (lane == 0) {
      uint32_t it = 0;
      for (int t = blockIdx.x; t < total && !*abort; t += gridDim.x) {
        const int row0 = a.plan.mtiles[2 * (t / n_tiles_n) + 1];
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(&sh.empty[s], ph ^ 1u, abort)) {
            fail(sh, a.status, 10);
            break;
          }
          mbar_arrive_expect_tx(&sh.full[s], A_BYTES);
          tma_load_2d(tiles + s * A_BYTES, &tmap_a, kb * BK, row0, &sh.full[s]);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    // The whole warp runs the loop (its waits are warp-uniform) and one
    // elected lane issues each tcgen05 instruction.
    // MXFP4: f16 A and B (format 0); FP8: bf16 A and B
    constexpr uint32_t idesc =
        FMT == kFmtMxfp4 ? ((1u << 4) | ((uint32_t(BN) >> 3) << 17) | ((uint32_t(BM) >> 4) << 24))
                         : umma_idesc_bf16(BM, BN);
    uint32_t it = 0, lt = 0;
    for (int t = blockIdx.x; t < total && !warp_aborted(abort); t += gridDim.x, ++lt) {
      const uint32_t acc = lt & 1u, acc_ph = (lt >> 1) & 1u;
      if (!warp_wait(&sh.tmem_empty[acc], acc_ph ^ 1u, abort)) {
        if (lane == 0) fail(sh, a.status, 11);
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem + acc * BN;
      bool ok = true;
      for (int kb = 0; kb < kblocks; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1u;
        if (!warp_wait(&sh.full[s], ph, abort)) {
          if (lane == 0) fail(sh, a.status, 12);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t da = umma_desc_sw128(a_smem + s * A_BYTES);
        const uint64_t db = umma_desc_sw128(b_smem + s * B_BYTES);
#pragma unroll
        for (int k = 0; k < BK / UMMA_K; ++k)  // K16 step = 32 bytes = 2 in the descriptor's address field
          umma_f16_elect(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
        umma_commit_elect(&sh.empty[s]);
      }
      if (!ok) break;
      umma_commit_elect(&sh.tmem_full[acc]);
    }
  } else if (warp < EPI_WARP0) {
    // ---------------------------------------------------------------- weight producers
    // Loads run PF K blocks ahead of the dequantisation (across tiles), so a
    // block's bytes are in registers when its turn comes.  MXFP4: the next
    // tile's row maximum of E8M0 bytes is gathered 4 bytes per K block during
    // the current tile.
    constexpr int PF = 2;
    constexpr int NW = FMT == kFmtMxfp4 ? 2 : 4;  // 16-byte weight loads per K block
    const int j = (warp - DQ_WARP0) * 32 + lane;  // B-tile row 0..255
    const int gate_base = a.gate_first ? 0 : a.I, up_base = a.gate_first ? a.I : 0;
    const int64_t rb = FMT == kFmtMxfp4 ? a.Kdim / 2 : a.Kdim;   // weight row bytes
    const int S32 = a.Kdim / 32;  // scale bytes per row: E8M0 (MXFP4) or UE8M0 per 32-row block (FP8 32x32)
    auto grow_of = [&](int t) {
      const int nt = t % n_tiles_n;
      if (KIND == 0) return j < BN / 2 ? gate_base + nt * (BN / 2) + j : up_base + nt * (BN / 2) + (j - BN / 2);
      return nt * BN + j;
    };
    auto expert_of = [&](int t) { return a.plan.mtiles[2 * (t / n_tiles_n)]; };
    auto wrow_of = [&](int t) -> const uint8_t* {
      const int e = expert_of(t);
      return (KIND == 0 ? a.wts.w13_of(e) : a.wts.w2_of(e)) + int64_t(grow_of(t)) * rb;
    };
    // E8M0 row (MXFP4) or the fp32 block-scale row of this weight row (FP8)
    auto srow_of = [&](int t) -> const uint8_t* {
      const int e = expert_of(t);
      const uint8_t* sb = KIND == 0 ? a.wts.s13_of(e) : a.wts.s2_of(e);
      if (FMT == kFmtMxfp4) return sb + int64_t(grow_of(t)) * S32;
      if (FMT == kFmtFp8B32) return sb + int64_t(grow_of(t) / 32) * S32;  // UE8M0 row of the 32-row block
      return sb + (int64_t(grow_of(t) / 128) * (a.Kdim / 128)) * 4;
    };
    auto byte_max = [](uint32_t m) { return max(max(m & 0xffu, (m >> 8) & 0xffu), max((m >> 16) & 0xffu, m >> 24)); };
    // load cursor
    int lt_t = blockIdx.x, lkb = 0;
    const uint8_t* lw = lt_t < total ? wrow_of(lt_t) : nullptr;
    const uint8_t* ls = lt_t < total ? srow_of(lt_t) : nullptr;
    uint4 wq[PF][NW];
    uint32_t sq[PF];  // MXFP4 / FP8 32x32: the K block's two scale bytes; FP8 128x128: the block scale's bits
    auto load_next = [&](uint4 (&w)[NW], uint32_t& sv) {
      if (lt_t >= total) return;
#pragma unroll
      for (int i = 0; i < NW; i += 2) {  // a weight row's K block: whole 32-byte sectors when aligned
        const uint8_t* src = lw + lkb * (16 * NW) + 16 * i;
        if (a.w32) {
          ldg_nc_v8(src, w[i], w[i + 1]);
        } else {
          w[i] = ldg_nc_v4(src);
          w[i + 1] = ldg_nc_v4(src + 16);
        }
      }
      if (FMT == kFmtMxfp4 || FMT == kFmtFp8B32) {
        uint16_t v;
        asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(ls + lkb * 2));
        sv = v;
      } else {
        sv = __float_as_uint(__ldg(reinterpret_cast<const float*>(ls) + lkb / 2));
      }
      if (++lkb == kblocks) {
        lkb = 0;
        lt_t += gridDim.x;
        if (lt_t < total) {
          lw = wrow_of(lt_t);
          ls = srow_of(lt_t);
        }
      }
    };
#pragma unroll
    for (int i = 0; i < PF; ++i) load_next(wq[i], sq[i]);

    // MXFP4: this tile's row maximum (the first tile's read directly)
    uint32_t smax_cur = 0;
    if (FMT == kFmtMxfp4 && int(blockIdx.x) < total) {
      const uint8_t* sr = srow_of(blockIdx.x);
      uint32_t m = 0;
      for (int i = 0; i < S32; i += 4) m = __vmaxu4(m, __ldg(reinterpret_cast<const uint32_t*>(sr + i)));
      smax_cur = byte_max(m);
    }
    uint32_t it = 0, lt = 0;
    for (int t = blockIdx.x; t < total && !*abort; t += gridDim.x, ++lt) {
      float rinv = 1.0f;  // MXFP4: 2^(127 - smax) of this weight row
      const uint8_t* nsr = nullptr;
      uint32_t nm = 0;    // the next tile's running maximum
      if (FMT == kFmtMxfp4) {
        rinv = __uint_as_float(uint32_t(254 - min(int(smax_cur), 254)) << 23);
        sh.colx[lt % CF_SETS][j] = uint8_t(smax_cur);
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.colf_full[lt % CF_SETS]);
        if (t + int(gridDim.x) < total) nsr = srow_of(t + gridDim.x);
      }
      bool ok = true;
      for (int kb = 0; kb < kblocks; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1u;
        uint4 w[NW];
#pragma unroll
        for (int i = 0; i < NW; ++i) w[i] = wq[0][i];
        const uint32_t sv = sq[0];
#pragma unroll
        for (int p = 0; p + 1 < PF; ++p) {
#pragma unroll
          for (int i = 0; i < NW; ++i) wq[p][i] = wq[p + 1][i];
          sq[p] = sq[p + 1];
        }
        load_next(wq[PF - 1], sq[PF - 1]);
        uint4 q[8];
        if (FMT == kFmtMxfp4) {
          if (nsr != nullptr)  // the next tile's E8M0 bytes, 4 per K block (S32 / 4 <= kblocks)
            if (kb * 4 < S32) nm = __vmaxu4(nm, __ldg(reinterpret_cast<const uint32_t*>(nsr + kb * 4)));
          const uint32_t m0 = e8m0_mult_f16x2(sv & 0xffu, rinv), m1 = e8m0_mult_f16x2(sv >> 8, rinv);
          q[0] = dq_mxfp4_word_f16(w[0].x, m0);
          q[1] = dq_mxfp4_word_f16(w[0].y, m0);
          q[2] = dq_mxfp4_word_f16(w[0].z, m0);
          q[3] = dq_mxfp4_word_f16(w[0].w, m0);
          q[4] = dq_mxfp4_word_f16(w[1].x, m1);
          q[5] = dq_mxfp4_word_f16(w[1].y, m1);
          q[6] = dq_mxfp4_word_f16(w[1].z, m1);
          q[7] = dq_mxfp4_word_f16(w[1].w, m1);
        } else {
          // FP8 128x128: one fp32 scale per K block; 32x32: a UE8M0 scale per 32 K
          const float sc0 = FMT == kFmtFp8B32 ? e8m0_to_f32(sv & 0xffu, true) : __uint_as_float(sv);
          const float sc1 = FMT == kFmtFp8B32 ? e8m0_to_f32(sv >> 8, true) : sc0;
          q[0] = dq_fp8_8(w[0].x, w[0].y, sc0);
          q[1] = dq_fp8_8(w[0].z, w[0].w, sc0);
          q[2] = dq_fp8_8(w[1].x, w[1].y, sc0);
          q[3] = dq_fp8_8(w[1].z, w[1].w, sc0);
          q[4] = dq_fp8_8(w[NW - 2].x, w[NW - 2].y, sc1);
          q[5] = dq_fp8_8(w[NW - 2].z, w[NW - 2].w, sc1);
          q[6] = dq_fp8_8(w[NW - 1].x, w[NW - 1].y, sc1);
          q[7] = dq_fp8_8(w[NW - 1].z, w[NW - 1].w, sc1);
        }
        if (!mbar_wait(&sh.empty[s], ph ^ 1u, abort)) {
          fail(sh, a.status, 13);
          ok = false;
          break;
        }
        const uint32_t row_addr = b_smem + s * B_BYTES + j * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) sts_v4(row_addr + ((c ^ (j & 7)) << 4), q[c]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.full[s]);
      }
      if (!ok) break;
      smax_cur = byte_max(nm);
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int quarter = warp & 3;          // TMEM lanes 32 * quarter ...
    const int r = quarter * 32 + lane;     // tile row of this thread
    uint32_t lt = 0;
    for (int t = blockIdx.x; t < total && !*abort; t += gridDim.x, ++lt) {
      const uint32_t acc = lt & 1u, acc_ph = (lt >> 1) & 1u;
      const int row = a.plan.mtiles[2 * (t / n_tiles_n) + 1] + r;
      const int nt = t % n_tiles_n;
      // MXFP4: column factors of this tile and the row's 2^-k
      const uint8_t* cx = sh.colx[lt % CF_SETS];
      float rinv = 1.0f;
      if (FMT == kFmtMxfp4) {
        rinv = 1.0f / a.ascale[row];
        if (!mbar_wait(&sh.colf_full[lt % CF_SETS], (lt / CF_SETS) & 1u, abort)) {
          fail(sh, a.status, 15);
          break;
        }
      }
      if (!mbar_wait(&sh.tmem_full[acc], acc_ph, abort)) {
        fail(sh, a.status, 14);
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem + acc * BN + (uint32_t(quarter * 32) << 16);
      if (KIND == 0) {
        uint16_t* dst = a.out + int64_t(row) * a.I + nt * (BN / 2);
        float amax = 0.0f;
#pragma unroll 1
        for (int jc = 0; jc < 4; ++jc) {
          uint32_t g[32], u[32];
          tmem_ld_32cols(taddr + jc * 32, g);
          tmem_ld_32cols(taddr + BN / 2 + jc * 32, u);
          tmem_ld_wait();
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float gf0 = __uint_as_float(g[2 * i]), gf1 = __uint_as_float(g[2 * i + 1]);
            float uf0 = __uint_as_float(u[2 * i]), uf1 = __uint_as_float(u[2 * i + 1]);
            if (FMT == kFmtMxfp4) {
              const int c = jc * 32 + 2 * i;
              gf0 = gf0 * e8m0_to_f32(cx[c]) * rinv;
              gf1 = gf1 * e8m0_to_f32(cx[c + 1]) * rinv;
              uf0 = uf0 * e8m0_to_f32(cx[BN / 2 + c]) * rinv;
              uf1 = uf1 * e8m0_to_f32(cx[BN / 2 + c + 1]) * rinv;
            }
            // the MLX path rounds the gate/up product to bf16 before the activation
            const float a0 = swiglu_f32(bf16_round(gf0), bf16_round(uf0), a.limit);
            const float a1 = swiglu_f32(bf16_round(gf1), bf16_round(uf1), a.limit);
            pk[i] = pack_bf16x2(a0, a1);
            amax = fmaxf(amax, fmaxf(fabsf(bf16_round(a0)), fabsf(bf16_round(a1))));
          }
          stg_v8(dst + jc * 32, pk);  // 64 bytes of the row: two full sectors
          stg_v8(dst + jc * 32 + 16, pk + 8);
        }
        if (a.rowmax != nullptr) atomicMax(a.rowmax + row, __float_as_uint(amax));
      } else {
        uint16_t* dst = a.out + int64_t(row) * a.N + nt * BN;
        if (a.ret.rows[0] != nullptr) {  // expert-parallel owner: straight into the sender's back block
          const int slot = a.plan.row_token[row];
          dst = slot < 0 ? nullptr
                         : a.ret.rows[slot / a.ret.capacity] + int64_t(slot % a.ret.capacity) * a.N + nt * BN;
        }
#pragma unroll 1
        for (int jc = 0; jc < 8; ++jc) {
          uint32_t v[32];
          tmem_ld_32cols(taddr + jc * 32, v);
          tmem_ld_wait();
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float v0 = __uint_as_float(v[2 * i]), v1 = __uint_as_float(v[2 * i + 1]);
            if (FMT == kFmtMxfp4) {
              v0 = v0 * e8m0_to_f32(cx[jc * 32 + 2 * i]) * rinv;
              v1 = v1 * e8m0_to_f32(cx[jc * 32 + 2 * i + 1]) * rinv;
            }
            pk[i] = pack_bf16x2(v0, v1);
          }
          if (dst != nullptr) {
            stg_v8(dst + jc * 32, pk);
            stg_v8(dst + jc * 32 + 16, pk + 8);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.tmem_empty[acc]);
    }
    // rows stored into other GPUs' memory: one system-scope fence per thread
    // after its last store, before the next kernel raises the flags
    if (KIND == 1 && a.ret.rows[0] != nullptr) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

namespace {

template <int FMT, int KIND>
void set_attr() {
  cudaFuncSetAttribute(gemm_kernel<FMT, KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
}

}  // namespace

void gemm_init_attributes() {
  set_attr<kFmtMxfp4, 0>();
  set_attr<kFmtMxfp4, 1>();
  set_attr<kFmtFp8B128, 0>();
  set_attr<kFmtFp8B128, 1>();
  set_attr<kFmtFp8B32, 0>();
  set_attr<kFmtFp8B32, 1>();
}

bool gemm_shape_ok(int H, int I) { return H % BN == 0 && I % (BN / 2) == 0 && H % BK == 0 && I % BK == 0; }

void launch_gemm(const GemmArgs& a, int kind, const void* tmap_host, int num_sms, cudaStream_t stream) {
  const CUtensorMap& tm = *static_cast<const CUtensorMap*>(tmap_host);
  const dim3 grid(num_sms), block(NUM_THREADS);
  if (a.fmt == kFmtMxfp4) {
    if (kind == 0)
      gemm_kernel<kFmtMxfp4, 0><<<grid, block, SMEM_BYTES, stream>>>(tm, a);
    else
      gemm_kernel<kFmtMxfp4, 1><<<grid, block, SMEM_BYTES, stream>>>(tm, a);
  } else if (a.fmt == kFmtFp8B32) {
    if (kind == 0)
      gemm_kernel<kFmtFp8B32, 0><<<grid, block, SMEM_BYTES, stream>>>(tm, a);
    else
      gemm_kernel<kFmtFp8B32, 1><<<grid, block, SMEM_BYTES, stream>>>(tm, a);
  } else {
    if (kind == 0)
      gemm_kernel<kFmtFp8B128, 0><<<grid, block, SMEM_BYTES, stream>>>(tm, a);
    else
      gemm_kernel<kFmtFp8B128, 1><<<grid, block, SMEM_BYTES, stream>>>(tm, a);
  }
}

}  // namespace wm
