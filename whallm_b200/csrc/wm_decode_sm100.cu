// Decode path on the tensor cores: for each expert with rows, Y^T = W_e X_e^T
// with the expert's weights as the M = 128 operand and its (at most 16 per
// item) token rows as N = 16 ("swap-AB"), tcgen05.mma kind::f16 with f16
// operands and fp32 accumulators in TMEM.
//
// Reference arithmetic: the decode GEMVs expert_linear4 / expert_group<R, K>
// (QwenNative/kernels.metal:1186-1219, DeepSeekNative/kernels.metal:933-987)
// and mx.quantized_matmul(mode="mxfp4") (model.py:504-513): exact dequantised
// weights times the activation rows, fp32 accumulation.  Exactness of the
// f16 operands:
//   * weight = E2M1 * 2^(s - 127).  Each 128-row tile row r gets the factor
//     2^(smax_r - 127) (smax_r = the row's largest E8M0 byte) in the epilogue,
//     so the operand is E2M1 * 2^(s - smax_r) <= 6: exact in f16 for every
//     group within 23 binades of the row's largest (smaller groups, if any,
//     would round -- their weight is below 2^-23 of the row's largest).
//   * activation rows (bf16) are multiplied by 2^k, k chosen from the row's
//     largest magnitude so it lands in [2^14, 2^15): exact in f16 for every
//     element within 2^-24 of the row's largest; the epilogue divides by 2^k.
// So the MMA sums the same products as the reference, in fp32.
//
// The weight operand goes to the tensor cores through TMEM: the producers
// convert nibbles to f16 in registers (one hardware E2M1 -> f16x2 conversion
// and one f16x2 multiply per pair, about one instruction per weight) and
// store them with tcgen05.st; the MMA reads A from TMEM ("[a-tmem]" form).
// Every other operand reaches shared memory by TMA (packed nibbles, the
// item's E8M0 tile, the f16 activation tile), so no thread waits on a global
// load.  At N = 16 an MMA moves little data, so the kernel is bound by how
// fast tiles, MMAs and barrier round trips flow: MMAs are issued by
// converged warps through elect.sync, two warps split the K blocks, and the
// weight and activation tiles of a K block complete on one barrier.
//
// Warp roles (one persistent CTA per SM):
//   warp 0      TMA: per item the E8M0 scale tile (2-slot ring); per 4 K
//               blocks the packed nibbles (128 rows x 128 bytes)
//   warps 1, 3  MMA issue, even / odd K blocks (warp 1 also owns TMEM)
//   warp 2      TMA: the f16 activation tile (16 rows x 64 K, 128-byte swizzle)
//   warps 4-19  weight producers: four groups of four warps (one per TMEM
//               lane quarter), K blocks round-robin; a thread converts its row
//   warps 20-23 epilogue: TMEM -> scaling -> SwiGLU (gate/up) or bf16 rows
//               (down), accumulator sets alternating between items
// Every mbarrier wait is bounded; a timeout reports status and unwinds.
#include <cuda.h>

#include "wm_kernels.h"

namespace wm {

namespace {

constexpr int DM = 128, DN = 16, DK = 64;
// A stage = one K block: the f16 weight tile (TMEM) and the f16 activation
// tile (shared memory), completed on one barrier.  A raw stage = RAW_KB K
// blocks of packed nibbles, 128 rows x 128 bytes with the 128-byte swizzle:
// the TMA engine's cost grows with the rows of a box, so long rows keep it
// ahead of HBM, and the swizzle keeps the producers' 16-byte reads of eight
// consecutive rows on distinct banks.
constexpr int RAW_KB = 4, RAW_STAGES = 6, A_STAGES = 8;
constexpr int RAW_ROW = DK * RAW_KB / 2;     // 128 bytes
constexpr int RAW_BYTES = DM * RAW_ROW;      // 16 KB of nibbles
constexpr int B_OP_BYTES = DN * DK * 2;      // 2 KB f16
constexpr int MMA_WARP0 = 1, MMA_WARP1 = 3;  // issue the even / the odd K blocks
// Weight producers: DQG groups of four warps (one per TMEM lane quarter)
// taking K blocks round-robin.  A group's step is a chain of barrier round
// trips, shared loads and the TMEM store that is long next to its ~100 cycles
// of conversion work, so several groups keep chains in flight at once.
constexpr int DQG = 4, DQ_WARPS = 4;
static_assert(8 % DQG == 0, "a group's K blocks take the same 16-byte scale chunk in turn");
static_assert(RAW_ROW == 128, "one swizzle atom row per weight row");
constexpr int DQW0 = 4, DQW = DQG * DQ_WARPS;
constexpr int EPG = 1;                       // epilogue groups of four warps
constexpr int EPW0 = DQW0 + DQW;
constexpr int NTHREADS = 32 * (EPW0 + 4 * EPG);
static_assert(DQW0 % 4 == 0 && EPW0 % 4 == 0, "a group's warp w serves TMEM lane quarter w % 4");
// An item's K steps rotate over NACC accumulators of DN columns: consecutive
// MMAs into one accumulator wait for each other, and at N = 16 that latency,
// not the tensor pipe, would pace the kernel.  The epilogue sums them.
constexpr int NACC = 8;
constexpr uint32_t ACC_COLS = NACC * DN;     // one accumulator set (of two)
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t A_COL0 = 2 * ACC_COLS;    // A stages: 32 columns (64 f16 per lane) each
static_assert(A_COL0 + A_STAGES * 32 <= TMEM_COLS, "TMEM layout");
static_assert((DK / 16) * 2 == NACC, "an even and an odd K block cover the accumulators once");
static_assert(A_STAGES % DQG == 0 && DQG % 2 == 0, "an A stage always belongs to the same producer group and MMA warp");
constexpr int XCHG_BYTES = EPG * 64 * DN * 4;  // per epilogue group: [64 rows][16 tokens] fp32
constexpr int FIXED_SMEM = A_STAGES * B_OP_BYTES + RAW_STAGES * RAW_BYTES + XCHG_BYTES;

struct Shared {
  uint64_t raw_full[RAW_STAGES], raw_empty[RAW_STAGES];
  uint64_t a_full[A_STAGES], a_empty[A_STAGES];  // f16 weight (TMEM) + activation (smem) tiles
  uint64_t tmem_full[2], tmem_empty[2];
  uint64_t x_full[2], x_empty[2];    // gate/up exchange inside each epilogue group
  uint64_t sc_full[2], sc_empty[2];  // the items' E8M0 tiles
  uint32_t tmem_base;
  int abort;
};

// Dynamic shared memory of one launch: fixed rings + two scale slots of
// 128 rows x Kdim/32 bytes + alignment slack + barriers.
size_t smem_bytes(int kdim) { return size_t(FIXED_SMEM) + 2 * size_t(DM) * (kdim / 32) + 1024 + 1024; }
static_assert(sizeof(Shared) <= 1024, "barrier block must fit its reserve");

__device__ __forceinline__ uint4 lds_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ uint32_t lds_u8(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// 8 E2M1 nibbles of `w` (element j = nibble j) times the f16x2 scale -> 4 f16x2.
__device__ __forceinline__ void e2m1x8_f16_scaled(uint32_t w, uint32_t scale2, uint32_t* out) {
  uint32_t h0, h1, h2, h3;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3)
      : "r"(w));
  out[0] = hmul2(h0, scale2);
  out[1] = hmul2(h1, scale2);
  out[2] = hmul2(h2, scale2);
  out[3] = hmul2(h3, scale2);
}

// f16x2 holding 2^d twice (d <= 0; below f16's range -> 0).
__device__ __forceinline__ uint32_t pow2_f16x2(int d) {
  uint32_t h;
  if (d >= -14)
    h = uint32_t(15 + d) << 10;  // normal
  else if (d >= -24)
    h = 1u << (d + 24);          // subnormal
  else
    h = 0u;
  return h | (h << 16);
}

// Largest E8M0 byte of `n` bytes in shared memory (n multiple of 16).
__device__ __forceinline__ uint32_t smem_max_scale(uint32_t addr, int n) {
  uint32_t m = 0;
  for (int i = 0; i < n; i += 16) {
    const uint4 v = lds_v4(addr + i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      m = max(m, w[j] & 0xffu);
      m = max(m, (w[j] >> 8) & 0xffu);
      m = max(m, (w[j] >> 16) & 0xffu);
      m = max(m, w[j] >> 24);
    }
  }
  return m;
}

// 2^k for a row whose largest magnitude has float bits `maxbits`: the scaled
// row's largest element lands in [2^14, 2^15).
__device__ __forceinline__ float row_prescale(uint32_t maxbits) {
  if (maxbits == 0u || maxbits >= 0x7f800000u) return 1.0f;
  const int e = int(maxbits >> 23) - 127;  // floor(log2(max)) for normal values
  const int k = min(max(14 - e, -100), 100);
  return exp2f(float(k));
}

__device__ __forceinline__ void fail(Shared& sh, uint32_t* status, uint32_t role) {
  report_status(status, kStatusWaitTimeout, role);
  sh.abort = 1;
}

// 3-D TMA load (x = bytes along the row, y = row, z = expert) completing on bar.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dst),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_2d_u32(uint32_t dst, const void* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 32 consecutive TMEM columns of this warp's 32 lanes <- 32 registers per thread.
__device__ __forceinline__ void tmem_st_32cols(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// 16 consecutive TMEM columns of this warp's 32 lanes <- 16 registers per thread.
__device__ __forceinline__ void tmem_st_16cols(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// kind::f16 instruction descriptor: f16 A and B, fp32 D, K-major, M x N.
constexpr uint32_t idesc_f16(uint32_t M, uint32_t N) { return (1u << 4) | ((N >> 3) << 17) | ((M >> 4) << 24); }

}  // namespace

// KIND 0: gate/up (+SwiGLU) -> act [rows, I] bf16 and per-row |act| maxima;
// KIND 1: down -> routed [rows, H] bf16.
// tm_w / tm_sh: packed weights of the routed / shared experts; tm_s / tm_ssh:
// their E8M0 scales; tm_b: the f16 activation rows.
template <int KIND>
__global__ void __launch_bounds__(NTHREADS, 1)
    decode_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_sh,
                  const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_ssh,
                  const __grid_constant__ CUtensorMap tm_b, const DecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const int Kdim = KIND == 0 ? a.H : a.I;
  const int sc_row = Kdim / 32;                // E8M0 bytes per weight row
  const int sc_bytes = DM * sc_row;            // one scale slot
  const uint32_t raw0 = smem_u32(smem_raw);
  const uint32_t base = (raw0 + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw0);
  const uint32_t b_op = base;                             // A_STAGES x 2 KB (1024-aligned)
  const uint32_t raw = b_op + A_STAGES * B_OP_BYTES;      // RAW_STAGES x 16 KB (1024-aligned)
  const uint32_t scl = raw + RAW_STAGES * RAW_BYTES;      // 2 x sc_bytes
  float* xchg = reinterpret_cast<float*>(gbase + (scl - base) + 2 * sc_bytes);  // [EPG][64][16]
  Shared& sh = *reinterpret_cast<Shared*>(reinterpret_cast<uint8_t*>(xchg) + XCHG_BYTES);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kblocks = Kdim / DK;
  const int n_mt = KIND == 0 ? (2 * a.I) / DM : a.H / DM;  // weight-row tiles per expert

  if (threadIdx.x == 0) {
    for (int s = 0; s < RAW_STAGES; ++s) {
      mbar_init(&sh.raw_full[s], 1);
      mbar_init(&sh.raw_empty[s], RAW_KB * DQ_WARPS);  // each of its K blocks: one group
    }
    for (int s = 0; s < A_STAGES; ++s) {
      mbar_init(&sh.a_full[s], DQ_WARPS + 1);  // the group's producer warps + the activation TMA
      mbar_init(&sh.a_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh.tmem_full[i], 2);   // both MMA warps

      mbar_init(&sh.tmem_empty[i], 4);
      mbar_init(&sh.x_full[i], 2);
      mbar_init(&sh.x_empty[i], 2);
      mbar_init(&sh.sc_full[i], 1);
      mbar_init(&sh.sc_empty[i], DQW + 4 * EPG);
    }
    sh.abort = 0;
    fence_mbarrier_init();
  }
  if (warp == MMA_WARP0) {
    tmem_alloc(&sh.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_sh);
    tma_prefetch_desc(&tm_s);
    tma_prefetch_desc(&tm_ssh);
    tma_prefetch_desc(&tm_b);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  volatile int* abort = &sh.abort;
  const int total = *a.plan.n_mtiles * n_mt;
  const int E = a.wts.E;
  const int gate_base = a.gate_first ? 0 : a.I, up_base = a.gate_first ? a.I : 0;

  if (warp == 0) {
    // ------------------------------------------------------------ scale tiles + raw weight tiles (TMA)
    if (lane == 0) {
      uint32_t it = 0, lt = 0;
      for (int t = blockIdx.x; t < total && !*abort; t += gridDim.x, ++lt) {
        const int e = a.plan.mtiles[2 * (t / n_mt)];
        const int mt = t % n_mt;
        const bool routed = e < E;
        const int z = routed ? e : 0;
        const uint32_t slot = lt & 1u, sph = (lt >> 1) & 1u;
        if (!mbar_wait(&sh.sc_empty[slot], sph ^ 1u, abort)) {
          fail(sh, a.status, 29);
          break;
        }
        mbar_arrive_expect_tx(&sh.sc_full[slot], uint32_t(sc_bytes));
        const uint32_t sdst = scl + slot * sc_bytes;
        const CUtensorMap* ts = routed ? &tm_s : &tm_ssh;
        if (KIND == 0) {
          tma_load_3d(sdst, ts, 0, gate_base + mt * (DM / 2), z, &sh.sc_full[slot]);
          tma_load_3d(sdst + sc_bytes / 2, ts, 0, up_base + mt * (DM / 2), z, &sh.sc_full[slot]);
        } else {
          tma_load_3d(sdst, ts, 0, mt * DM, z, &sh.sc_full[slot]);
        }
        const CUtensorMap* tm = routed ? &tm_w : &tm_sh;
        bool ok = true;
        for (int kq = 0; kq < kblocks / RAW_KB; ++kq, ++it) {
          const int s = it % RAW_STAGES;
          const uint32_t ph = (it / RAW_STAGES) & 1u;
          if (!mbar_wait(&sh.raw_empty[s], ph ^ 1u, abort)) {
            fail(sh, a.status, 20);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&sh.raw_full[s], RAW_BYTES);
          const uint32_t dst = raw + s * RAW_BYTES;
          if (KIND == 0) {
            tma_load_3d(dst, tm, kq * RAW_ROW, gate_base + mt * (DM / 2), z, &sh.raw_full[s]);
            tma_load_3d(dst + RAW_BYTES / 2, tm, kq * RAW_ROW, up_base + mt * (DM / 2), z, &sh.raw_full[s]);
          } else {
            tma_load_3d(dst, tm, kq * RAW_ROW, mt * DM, z, &sh.raw_full[s]);
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == MMA_WARP0 || warp == MMA_WARP1) {
    // ------------------------------------------------------------ MMA issuers
    // Two warps, one for the even and one for the odd K blocks of each item
    // (accumulators 0-3 and 4-7): a warp's issue loop is latency-bound, two
    // of them keep the tensor pipe twice as busy.  The whole warp runs the
    // loop (its waits are warp-uniform) and one elected lane issues.
    const int par = warp == MMA_WARP0 ? 0 : 1;
    constexpr uint32_t idesc = idesc_f16(DM, DN);
    uint32_t it0 = 0, lt = 0;
    for (int t = blockIdx.x; t < total && !warp_aborted(abort); t += gridDim.x, ++lt) {
      const uint32_t acc = lt & 1u, acc_ph = (lt >> 1) & 1u;
      if (!warp_wait(&sh.tmem_empty[acc], acc_ph ^ 1u, abort)) {
        if (lane == 0) fail(sh, a.status, 21);
        break;
      }
      tc_fence_after();
      const uint32_t d0 = tmem + acc * ACC_COLS + par * (DK / 16) * DN;
      bool ok = true;
      for (int kb = par; kb < kblocks; kb += 2) {
        const uint32_t it = it0 + kb;
        const int s = it % A_STAGES;
        if (!warp_wait(&sh.a_full[s], (it / A_STAGES) & 1u, abort)) {
          if (lane == 0) fail(sh, a.status, 22);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = tmem + A_COL0 + s * 32;
        const uint64_t b0 = umma_desc_sw128(b_op + s * B_OP_BYTES);
        const uint32_t accumulate = kb >= 2 ? 1u : 0u;
#pragma unroll
        for (int k = 0; k < DK / 16; ++k)  // K16 step: 8 TMEM columns of A, 32 bytes (2 in the descriptor) of B
          umma_f16_ts_elect(d0 + k * DN, a0 + k * 8, b0 + 2 * k, idesc, accumulate);
        umma_commit_elect(&sh.a_empty[s]);
      }
      if (!ok) break;
      umma_commit_elect(&sh.tmem_full[acc]);
      it0 += kblocks;
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ activation tiles (TMA)
    if (lane == 0) {
      uint32_t it = 0;
      for (int t = blockIdx.x; t < total && !*abort; t += gridDim.x) {
        const int row0 = a.plan.mtiles[2 * (t / n_mt) + 1];
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % A_STAGES;
          const uint32_t ph = (it / A_STAGES) & 1u;
          if (!mbar_wait(&sh.a_empty[s], ph ^ 1u, abort)) {
            fail(sh, a.status, 23);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&sh.a_full[s], B_OP_BYTES);
          tma_load_2d_u32(b_op + s * B_OP_BYTES, &tm_b, kb * DK, row0, &sh.a_full[s]);
        }
        if (!ok) break;
      }
    }
  } else if (warp < EPW0) {
    // ------------------------------------------------------------ weight producers
    // DQG groups take an item's K blocks round-robin; warp w of a group
    // serves TMEM lane quarter w % 4, one weight row per thread.
    const int grp = (warp - DQW0) / DQ_WARPS;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // tile row
    uint32_t it0 = 0, lt = 0;           // global K-block counter at the item's start
    for (int t = blockIdx.x; t < total && !warp_aborted(abort); t += gridDim.x, ++lt) {
      const uint32_t slot = lt & 1u, sph = (lt >> 1) & 1u;
      if (!warp_wait(&sh.sc_full[slot], sph, abort)) {
        if (lane == 0) fail(sh, a.status, 30);
        break;
      }
      const uint32_t srow = scl + slot * sc_bytes + r * sc_row;
      const int smax = int(smem_max_scale(srow, sc_row));
      bool ok = true;
      uint4 sq = make_uint4(0u, 0u, 0u, 0u);
      for (int kb = grp; kb < kblocks; kb += DQG) {
        const uint32_t it = it0 + kb, rit = it / RAW_KB;
        const int rs = rit % RAW_STAGES, as = it % A_STAGES;
        const uint32_t rph = (rit / RAW_STAGES) & 1u, aph = (it / A_STAGES) & 1u;
        // The scale tile is resident: take this block's two E8M0 bytes before
        // waiting for the nibbles.  Rows are Kdim/32 bytes apart, so a warp's
        // byte loads would share two banks; one 16-byte load per row serves
        // eight K blocks instead.
        if (kb % 8 < DQG) sq = lds_v4(srow + (kb / 8) * 16);
        const int wi = (kb % 8) >> 1;
        const uint32_t word = wi == 0 ? sq.x : wi == 1 ? sq.y : wi == 2 ? sq.z : sq.w;
        const uint32_t pair = (kb & 1) ? (word >> 16) : (word & 0xffffu);
        const int s0 = int(pair & 0xffu), s1 = int(pair >> 8);
        const uint32_t c0 = s0 == 0 ? 0u : pow2_f16x2(s0 - smax), c1 = s1 == 0 ? 0u : pow2_f16x2(s1 - smax);
        if (!warp_wait(&sh.raw_full[rs], rph, abort)) {
          if (lane == 0) fail(sh, a.status, 24);
          ok = false;
          break;
        }
        // 32 bytes = 64 E2M1 = the row's two scale groups of this K block:
        // 16-byte chunks 2j, 2j+1 of the row, swizzled by row % 8
        const uint32_t rrow = raw + rs * RAW_BYTES + r * RAW_ROW;
        const uint32_t j2 = uint32_t(kb % RAW_KB) * 2u;
        const uint4 lo = lds_v4(rrow + ((j2 ^ uint32_t(r & 7)) << 4));
        const uint4 hi = lds_v4(rrow + (((j2 + 1u) ^ uint32_t(r & 7)) << 4));
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.raw_empty[rs]);
        uint32_t v[32];
        e2m1x8_f16_scaled(lo.x, c0, v + 0);
        e2m1x8_f16_scaled(lo.y, c0, v + 4);
        e2m1x8_f16_scaled(lo.z, c0, v + 8);
        e2m1x8_f16_scaled(lo.w, c0, v + 12);
        e2m1x8_f16_scaled(hi.x, c1, v + 16);
        e2m1x8_f16_scaled(hi.y, c1, v + 20);
        e2m1x8_f16_scaled(hi.z, c1, v + 24);
        e2m1x8_f16_scaled(hi.w, c1, v + 28);
        if (!warp_wait(&sh.a_empty[as], aph ^ 1u, abort)) {
          if (lane == 0) fail(sh, a.status, 25);
          ok = false;
          break;
        }
        tc_fence_after();
        tmem_st_32cols(tmem + A_COL0 + as * 32 + (uint32_t(quarter * 32) << 16), v);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.a_full[as]);
      }
      if (!ok) break;
      it0 += kblocks;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.sc_empty[slot]);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int grp = (warp - EPW0) >> 2;  // handles items lt with lt % EPG == grp
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;   // TMEM lane = weight row of the tile
    float* xg = xchg + grp * 64 * DN;
    uint32_t lt = 0;
    for (int t = blockIdx.x; t < total && !*abort; t += gridDim.x, ++lt) {
      if (int(lt % EPG) != grp) continue;
      const uint32_t acc = lt & 1u, ph2 = (lt >> 1) & 1u, xph = (lt / EPG) & 1u;
      const int ent = t / n_mt;
      const int e = a.plan.mtiles[2 * ent], row0 = a.plan.mtiles[2 * ent + 1];
      const int mt = t % n_mt;
      const int valid = min(DN, a.plan.counts[e] - (row0 - a.plan.offsets[e]));
      float bs[DN];
#pragma unroll
      for (int n = 0; n < DN; ++n) bs[n] = n < valid ? a.bscale[row0 + n] : 1.0f;
      if (!mbar_wait(&sh.sc_full[acc], ph2, abort)) {
        fail(sh, a.status, 31);
        break;
      }
      const float rowf = e8m0_to_f32(smem_max_scale(scl + acc * sc_bytes + r * sc_row, sc_row));
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.sc_empty[acc]);
      if (!mbar_wait(&sh.tmem_full[acc], ph2, abort)) {
        fail(sh, a.status, 26);
        break;
      }
      tc_fence_after();
      float y[DN];
#pragma unroll
      for (int n = 0; n < DN; ++n) y[n] = 0.0f;
#pragma unroll
      for (int c = 0; c < NACC; c += 2) {
        uint32_t v[2 * DN];
        tmem_ld_32cols(tmem + acc * ACC_COLS + c * DN + (uint32_t(quarter * 32) << 16), v);
        tmem_ld_wait();
#pragma unroll
        for (int n = 0; n < DN; ++n) y[n] += __uint_as_float(v[n]) + __uint_as_float(v[DN + n]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.tmem_empty[acc]);
#pragma unroll
      for (int n = 0; n < DN; ++n) y[n] = n < valid ? y[n] * (rowf / bs[n]) : 0.0f;
      if (KIND == 0) {
        // rows 64..127 hold the up projections of the features of rows 0..63;
        // they pass them to the gate rows through `xg` (bounded waits).
        if (r >= DM / 2) {
          if (!mbar_wait(&sh.x_empty[grp], xph ^ 1u, abort)) {
            fail(sh, a.status, 27);
            break;
          }
#pragma unroll
          for (int n = 0; n < DN; ++n) xg[(r - DM / 2) * DN + n] = y[n];
          __syncwarp();
          if (lane == 0) mbar_arrive(&sh.x_full[grp]);
          continue;
        }
        if (!mbar_wait(&sh.x_full[grp], xph, abort)) {
          fail(sh, a.status, 28);
          break;
        }
        const int f = mt * (DM / 2) + r;
#pragma unroll
        for (int n = 0; n < DN; ++n) {
          if (n < valid) {
            // the MLX path rounds the gate/up product to bf16 before the activation
            const float g = bf16_round(y[n]), u = bf16_round(xg[r * DN + n]);
            const uint16_t bits = f32_to_bf16_bits(swiglu_f32(g, u, a.limit));
            a.act[int64_t(row0 + n) * a.I + f] = bits;
            float m = fabsf(bf16_bits_to_f32(bits));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == 0) atomicMax(a.plan.rowmax + row0 + n, __float_as_uint(m));
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.x_empty[grp]);
      } else {
        const int hcol = mt * DM + r;
#pragma unroll
        for (int n = 0; n < DN; ++n)
          if (n < valid) a.routed[int64_t(row0 + n) * a.H + hcol] = f32_to_bf16_bits(y[n]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
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

void decode_init_attributes() {
  const int s = int(smem_bytes(7168));
  cudaFuncSetAttribute(decode_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, s);
  cudaFuncSetAttribute(decode_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, s);
}

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

void launch_decode(const DecodeArgs& a, int kind, const void* const* maps, int num_sms, cudaStream_t stream) {
  const CUtensorMap& w = *static_cast<const CUtensorMap*>(maps[0]);
  const CUtensorMap& ws = *static_cast<const CUtensorMap*>(maps[1]);
  const CUtensorMap& s = *static_cast<const CUtensorMap*>(maps[2]);
  const CUtensorMap& ss = *static_cast<const CUtensorMap*>(maps[3]);
  const CUtensorMap& b = *static_cast<const CUtensorMap*>(maps[4]);
  if (kind == 0)
    decode_kernel<0><<<num_sms, NTHREADS, smem_bytes(a.H), stream>>>(w, ws, s, ss, b, a);
  else
    decode_kernel<1><<<num_sms, NTHREADS, smem_bytes(a.I), stream>>>(w, ws, s, ss, b, a);
}

}  // namespace wm
