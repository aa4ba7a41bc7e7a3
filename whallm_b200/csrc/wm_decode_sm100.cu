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
// Per weight value the producers spend one hardware E2M1 -> f16x2 conversion
// per pair and one f16x2 multiply per pair: about one instruction per weight,
// which keeps the path bound by HBM rather than by instruction issue.  Every
// operand reaches shared memory by TMA (packed nibbles, the item's E8M0 tile,
// the f16 activation tile), so no thread waits on a global load in the loop.
//
// Warp roles (608 threads, one persistent CTA per SM):
//   warp 0      TMA: per item the E8M0 scale tile (2-slot ring), per K block
//               the raw packed-nibble tile (128 rows x 32 bytes, 16-deep ring)
//   warp 1      TMEM allocator and the MMA-issuing thread
//   warp 2      TMA: the f16 activation tile (16 rows x 64 K, 128-byte
//               swizzle) into its own 16-deep ring, far ahead of the MMA
//   warps 3-10  weight producers: raw nibbles + E8M0 -> f16 tile, four
//               groups of two warps taking K blocks round-robin (two rows
//               per thread)
//   warps 11-18 epilogue, two groups of four, one per TMEM accumulator:
//               TMEM -> scaling -> SwiGLU (gate/up) or bf16 rows (down)
// Every mbarrier wait is bounded; a timeout reports status and unwinds.
#include <cuda.h>

#include "wm_kernels.h"

namespace wm {

namespace {

constexpr int DM = 128, DN = 16, DK = 64;
constexpr int RAW_STAGES = 16, OP_STAGES = 4, B_STAGES = 16;
constexpr int RAW_BYTES = DM * DK / 2;       // 4 KB of nibbles
constexpr int A_OP_BYTES = DM * DK * 2;      // 16 KB f16
constexpr int B_OP_BYTES = DN * DK * 2;      // 2 KB f16
constexpr int NTHREADS = 608;
constexpr int DQW0 = 3, DQW = 8, DQG = 4, EPW0 = 11;  // DQG weight-producer groups of DQW / DQG warps
static_assert(OP_STAGES >= DQG, "each producer group needs its own operand stage");
constexpr uint32_t TMEM_COLS = 32;
constexpr int XCHG_BYTES = 2 * 64 * DN * 4;  // per epilogue group: [64 rows][16 tokens] fp32
constexpr int FIXED_SMEM = OP_STAGES * A_OP_BYTES + B_STAGES * B_OP_BYTES + RAW_STAGES * RAW_BYTES + XCHG_BYTES;

struct Shared {
  uint64_t raw_full[RAW_STAGES], raw_empty[RAW_STAGES];
  uint64_t op_full[OP_STAGES], op_empty[OP_STAGES];  // f16 weight tiles
  uint64_t b_full[B_STAGES], b_empty[B_STAGES];      // f16 activation tiles
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

__device__ __forceinline__ void sts_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

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
__device__ __forceinline__ uint4 e2m1x8_f16_scaled(uint32_t w, uint32_t scale2) {
  uint32_t h0, h1, h2, h3;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3)
      : "r"(w));
  return make_uint4(hmul2(h0, scale2), hmul2(h1, scale2), hmul2(h2, scale2), hmul2(h3, scale2));
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

__device__ __forceinline__ void tmem_ld_16cols(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

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
  const uint32_t a_op = base;                             // OP_STAGES x 16 KB (1024-aligned)
  const uint32_t b_op = a_op + OP_STAGES * A_OP_BYTES;    // B_STAGES x 2 KB (1024-aligned)
  const uint32_t raw = b_op + B_STAGES * B_OP_BYTES;      // RAW_STAGES x 4 KB
  const uint32_t scl = raw + RAW_STAGES * RAW_BYTES;      // 2 x sc_bytes
  float* xchg = reinterpret_cast<float*>(gbase + (scl - base) + 2 * sc_bytes);  // [2][64][16]
  Shared& sh = *reinterpret_cast<Shared*>(reinterpret_cast<uint8_t*>(xchg) + XCHG_BYTES);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kblocks = Kdim / DK;
  const int n_mt = KIND == 0 ? (2 * a.I) / DM : a.H / DM;  // weight-row tiles per expert

  if (threadIdx.x == 0) {
    for (int s = 0; s < RAW_STAGES; ++s) {
      mbar_init(&sh.raw_full[s], 1);
      mbar_init(&sh.raw_empty[s], DQW / DQG);
    }
    for (int s = 0; s < OP_STAGES; ++s) {
      mbar_init(&sh.op_full[s], DQW / DQG);
      mbar_init(&sh.op_empty[s], 1);
    }
    for (int s = 0; s < B_STAGES; ++s) {
      mbar_init(&sh.b_full[s], 1);
      mbar_init(&sh.b_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh.tmem_full[i], 1);
      mbar_init(&sh.tmem_empty[i], 4);
      mbar_init(&sh.x_full[i], 2);
      mbar_init(&sh.x_empty[i], 2);
      mbar_init(&sh.sc_full[i], 1);
      mbar_init(&sh.sc_empty[i], DQW + 4);
    }
    sh.abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
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
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
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
            tma_load_3d(dst, tm, kb * (DK / 2), gate_base + mt * (DM / 2), z, &sh.raw_full[s]);
            tma_load_3d(dst + RAW_BYTES / 2, tm, kb * (DK / 2), up_base + mt * (DM / 2), z, &sh.raw_full[s]);
          } else {
            tma_load_3d(dst, tm, kb * (DK / 2), mt * DM, z, &sh.raw_full[s]);
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(DM, DN);
      uint32_t it = 0, lt = 0;
      for (int t = blockIdx.x; t < total && !*abort; t += gridDim.x, ++lt) {
        const uint32_t acc = lt & 1u, acc_ph = (lt >> 1) & 1u;
        if (!mbar_wait(&sh.tmem_empty[acc], acc_ph ^ 1u, abort)) {
          fail(sh, a.status, 21);
          break;
        }
        tc_fence_after();
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % OP_STAGES, sb = it % B_STAGES;
          const uint32_t ph = (it / OP_STAGES) & 1u, phb = (it / B_STAGES) & 1u;
          if (!mbar_wait(&sh.b_full[sb], phb, abort) || !mbar_wait(&sh.op_full[s], ph, abort)) {
            fail(sh, a.status, 22);
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < DK / 16; ++k) {
            const uint64_t da = umma_desc_sw128(a_op + s * A_OP_BYTES + k * 32);
            const uint64_t db = umma_desc_sw128(b_op + sb * B_OP_BYTES + k * 32);
            umma_f16(tmem + acc * DN, da, db, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&sh.op_empty[s]);
          umma_commit(&sh.b_empty[sb]);
        }
        if (!ok) break;
        umma_commit(&sh.tmem_full[acc]);
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ activation tiles (TMA)
    if (lane == 0) {
      uint32_t it = 0;
      for (int t = blockIdx.x; t < total && !*abort; t += gridDim.x) {
        const int row0 = a.plan.mtiles[2 * (t / n_mt) + 1];
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % B_STAGES;
          const uint32_t ph = (it / B_STAGES) & 1u;
          if (!mbar_wait(&sh.b_empty[s], ph ^ 1u, abort)) {
            fail(sh, a.status, 23);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&sh.b_full[s], B_OP_BYTES);
          tma_load_2d_u32(b_op + s * B_OP_BYTES, &tm_b, kb * DK, row0, &sh.b_full[s]);
        }
        if (!ok) break;
      }
    }
  } else if (warp < EPW0) {
    // ------------------------------------------------------------ weight producers
    // DQG groups of two warps take an item's K blocks round-robin, so DQG K
    // blocks are converted at once (one group's chain of waits, loads,
    // conversions and stores would otherwise pace the whole pipeline); each
    // thread converts two whole rows (r and r + 64) of its group's K block.
    const int grp = (warp - DQW0) >> 1;
    const int tid = ((warp - DQW0) & 1) * 32 + lane;  // 0..63
    uint32_t it0 = 0, lt = 0;  // global K-block counter at the item's start
    for (int t = blockIdx.x; t < total && !*abort; t += gridDim.x, ++lt) {
      const uint32_t slot = lt & 1u, sph = (lt >> 1) & 1u;
      if (!mbar_wait(&sh.sc_full[slot], sph, abort)) {
        fail(sh, a.status, 30);
        break;
      }
      const uint32_t srow0 = scl + slot * sc_bytes + tid * sc_row;
      const uint32_t srow1 = srow0 + (DM / 2) * sc_row;
      const int smax0 = int(smem_max_scale(srow0, sc_row)), smax1 = int(smem_max_scale(srow1, sc_row));
      bool ok = true;
      for (int kb = grp; kb < kblocks; kb += DQG) {
        const uint32_t it = it0 + kb;
        const int rs = it % RAW_STAGES, os = it % OP_STAGES;
        const uint32_t rph = (it / RAW_STAGES) & 1u, oph = (it / OP_STAGES) & 1u;
        if (!mbar_wait(&sh.raw_full[rs], rph, abort)) {
          fail(sh, a.status, 24);
          ok = false;
          break;
        }
        const uint32_t rsrc = raw + rs * RAW_BYTES + tid * 32;
        const uint4 n00 = lds_v4(rsrc), n01 = lds_v4(rsrc + 16);
        const uint4 n10 = lds_v4(rsrc + (DM / 2) * 32), n11 = lds_v4(rsrc + (DM / 2) * 32 + 16);
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.raw_empty[rs]);
        const int s00 = int(lds_u8(srow0 + kb * 2)), s01 = int(lds_u8(srow0 + kb * 2 + 1));
        const int s10 = int(lds_u8(srow1 + kb * 2)), s11 = int(lds_u8(srow1 + kb * 2 + 1));
        if (!mbar_wait(&sh.op_empty[os], oph ^ 1u, abort)) {
          fail(sh, a.status, 25);
          ok = false;
          break;
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int r = tid + j * (DM / 2);
          const uint4 lo = j == 0 ? n00 : n10, hi = j == 0 ? n01 : n11;
          const int sa = j == 0 ? s00 : s10, sb = j == 0 ? s01 : s11, sm = j == 0 ? smax0 : smax1;
          const uint32_t c0 = sa == 0 ? 0u : pow2_f16x2(sa - sm), c1 = sb == 0 ? 0u : pow2_f16x2(sb - sm);
          const uint32_t row_addr = a_op + os * A_OP_BYTES + r * 128;
          const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
          for (int c = 0; c < 8; ++c) sts_v4(row_addr + ((c ^ (r & 7)) << 4), e2m1x8_f16_scaled(w[c], c < 4 ? c0 : c1));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.op_full[os]);
      }
      if (!ok) break;
      it0 += kblocks;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.sc_empty[slot]);
    }
  } else {
    // ------------------------------------------------------------ epilogue (two groups)
    const int grp = (warp - EPW0) >> 2;  // handles the items of TMEM accumulator / scale slot `grp`
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;   // TMEM lane = weight row of the tile
    float* xg = xchg + grp * 64 * DN;
    uint32_t lt = 0;
    for (int t = blockIdx.x; t < total && !*abort; t += gridDim.x, ++lt) {
      if (int(lt & 1u) != grp) continue;
      const uint32_t acc = lt & 1u, ph2 = (lt >> 1) & 1u;
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
      uint32_t v[DN];
      tmem_ld_16cols(tmem + acc * DN + (uint32_t(quarter * 32) << 16), v);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.tmem_empty[acc]);
      float y[DN];
#pragma unroll
      for (int n = 0; n < DN; ++n) y[n] = n < valid ? __uint_as_float(v[n]) * (rowf / bs[n]) : 0.0f;
      if (KIND == 0) {
        // rows 64..127 hold the up projections of the features of rows 0..63;
        // they pass them to the gate rows through `xg` (bounded waits).
        if (r >= DM / 2) {
          if (!mbar_wait(&sh.x_empty[grp], ph2 ^ 1u, abort)) {
            fail(sh, a.status, 27);
            break;
          }
#pragma unroll
          for (int n = 0; n < DN; ++n) xg[(r - DM / 2) * DN + n] = y[n];
          __syncwarp();
          if (lane == 0) mbar_arrive(&sh.x_full[grp]);
          continue;
        }
        if (!mbar_wait(&sh.x_full[grp], ph2, abort)) {
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
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// Sorted f16 copy of the activation rows: out[r] = x[row_token[r]] * 2^k,
// scale[r] = 2^k (largest magnitude of the row lands in [2^14, 2^15)).
// One warp per sorted row.
__global__ void __launch_bounds__(256) gather_f16_kernel(const uint16_t* __restrict__ x, Plan p, int E, int H,
                                                         uint16_t* __restrict__ out, float* __restrict__ scale) {
  const int rows = p.offsets[E + 1];
  const int lane = threadIdx.x & 31;
  for (int r = blockIdx.x * 8 + (threadIdx.x >> 5); r < rows; r += gridDim.x * 8) {
    const int t = p.row_token[r];
    const uint4* src = reinterpret_cast<const uint4*>(x + int64_t(t < 0 ? 0 : t) * H);
    uint32_t m = 0;
    if (t >= 0)
      for (int i = lane; i < H / 8; i += 32) {
        const uint4 v = src[i];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) m = max(m, max((w[j] & 0x7fffu) << 16, w[j] & 0x7fff0000u));
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float k2 = row_prescale(m);
    uint4* dst = reinterpret_cast<uint4*>(out + int64_t(r) * H);
    for (int i = lane; i < H / 8; i += 32) {
      uint4 o = make_uint4(0, 0, 0, 0);
      if (t >= 0) {
        const uint4 v = src[i];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t q[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_bf16x2(w[j]);
          const __half2 hh = __floats2half2_rn(f.x * k2, f.y * k2);
          q[j] = *reinterpret_cast<const uint32_t*>(&hh);
        }
        o = make_uint4(q[0], q[1], q[2], q[3]);
      }
      dst[i] = o;
    }
    if (lane == 0) scale[r] = k2;
  }
}

// act16[r] = act[r] * 2^k with k from the row's largest |act| (rowmax, float bits).
__global__ void __launch_bounds__(256) act_f16_kernel(const uint16_t* __restrict__ act, Plan p, int E, int I,
                                                      uint16_t* __restrict__ out, float* __restrict__ scale) {
  const int rows = p.offsets[E + 1];
  const int lane = threadIdx.x & 31;
  for (int r = blockIdx.x * 8 + (threadIdx.x >> 5); r < rows; r += gridDim.x * 8) {
    const float k2 = row_prescale(p.rowmax[r]);
    const uint4* src = reinterpret_cast<const uint4*>(act + int64_t(r) * I);
    uint4* dst = reinterpret_cast<uint4*>(out + int64_t(r) * I);
    for (int i = lane; i < I / 8; i += 32) {
      const uint4 v = src[i];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      uint32_t q[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(w[j]);
        const __half2 hh = __floats2half2_rn(f.x * k2, f.y * k2);
        q[j] = *reinterpret_cast<const uint32_t*>(&hh);
      }
      dst[i] = make_uint4(q[0], q[1], q[2], q[3]);
    }
    if (lane == 0) scale[r] = k2;
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
  gather_f16_kernel<<<num_sms * 4, 256, 0, stream>>>(x, p, E, H, out, scale);
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
