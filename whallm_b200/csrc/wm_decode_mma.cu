// Decode path, register-direct: every warp streams its own weight rows with
// 16-byte loads, dequantises the E2M1 nibbles in registers straight into the
// A fragments of mma.sync.m16n8k16 (f16 x f16 -> fp32), and multiplies them
// by the (at most 8) token rows of its item, the N = 8 operand.  No weight
// byte passes through shared memory or TMEM and no warp waits on another
// warp inside an item, so the loads of many warps stay in flight at once and
// HBM, not a chain of hand-offs, sets the pace.
//
// Reference arithmetic: the decode GEMVs expert_linear4 / expert_group<R, K>
// (QwenNative/kernels.metal:1186-1219, DeepSeekNative/kernels.metal:933-987)
// and mx.quantized_matmul(mode="mxfp4") (model.py:504-513): exact dequantised
// weights times the activation rows, fp32 accumulation.  The f16 operands are
// exact, as in the tcgen05 decode kernel:
//   * weight = E2M1 * 2^(s - smax_r) with smax_r the row's largest E8M0 byte
//     (<= 6: exact in f16 for every group within 23 binades of the row's
//     largest); the epilogue applies 2^(smax_r - 127);
//   * activation rows are the f16 copies of gather_f16 / act_f16, scaled by
//     2^k per row; the epilogue divides by 2^k.
//
// Work: an item is (8-token tile of one expert, block of weight rows).  A CTA
// of 16 warps takes one item at a time; warp w owns 32 of its weight rows
// (two 16-row MMA tiles).  For gate/up a 16-row tile is 8 gate rows and the
// 8 up rows of the same features, so SwiGLU runs on the accumulators.  The
// item's f16 token tile (TMA, 128-byte swizzle) and its E8M0 scale block (one
// or two bulk copies) land in shared memory, double-buffered (one buffer when
// a CTA gets a single item or the tile is large); the warp that finishes an
// item last refills that buffer for the item after next.  The weight loads
// run kStages chunks ahead across item boundaries; the metadata of the next
// items is read an item early, so no load waits on another.
//
// FP8 experts (E4M3 with 128 x 128 fp32 or 32 x 32 UE8M0 block scales) take
// the same kernel: a lane's 16 bytes are 16 weights, each rounded to bf16
// after its fp32 scaling as the reference decodes them, into bf16 MMAs with
// the plain bf16 token rows (no prescale).
//
// Measured on B200 (config-1 decode, 64 tokens): gate/up ~100 us for 407 MB
// (4.1 TB/s), down ~62 us.  Two limits meet there: this row-striped access
// (64 bytes of each row per chunk) streams at most ~4.4 TB/s, and with the
// weight loads removed the kernel still takes ~72 us (about 1.6 issued
// instructions per weight: dequantisation, scaling, MMAs).  Deeper rings
// (3-4 chunks), two CTAs per SM, 16 rows per warp, TMA-fed shared-memory
// rings of whole 128-byte lines and L2 prefetch hints all measured slower.
//
// Per thread (lane = 4g + t): weight row g and g + 8 of each 16-row tile, and
// for chunk c (128 K) the 16 bytes at K offset 128c + 32t: 32 consecutive
// weights = exactly one scale group (4c + t).  K step j (of 8) of the chunk
// feeds MMA slots {2t, 2t+1} with K offsets 4j, 4j+1 and slots {2t+8, 2t+9}
// with 4j+2, 4j+3; the token operand uses the same K positions, so the MMA
// sums the same products as the reference in another order.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "wm_kernels.h"

namespace wm {

namespace {

constexpr int kWarps = 16;   // warps per CTA
constexpr int kCtas = 1;     // CTAs per SM (two measured slower)
constexpr int kThreads = 32 * kWarps;
constexpr int kTok = 8;      // tokens per item (the MMA's N)
constexpr int kRG = 2;       // 16-row MMA tiles per warp
constexpr int kStages = 2;   // chunks of weight loads in flight per thread
// Split K: with KS > 1 the CTA's warps form kWarps / KS row groups of KS
// warps, each warp taking 1 / KS of the K chunks of its group's rows, so an
// item covers 1 / KS of the rows and short calls (few token tiles) still
// spread over every SM.  The sums do not depend on the split: K is cut into
// q_nseg(K) segments, each summed from zero, and a row's result is
// (((0 + s_0) + s_1) + ...) in segment order.  A split warp parks its
// segment sums in shared memory; the group's first warp adds them in order
// and runs the epilogue.
__host__ __device__ constexpr int q_feat_item(int ks) { return kWarps / ks * kRG * 8; }   // gate/up features
__host__ __device__ constexpr int q_rows_item(int ks) { return kWarps / ks * kRG * 16; }  // down output rows

struct QShared {
  uint64_t full[2];
  uint64_t red_full[2][kWarps];  // per buffer and row group: the K-slice partials are in
  int done[2];  // warps finished with the buffer's item
  int abort;
};

__host__ __device__ constexpr int q_round1k(int v) { return (v + 1023) & ~1023; }

// K of a chunk: a lane's 16 bytes of a row are 32 E2M1 weights or 16 E4M3 weights.
__host__ __device__ constexpr int q_chunk_k(int fmt) { return fmt == kFmtMxfp4 ? 128 : 64; }
// Weight rows per scale row: MXFP4 one E8M0 byte per 32 K of every row; FP8
// one scale per 32 x 32 (UE8M0 byte) or 128 x 128 (fp32) block.  A scale row
// is K / 32 bytes in every format.
__host__ __device__ constexpr int q_block_rows(int fmt) { return fmt == kFmtMxfp4 ? 1 : fmt == kFmtFp8B32 ? 32 : 128; }
// Scale rows of `rows` weight rows that start on a multiple of min(rows, block).
__host__ __device__ constexpr int q_srows(int fmt, int rows) {
  return (rows + q_block_rows(fmt) - 1) / q_block_rows(fmt);
}

// Bytes of one buffer: the token tile (K/64 boxes of 8 rows x 128 B) and the scale block.
__host__ __device__ inline int q_xbytes(int K) { return kTok * K * 2; }
__host__ __device__ inline int q_sbytes(int kind, int K, int ks, int fmt) {
  return (kind == 0 ? 2 * q_srows(fmt, q_feat_item(ks)) : q_srows(fmt, q_rows_item(ks))) * (K / 32);
}
__host__ __device__ inline int q_bufbytes(int kind, int K, int ks, int fmt) {
  return q_round1k(q_xbytes(K) + q_sbytes(kind, K, ks, fmt));
}
// Segments of K: the most (up to 8, a power of two) that divide its chunks
// into whole rings of kStages chunks.  A split KS must divide it.
__host__ __device__ inline int q_nseg(int K, int fmt) {
  const int rings = K / q_chunk_k(fmt) / kStages;
  int n = 1;
  while (n < 8 && rings % (2 * n) == 0) n *= 2;
  return n;
}
// Segment sums of the K slices 1 .. KS-1: per buffer, per slice, per segment
// of the slice and per warp, 32 lanes x kRG * 4 floats.
__host__ __device__ inline int q_redbytes(int ks, int nseg, int nbuf) {
  return ks > 1 ? nbuf * (ks - 1) * (nseg / ks) * (kWarps / ks) * 32 * kRG * 16 : 0;
}

// nbuf: token-tile buffers (2: the next item's tile loads during this one)
size_t q_smem_bytes(int kind, int K, int ks, int fmt, int nbuf) {
  return size_t(nbuf) * q_bufbytes(kind, K, ks, fmt) + q_redbytes(ks, q_nseg(K, fmt), nbuf) + 1024 + sizeof(QShared) +
         16;
}

__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t lds_u8q(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ uint4 lds_v4q(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ uint32_t hmul2q(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Four E2M1 pairs of one word -> four f16x2 (pair p = byte p, low nibble in the low half).
__device__ __forceinline__ void e2m1x8_f16x2(uint32_t w, uint32_t* h) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
}

// f16x2 holding 2^(s - smax) twice, given rinv = 2^(127 - smax): the E8M0
// byte s as a float is 2^(s - 127) (0 for s = 0, the Metal convention), the
// product is exact and rounds to 0 below f16's range.
__device__ __forceinline__ uint32_t group_mult(uint32_t s, float rinv) {
  const float f = __uint_as_float(s << 23) * rinv;
  uint32_t h;
  asm("cvt.rn.f16x2.f32 %0, %1, %1;" : "=r"(h) : "f"(f));
  return h;
}

__device__ __forceinline__ void mma_f16(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16q(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tma_load_2d_q(uint32_t dst, const void* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Item -> (expert, first sorted row, valid tokens, row block).
struct QItem {
  int e, row0, valid, blk;
};

__device__ __forceinline__ QItem q_item(const DecodeArgs& a, int q, int nb) {
  QItem it;
  const int ent = q / nb;
  it.blk = q - ent * nb;
  it.e = a.plan.mtiles[2 * ent];
  it.row0 = a.plan.mtiles[2 * ent + 1];
  it.valid = min(kTok, a.plan.counts[it.e] - (it.row0 - a.plan.offsets[it.e]));
  return it;
}

}  // namespace

// KIND 0: gate/up (+SwiGLU) -> act [rows, I] bf16 (and, MXFP4, per-row |act|
// maxima); KIND 1: down -> routed [rows, H] bf16.  tm_x: the token rows
// ([max_rows, K], boxes of 64 x 8, 128-byte swizzle): f16 prescaled rows for
// MXFP4 (f16 MMAs), plain bf16 rows for FP8 (bf16 MMAs on weights rounded to
// bf16 after their block scale, as the reference decodes them).
template <int KIND, int KS, int FMT>
__global__ void __launch_bounds__(kThreads, kCtas) decode_mma_kernel(const __grid_constant__ CUtensorMap tm_x,
                                                                 const DecodeArgs a) {
  constexpr int kFeatItem = q_feat_item(KS), kRowsItem = q_rows_item(KS);
  constexpr int kRowWarps = kWarps / KS;
  constexpr bool kFp4 = FMT == kFmtMxfp4;
  constexpr int BR = q_block_rows(FMT);
  extern __shared__ uint8_t smem_raw[];
  const int K = KIND == 0 ? a.H : a.I;
  const int S = K / 32;       // bytes per scale row (E8M0 per row, or per FP8 block row)
  const int KC = K / q_chunk_k(FMT);  // chunks per row (64 bytes of each row)
  const int KCw = KC / KS;    // chunks of this warp's K slice
  const int nseg = q_nseg(K, FMT), SEGC = KC / nseg;  // segments of K, chunks per segment
  const int wseg = nseg / KS;                          // segments of this warp's slice
  const int64_t rowb = kFp4 ? K / 2 : K;  // bytes per weight row
  const int xbytes = q_xbytes(K), bufbytes = q_bufbytes(KIND, K, KS, FMT);
  const uint32_t raw0 = smem_u32(smem_raw);
  const uint32_t base = (raw0 + 1023u) & ~1023u;
  const int NB = a.nbuf;  // token-tile buffers: 2, or 1 when the CTA has one item or the tile is large
  float* red = reinterpret_cast<float*>(smem_raw + (base - raw0) + NB * bufbytes);
  QShared& sh = *reinterpret_cast<QShared*>(smem_raw + (base - raw0) + NB * bufbytes + q_redbytes(KS, nseg, NB));
  const int gsrows = q_srows(FMT, kFeatItem);  // scale rows of the gate (and of the up) rows of an item

  const int warp_id = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int warp = warp_id % kRowWarps;  // row group
  const int ks = warp_id / kRowWarps;    // K slice: chunks [ks * KCw, (ks + 1) * KCw)
  const int g = lane >> 2, t = lane & 3;
  const int nb = KIND == 0 ? a.I / kFeatItem : a.H / kRowsItem;  // row blocks per token tile
  const int n_items = *a.plan.n_mtiles * nb;
  const int gate_base = a.gate_first ? 0 : a.I, up_base = a.gate_first ? a.I : 0;

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sh.full[b], 1);
      for (int w = 0; w < kRowWarps; ++w) mbar_init(&sh.red_full[b][w], (KS - 1) * 32);
      sh.done[b] = 0;
    }
    sh.abort = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  volatile int* abort = &sh.abort;

  // Issues the token tile and scale block of item `it` into buffer b.
  auto issue = [&](const QItem& it, int b) {
    const uint32_t xdst = base + b * bufbytes, sdst = xdst + xbytes;
    mbar_arrive_expect_tx(&sh.full[b], uint32_t(xbytes + q_sbytes(KIND, K, KS, FMT)));
    for (int kb = 0; kb < K / 64; ++kb) tma_load_2d_q(xdst + kb * 1024, &tm_x, kb * 64, it.row0, &sh.full[b]);
    if (KIND == 0) {
      const uint8_t* s = a.wts.s13_of(it.e);
      const int n = gsrows * S;
      bulk_load(sdst, s + int64_t((gate_base + it.blk * kFeatItem) / BR) * S, n, &sh.full[b]);
      bulk_load(sdst + n, s + int64_t((up_base + it.blk * kFeatItem) / BR) * S, n, &sh.full[b]);
    } else {
      bulk_load(sdst, a.wts.s2_of(it.e) + int64_t(it.blk * kRowsItem / BR) * S, q_srows(FMT, kRowsItem) * S,
                &sh.full[b]);
    }
  };
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tm_x);
    for (int b = 0; b < NB; ++b)
      if (int(blockIdx.x) + b * int(gridDim.x) < n_items) issue(q_item(a, blockIdx.x + b * gridDim.x, nb), b);
  }

  // This thread's four weight rows, j = 2r + h: MMA tile r, fragment row g (h = 0) or g + 8 (h = 1).
  // Weight-row offsets from row j = 0, and scale-block rows.
  int64_t roff[2 * kRG];
  int srow[2 * kRG];
#pragma unroll
  for (int r = 0; r < kRG; ++r)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      // scale row in the staged block: the row's block, counted from the item's
      // first block (items never straddle a block they do not start on)
      if (KIND == 0) {
        roff[2 * r + h] = (int64_t(h ? up_base - gate_base : 0) + 8 * r) * rowb;
        srow[2 * r + h] = h * gsrows + (warp * (kRG * 8) + 8 * r + g) / BR;
      } else {
        roff[2 * r + h] = int64_t(16 * r + 8 * h) * rowb;
        srow[2 * r + h] = (warp * (kRG * 16) + 16 * r + 8 * h + g) / BR;
      }
    }
  // First weight row of this thread in item `it` (plus its 16-byte column of
  // the first chunk of its K slice).
  auto row_ptr = [&](const QItem& it) -> const uint8_t* {
    const int64_t col = 16 * t + int64_t(64) * KCw * ks;
    if (KIND == 0)
      return a.wts.w13_of(it.e) + int64_t(gate_base + it.blk * kFeatItem + warp * (kRG * 8) + g) * rowb + col;
    return a.wts.w2_of(it.e) + int64_t(it.blk * kRowsItem + warp * (kRG * 16) + g) * rowb + col;
  };

  // Item metadata, fetched an item before it is needed (q beyond the list: unused).
  auto fetch = [&](int q) -> QItem { return q < n_items ? q_item(a, q, nb) : QItem{0, 0, 0, 0}; };

  // Load cursor: item (lq) and chunk (lc) of the next chunk to load; lnext =
  // metadata of item lq + gridDim.x.
  int lq = blockIdx.x, lc = 0;
  const uint8_t* lp = lq < n_items ? row_ptr(q_item(a, lq, nb)) : nullptr;
  QItem lnext = fetch(lq + gridDim.x);
  uint4 wr[kStages][2 * kRG];
  auto load_next = [&](uint4 (&dst)[2 * kRG]) {
    if (lq < n_items) {
#pragma unroll
      for (int j = 0; j < 2 * kRG; ++j) dst[j] = ldg_nc_v4(lp + roff[j] + 64 * lc);
      if (++lc == KCw) {
        lc = 0;
        lq += gridDim.x;
        lp = row_ptr(lnext);
        lnext = fetch(lq + gridDim.x);
      }
    }
  };
#pragma unroll
  for (int s = 0; s < kStages; ++s) load_next(wr[s]);

  // Consumer state of the current item; nxt / nxt2 = metadata of the next
  // two items of this CTA (nxt2 feeds the refill of the buffer), bs = the
  // prescales of this thread's two tokens.
  int cq = blockIdx.x, cc = 0, li = 0;  // item, chunk, local item counter
  QItem cur{}, nxt = fetch(cq), nxt2{};
  float bs0 = 1.0f, bs1 = 1.0f;
  float rinv[2 * kRG];
  int smax[2 * kRG];
  float acc[kRG][2][4];  // per MMA tile, even and odd K steps (two independent chains)
  float y[kRG][4];       // the row sums so far: ((0 + s_0) + s_1) + ... over segments
  uint32_t xb = 0, sb = 0;
  bool alive = cq < n_items;

  auto begin_item = [&]() -> bool {
    cur = nxt;
    nxt = fetch(cq + gridDim.x);
    nxt2 = fetch(cq + 2 * gridDim.x);
    if (kFp4) {
      bs0 = 2 * t < cur.valid ? a.bscale[cur.row0 + 2 * t] : 1.0f;
      bs1 = 2 * t + 1 < cur.valid ? a.bscale[cur.row0 + 2 * t + 1] : 1.0f;
    }
    const int b = li % NB;
    if (!warp_wait(&sh.full[b], (li / NB) & 1, abort)) {
      if (lane == 0 && !*abort) {
        report_status(a.status, kStatusWaitTimeout, 40 + KIND);
        sh.abort = 1;
      }
      return false;
    }
    xb = base + b * bufbytes;
    sb = xb + xbytes;
    // largest E8M0 byte of each of this thread's rows (the four t lanes split a row)
#pragma unroll
    for (int j = 0; j < (kFp4 ? 2 * kRG : 0); ++j) {
      const uint32_t rb = sb + srow[j] * S + t * (S / 4);
      uint32_t m = 0;
      if ((S & 15) == 0) {  // a lane's S / 4 bytes are whole, aligned words
        for (int i = 0; i < S / 4; i += 4) m = __vmaxu4(m, lds_u32(rb + i));
        m = max(max(m & 0xffu, (m >> 8) & 0xffu), max((m >> 16) & 0xffu, m >> 24));
      } else {
        for (int i = 0; i < S / 4; ++i) m = max(m, lds_u8q(rb + i));
      }
      m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
      m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
      smax[j] = int(m);
      rinv[j] = __uint_as_float(uint32_t(254 - min(int(m), 254)) << 23);
    }
#pragma unroll
    for (int r = 0; r < kRG; ++r)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[r][0][i] = acc[r][1][i] = y[r][i] = 0.0f;
    return true;
  };

  // red: [buffer][K slice 1 .. KS-1][segment of the slice][row group][tile r][lane] float4.
  // A buffer's slots are rewritten NB items later, after every warp
  // released that buffer, so the group's first warp has read them by then.
  auto red_slot = [&](int b, int k, int sg) {
    return reinterpret_cast<float4*>(red) + (((b * (KS - 1) + k - 1) * wseg + sg) * kRowWarps + warp) * 32 * kRG + lane;
  };
  // End of segment sg of this warp's slice: its sum s = chain0 + chain1 goes
  // into y (the group's first warp) or to shared memory; the chains restart.
  auto end_segment = [&](int sg) {
    const int b = li % NB;
#pragma unroll
    for (int r = 0; r < kRG; ++r) {
      float sv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        sv[i] = acc[r][0][i] + acc[r][1][i];
        acc[r][0][i] = acc[r][1][i] = 0.0f;
      }
      if (ks == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) y[r][i] += sv[i];
      } else {
        red_slot(b, ks, sg)[32 * r] = make_float4(sv[0], sv[1], sv[2], sv[3]);
      }
    }
  };

  auto end_item = [&]() {
    const int n0 = 2 * t, n1 = 2 * t + 1;
    const float is0 = 1.0f / bs0, is1 = 1.0f / bs1;
    bool lead = true;  // this warp runs the epilogue of its rows
    if (KS > 1) {
      const int b = li % NB;
      if (ks > 0) {  // the segment sums are in place
        mbar_arrive(&sh.red_full[b][warp]);
        lead = false;
      } else if (!warp_wait(&sh.red_full[b][warp], (li / NB) & 1, abort)) {
        if (lane == 0 && !*abort) {
          report_status(a.status, kStatusWaitTimeout, 44 + KIND);
          sh.abort = 1;
        }
        lead = false;
      } else {
        for (int k = 1; k < KS; ++k)  // segment order: slices are consecutive segments
          for (int sg = 0; sg < wseg; ++sg) {
            const float4* src = red_slot(b, k, sg);
#pragma unroll
            for (int r = 0; r < kRG; ++r) {
              const float4 v = src[32 * r];
              y[r][0] += v.x;
              y[r][1] += v.y;
              y[r][2] += v.z;
              y[r][3] += v.w;
            }
          }
      }
    }
    if (!lead) {
      // partial sums only: the group's first warp writes these rows
    } else if (KIND == 0) {
      float m0 = 0.0f, m1 = 0.0f;
#pragma unroll
      for (int r = 0; r < kRG; ++r) {
        const float fg = kFp4 ? e8m0_to_f32(uint32_t(smax[2 * r])) : 1.0f;
        const float fu = kFp4 ? e8m0_to_f32(uint32_t(smax[2 * r + 1])) : 1.0f;
        const int f = cur.blk * kFeatItem + warp * (kRG * 8) + 8 * r + g;
        if (n0 < cur.valid) {
          const float gv = bf16_round(y[r][0] * fg * is0), uv = bf16_round(y[r][2] * fu * is0);
          const uint16_t bits = f32_to_bf16_bits(swiglu_f32(gv, uv, a.limit));
          a.act[int64_t(cur.row0 + n0) * a.I + f] = bits;
          m0 = fmaxf(m0, fabsf(bf16_bits_to_f32(bits)));
        }
        if (n1 < cur.valid) {
          const float gv = bf16_round(y[r][1] * fg * is1), uv = bf16_round(y[r][3] * fu * is1);
          const uint16_t bits = f32_to_bf16_bits(swiglu_f32(gv, uv, a.limit));
          a.act[int64_t(cur.row0 + n1) * a.I + f] = bits;
          m1 = fmaxf(m1, fabsf(bf16_bits_to_f32(bits)));
        }
      }
      // per-token maxima over the warp's features (lanes with the same t)
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
      }
      if (kFp4 && g == 0) {  // the f16 prescale of the act rows (FP8 keeps bf16 rows)
        if (n0 < cur.valid) atomicMax(a.plan.rowmax + cur.row0 + n0, __float_as_uint(m0));
        if (n1 < cur.valid) atomicMax(a.plan.rowmax + cur.row0 + n1, __float_as_uint(m1));
      }
    } else {
#pragma unroll
      for (int r = 0; r < kRG; ++r)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float fr = kFp4 ? e8m0_to_f32(uint32_t(smax[2 * r + h])) : 1.0f;
          const int hc = cur.blk * kRowsItem + warp * (kRG * 16) + 16 * r + 8 * h + g;
          if (n0 < cur.valid) a.routed[int64_t(cur.row0 + n0) * a.H + hc] = f32_to_bf16_bits(y[r][2 * h] * fr * is0);
          if (n1 < cur.valid)
            a.routed[int64_t(cur.row0 + n1) * a.H + hc] = f32_to_bf16_bits(y[r][2 * h + 1] * fr * is1);
        }
    }
    // release the buffer; the last warp refills it with the item NB items on
    __syncwarp();
    if (lane == 0) {
      const int b = li % NB;
      __threadfence_block();
      if (atomicAdd(&sh.done[b], 1) == kWarps - 1) {
        sh.done[b] = 0;
        if (cq + NB * int(gridDim.x) < n_items && !*abort) issue(NB == 2 ? nxt2 : nxt, b);
      }
    }
    __syncwarp();
  };

  // FP8: lane t's 16 bytes of a row are 16 E4M3 weights at K offset 64cc + 16t,
  // one block scale; each weight is rounded to bf16 after its fp32 scaling
  // (the reference's decode), the token operand is the plain bf16 row.  Word
  // q (4 weights) is one MMA step: slots {2t, 2t+1} <- weights 4q, 4q+1 and
  // slots {2t+8, 2t+9} <- 4q+2, 4q+3, the token operand at the same K.
  auto chunk_fp8 = [&](const uint4 (&w)[2 * kRG], int cc) {
    float sc[2 * kRG];
#pragma unroll
    for (int j = 0; j < 2 * kRG; ++j) {
      const uint32_t sa = sb + srow[j] * S;
      if (FMT == kFmtFp8B32)
        sc[j] = e8m0_to_f32(lds_u8q(sa + 2 * cc + (t >> 1)), true);
      else
        sc[j] = __uint_as_float(lds_u32(sa + 4 * (cc >> 1)));
    }
    const uint32_t xrow = xb + cc * 1024 + g * 128;  // box cc: this chunk's 64 K of token row g
    uint4 xv[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) xv[u] = lds_v4q(xrow + (((2 * t + u) ^ g) << 4));
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4& xq = xv[q >> 1];
      const uint32_t x0 = (q & 1) ? xq.z : xq.x, x1 = (q & 1) ? xq.w : xq.y;
#pragma unroll
      for (int r = 0; r < kRG; ++r) {
        const uint4& wa = w[2 * r];
        const uint4& wb = w[2 * r + 1];
        const uint32_t va = q == 0 ? wa.x : q == 1 ? wa.y : q == 2 ? wa.z : wa.w;
        const uint32_t vb = q == 0 ? wb.x : q == 1 ? wb.y : q == 2 ? wb.z : wb.w;
        float fa[4], fb[4];
        e4m3x4_to_f32(va, fa);
        e4m3x4_to_f32(vb, fb);
        const float sa = sc[2 * r], sbv = sc[2 * r + 1];
        const uint32_t a01 = pack_bf16x2(__fmul_rn(fa[0], sa), __fmul_rn(fa[1], sa));
        const uint32_t a23 = pack_bf16x2(__fmul_rn(fa[2], sa), __fmul_rn(fa[3], sa));
        const uint32_t b01 = pack_bf16x2(__fmul_rn(fb[0], sbv), __fmul_rn(fb[1], sbv));
        const uint32_t b23 = pack_bf16x2(__fmul_rn(fb[2], sbv), __fmul_rn(fb[3], sbv));
        mma_bf16q(acc[r][q & 1], a01, b01, a23, b23, x0, x1);
      }
    }
  };

  // One chunk of the current item from the weight registers w.
  auto chunk = [&](const uint4 (&w)[2 * kRG], int cc) {
    if constexpr (!kFp4) {
      chunk_fp8(w, cc);
    } else {
      uint32_t mult[2 * kRG];
  #pragma unroll
      for (int j = 0; j < 2 * kRG; ++j) mult[j] = group_mult(lds_u8q(sb + srow[j] * S + 4 * cc + t), rinv[j]);
      // token operand: 32 f16 at K offset 128cc + 32t of token row g (4 swizzled 16-byte units)
      const int kb = 2 * cc + (t >> 1);
      const uint32_t xrow = xb + kb * 1024 + g * 128;
      uint4 xv[4];
  #pragma unroll
      for (int u = 0; u < 4; ++u) xv[u] = lds_v4q(xrow + (((4 * (t & 1) + u) ^ g) << 4));
  #pragma unroll
      for (int q = 0; q < 4; ++q) {  // word q of the 16 bytes: K offsets 8q .. 8q + 7 = steps 2q, 2q + 1
        const uint32_t xw[4] = {xv[q].x, xv[q].y, xv[q].z, xv[q].w};
  #pragma unroll
        for (int r = 0; r < kRG; ++r) {
          const uint4& wa = w[2 * r];
          const uint4& wb = w[2 * r + 1];
          const uint32_t va = q == 0 ? wa.x : q == 1 ? wa.y : q == 2 ? wa.z : wa.w;
          const uint32_t vb = q == 0 ? wb.x : q == 1 ? wb.y : q == 2 ? wb.z : wb.w;
          uint32_t ha[4], hb[4];
          e2m1x8_f16x2(va, ha);
          e2m1x8_f16x2(vb, hb);
  #pragma unroll
          for (int p = 0; p < 4; ++p) {
            ha[p] = hmul2q(ha[p], mult[2 * r]);
            hb[p] = hmul2q(hb[p], mult[2 * r + 1]);
          }
          // step 2q: bytes 0, 1 (K 8q .. 8q+3); step 2q + 1: bytes 2, 3 (K 8q+4 .. 8q+7)
          mma_f16(acc[r][0], ha[0], hb[0], ha[1], hb[1], xw[0], xw[1]);
          mma_f16(acc[r][1], ha[2], hb[2], ha[3], hb[3], xw[2], xw[3]);
        }
      }
    }
  };

  // Items are whole multiples of kStages chunks (KC % kStages == 0), so the
  // ring slot of a chunk is static and one copy of the item code serves.
  const int c0 = ks * KCw;  // first chunk of this warp's K slice
  if (alive) alive = begin_item();
  while (alive) {
    for (int sg = 0; sg < wseg; ++sg) {
      for (cc = 0; cc < SEGC; cc += kStages) {
#pragma unroll
        for (int s = 0; s < kStages; ++s) {
          chunk(wr[s], c0 + sg * SEGC + cc + s);
          load_next(wr[s]);
        }
      }
      end_segment(sg);
    }
    end_item();
    ++li;
    cq += gridDim.x;
    alive = cq < n_items && !warp_aborted(abort);
    if (alive) alive = begin_item();
  }
  __syncthreads();
}

bool decode_mma_shape_ok(int H, int I, int fmt) {
  const int ck = q_chunk_k(fmt) * kStages;
  // FP8 scale rows (K / 32 bytes) are bulk copies: whole 16-byte units
  const bool scale_rows = fmt == kFmtMxfp4 || (H % 512 == 0 && I % 512 == 0);
  return I % q_feat_item(1) == 0 && H % q_rows_item(1) == 0 && H % ck == 0 && I % ck == 0 && scale_rows &&
         q_smem_bytes(0, H, 1, fmt, 1) <= 227 * 1024 && q_smem_bytes(1, I, 1, fmt, 1) <= 227 * 1024;
}

namespace {

template <int KIND, int KS, int FMT>
void set_smem(int K) {
  cudaFuncSetAttribute(decode_mma_kernel<KIND, KS, FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       int(std::min(q_smem_bytes(KIND, K, KS, FMT, 2), size_t(227 * 1024))));
}

template <int FMT>
void set_smem_all(int max_h, int max_i) {
  set_smem<0, 1, FMT>(max_h);
  set_smem<0, 2, FMT>(max_h);
  set_smem<0, 4, FMT>(max_h);
  set_smem<0, 8, FMT>(max_h);
  set_smem<1, 1, FMT>(max_i);
  set_smem<1, 2, FMT>(max_i);
  set_smem<1, 4, FMT>(max_i);
  set_smem<1, 8, FMT>(max_i);
}

template <int KIND, int KS, int FMT>
void launch_ks(const DecodeArgs& a, const CUtensorMap& x, int num_sms, cudaStream_t stream) {
  const int K = KIND == 0 ? a.H : a.I;
  decode_mma_kernel<KIND, KS, FMT>
      <<<num_sms * kCtas, kThreads, q_smem_bytes(KIND, K, KS, FMT, a.nbuf), stream>>>(x, a);
}

template <int KIND, int FMT>
void launch_kind(const DecodeArgs& a, const CUtensorMap& x, int num_sms, cudaStream_t stream, int ks) {
  if (ks >= 8) launch_ks<KIND, 8, FMT>(a, x, num_sms, stream);
  else if (ks >= 4) launch_ks<KIND, 4, FMT>(a, x, num_sms, stream);
  else if (ks >= 2) launch_ks<KIND, 2, FMT>(a, x, num_sms, stream);
  else launch_ks<KIND, 1, FMT>(a, x, num_sms, stream);
}

template <int FMT>
void launch_fmt(const DecodeArgs& a, int kind, const CUtensorMap& x, int num_sms, cudaStream_t stream, int ks) {
  if (kind == 0) launch_kind<0, FMT>(a, x, num_sms, stream, ks);
  else launch_kind<1, FMT>(a, x, num_sms, stream, ks);
}

}  // namespace

// Shapes beyond the shared-memory limit never take this kernel (decode_mma_shape_ok).
void decode_mma_init_attributes(int max_h, int max_i) {
  static std::mutex mu;
  static int set_h[kMaxDevices] = {}, set_i[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return;
  std::lock_guard<std::mutex> lock(mu);  // only ever raised (see gemv_init_attributes)
  max_h = std::max(max_h, set_h[dev]);
  max_i = std::max(max_i, set_i[dev]);
  set_h[dev] = max_h;
  set_i[dev] = max_i;
  set_smem_all<kFmtMxfp4>(max_h, max_i);
  set_smem_all<kFmtFp8B128>(max_h, max_i);
  set_smem_all<kFmtFp8B32>(max_h, max_i);
}

int decode_mma_split(int kind, int H, int I, int tiles, int num_sms, int fmt) {
  const int K = kind == 0 ? H : I;
  const int nb = kind == 0 ? I / q_feat_item(1) : H / q_rows_item(1);  // row blocks of an unsplit item
  // Split while the items would leave over half of the SMs idle (measured on
  // config-1 decode: batch 1 gate/up 22 -> 88 items, down 44 -> 88; from
  // about 80 unsplit items on, splitting costs more than it spreads).
  int ks = 1;
  while (2 * ks <= q_nseg(K, fmt) && int64_t(tiles) * nb * ks * 2 < num_sms &&
         q_smem_bytes(kind, K, 2 * ks, fmt, 1) <= 227 * 1024)
    ks *= 2;
  return ks;
}

int decode_mma_buffers(int kind, int H, int I, int ks, int tiles, int num_sms, int fmt) {
  const int K = kind == 0 ? H : I;
  const int64_t items = int64_t(tiles) * (kind == 0 ? I / q_feat_item(ks) : H / q_rows_item(ks));
  // A second token-tile buffer only pays when CTAs get several items, and
  // shared memory past ~160 KB leaves the L1 too small for the weight loads
  // in flight (the carve-out steps of the B200 SM).
  return items > num_sms && q_smem_bytes(kind, K, ks, fmt, 2) <= 160 * 1024 ? 2 : 1;
}

void launch_decode_mma(const DecodeArgs& a, int kind, const void* tmap_x, int num_sms, cudaStream_t stream, int ks,
                       int fmt) {
  const CUtensorMap& x = *static_cast<const CUtensorMap*>(tmap_x);
  if (fmt == kFmtFp8B128) launch_fmt<kFmtFp8B128>(a, kind, x, num_sms, stream, ks);
  else if (fmt == kFmtFp8B32) launch_fmt<kFmtFp8B32>(a, kind, x, num_sms, stream, ks);
  else launch_fmt<kFmtMxfp4>(a, kind, x, num_sms, stream, ks);
}

}  // namespace wm
