// Prefill path: grouped GEMM over expert-sorted rows on the 5th-generation
// tensor cores (tcgen05.mma, kind::f16, bf16 operands, fp32 accumulators in
// TMEM), with the expert weights dequantised on the fly.
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
//               dequantises them to bf16 and stores them in the 128-byte
//               swizzled K-major layout the MMA reads
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
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;

struct Shared {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint32_t tmem_base;
  int abort;
};

// One 32-bit word of E2M1 nibbles (8 values) times `scale` -> 4 bf16x2.
__device__ __forceinline__ uint4 dq_mxfp4_word(uint32_t w, float scale) {
  float v[8];
  e2m1x8_to_f32(w, v);
  uint4 o;
  o.x = pack_bf16x2(v[0] * scale, v[1] * scale);
  o.y = pack_bf16x2(v[2] * scale, v[3] * scale);
  o.z = pack_bf16x2(v[4] * scale, v[5] * scale);
  o.w = pack_bf16x2(v[6] * scale, v[7] * scale);
  return o;
}

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

__device__ __forceinline__ void sts_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void stg_v4(void* p, uint4 v) {
  asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
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
    constexpr uint32_t idesc = umma_idesc_bf16(BM, BN);
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
    const int j = (warp - DQ_WARP0) * 32 + lane;  // B-tile row 0..255
    const int gate_base = a.gate_first ? 0 : a.I, up_base = a.gate_first ? a.I : 0;
    const int64_t rb = FMT == kFmtMxfp4 ? a.Kdim / 2 : a.Kdim;   // weight row bytes
    uint32_t it = 0;
    for (int t = blockIdx.x; t < total && !*abort; t += gridDim.x) {
      const int e = a.plan.mtiles[2 * (t / n_tiles_n)];
      const int nt = t % n_tiles_n;
      int grow;
      if (KIND == 0)
        grow = j < BN / 2 ? gate_base + nt * (BN / 2) + j : up_base + nt * (BN / 2) + (j - BN / 2);
      else
        grow = nt * BN + j;
      const uint8_t* wrow = (KIND == 0 ? a.wts.w13_of(e) : a.wts.w2_of(e)) + int64_t(grow) * rb;
      const uint8_t* srow = KIND == 0 ? a.wts.s13_of(e) : a.wts.s2_of(e);
      bool ok = true;
      for (int kb = 0; kb < kblocks; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1u;
        uint4 q[8];
        if (FMT == kFmtMxfp4) {
          const uint4 w0 = ldg_nc_v4(wrow + kb * 32);
          const uint4 w1 = ldg_nc_v4(wrow + kb * 32 + 16);
          const uint8_t* sr = srow + int64_t(grow) * (a.Kdim / 32) + kb * 2;
          const float s0 = e8m0_to_f32(ldg_nc_u8(sr)), s1 = e8m0_to_f32(ldg_nc_u8(sr + 1));
          q[0] = dq_mxfp4_word(w0.x, s0);
          q[1] = dq_mxfp4_word(w0.y, s0);
          q[2] = dq_mxfp4_word(w0.z, s0);
          q[3] = dq_mxfp4_word(w0.w, s0);
          q[4] = dq_mxfp4_word(w1.x, s1);
          q[5] = dq_mxfp4_word(w1.y, s1);
          q[6] = dq_mxfp4_word(w1.z, s1);
          q[7] = dq_mxfp4_word(w1.w, s1);
        } else {
          const uint4 w0 = ldg_nc_v4(wrow + kb * 64);
          const uint4 w1 = ldg_nc_v4(wrow + kb * 64 + 16);
          const uint4 w2 = ldg_nc_v4(wrow + kb * 64 + 32);
          const uint4 w3 = ldg_nc_v4(wrow + kb * 64 + 48);
          const float* sf = reinterpret_cast<const float*>(srow);
          const float sc = __ldg(sf + int64_t(grow / 128) * (a.Kdim / 128) + kb / 2);
          q[0] = dq_fp8_8(w0.x, w0.y, sc);
          q[1] = dq_fp8_8(w0.z, w0.w, sc);
          q[2] = dq_fp8_8(w1.x, w1.y, sc);
          q[3] = dq_fp8_8(w1.z, w1.w, sc);
          q[4] = dq_fp8_8(w2.x, w2.y, sc);
          q[5] = dq_fp8_8(w2.z, w2.w, sc);
          q[6] = dq_fp8_8(w3.x, w3.y, sc);
          q[7] = dq_fp8_8(w3.z, w3.w, sc);
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
      if (!mbar_wait(&sh.tmem_full[acc], acc_ph, abort)) {
        fail(sh, a.status, 14);
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem + acc * BN + (uint32_t(quarter * 32) << 16);
      if (KIND == 0) {
        uint16_t* dst = a.out + int64_t(row) * a.I + nt * (BN / 2);
#pragma unroll 1
        for (int jc = 0; jc < 4; ++jc) {
          uint32_t g[32], u[32];
          tmem_ld_32cols(taddr + jc * 32, g);
          tmem_ld_32cols(taddr + BN / 2 + jc * 32, u);
          tmem_ld_wait();
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            // the MLX path rounds the gate/up product to bf16 before the activation
            const float g0 = bf16_round(__uint_as_float(g[2 * i])), g1 = bf16_round(__uint_as_float(g[2 * i + 1]));
            const float u0 = bf16_round(__uint_as_float(u[2 * i])), u1 = bf16_round(__uint_as_float(u[2 * i + 1]));
            pk[i] = pack_bf16x2(swiglu_f32(g0, u0, a.limit), swiglu_f32(g1, u1, a.limit));
          }
#pragma unroll
          for (int i = 0; i < 4; ++i)
            stg_v4(dst + jc * 32 + i * 8, make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]));
        }
      } else {
        uint16_t* dst = a.out + int64_t(row) * a.N + nt * BN;
#pragma unroll 1
        for (int jc = 0; jc < 8; ++jc) {
          uint32_t v[32];
          tmem_ld_32cols(taddr + jc * 32, v);
          tmem_ld_wait();
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) pk[i] = pack_bf16x2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
#pragma unroll
          for (int i = 0; i < 4; ++i)
            stg_v4(dst + jc * 32 + i * 8, make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.tmem_empty[acc]);
    }
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
  } else {
    if (kind == 0)
      gemm_kernel<kFmtFp8B128, 0><<<grid, block, SMEM_BYTES, stream>>>(tm, a);
    else
      gemm_kernel<kFmtFp8B128, 1><<<grid, block, SMEM_BYTES, stream>>>(tm, a);
  }
}

}  // namespace wm
