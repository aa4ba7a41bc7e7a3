// Router logits on the tensor cores for long calls (prefill):
//   logits[T, E] = x[T, H] . W_r[E, H]^T, bf16 operands, fp32 accumulation.
//
// Reference: the router projection of SparseMoE.route (qwen4_exp.py:1009-1013),
// Gate.__call__ (deepseek_v41/moe.py:58-62) and Router.__call__
// (mimo/model.py:139-141) -- a plain bf16 matmul with fp32 results, here a
// tcgen05 GEMM; the top-k selection that follows is router_topk_kernel.
// Decode-sized calls keep the CUDA-core router (wm_route.cu): there the
// router weights' bytes, not arithmetic, set the time.
//
// One persistent CTA per SM walks the (128-token, 128-expert) output tiles.
// Warp 0 issues the TMA loads of both operands (128-byte swizzle, six
// stages); warp 1 owns TMEM and issues the MMAs (elect.sync in a converged
// warp); warps 2-5 drain the two TMEM accumulators into fp32 logits.  Rows
// past T load as zeros (TMA out-of-bounds fill) and are not stored.  Every
// mbarrier wait is bounded; a timeout records the status and unwinds.
#include <cuda.h>

#include "wm_kernels.h"

namespace wm {

namespace {

constexpr int RBM = 128, RBN = 128, RBK = 64, RSTAGES = 6, RUMMA_K = 16;
constexpr int RA_BYTES = RBM * RBK * 2;  // 16 KB
constexpr int RB_BYTES = RBN * RBK * 2;  // 16 KB
constexpr int R_THREADS = 192;
constexpr uint32_t R_TMEM_COLS = 2 * RBN;
constexpr int R_SMEM = RSTAGES * (RA_BYTES + RB_BYTES) + 1024 + 256;

struct RShared {
  uint64_t full[RSTAGES], empty[RSTAGES];
  uint64_t tmem_full[2], tmem_empty[2];
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void rfail(RShared& sh, uint32_t* status, uint32_t role) {
  report_status(status, kStatusWaitTimeout, role);
  sh.abort = 1;
}

__device__ __forceinline__ void stg_f4(float* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

}  // namespace

__global__ void __launch_bounds__(R_THREADS, 1)
    router_gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w, int T,
                       int H, int E, float* __restrict__ logits, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* tiles = smem_raw + (base - raw);
  RShared& sh = *reinterpret_cast<RShared*>(tiles + RSTAGES * (RA_BYTES + RB_BYTES));
  const uint32_t a_smem = base, b_smem = base + RSTAGES * RA_BYTES;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_n = E / RBN, n_m = (T + RBM - 1) / RBM, total = n_m * n_n, kblocks = H / RBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < RSTAGES; ++s) {
      mbar_init(&sh.full[s], 1);
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
    tmem_alloc(&sh.tmem_base, R_TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  volatile int* abort = &sh.abort;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok && !*abort; t += gridDim.x) {
        const int mt = t / n_n, nt = t % n_n;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % RSTAGES;
          if (!mbar_wait(&sh.empty[s], ((it / RSTAGES) & 1u) ^ 1u, abort)) {
            rfail(sh, status, 40);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&sh.full[s], RA_BYTES + RB_BYTES);
          tma_load_2d(tiles + s * RA_BYTES, &tm_x, kb * RBK, mt * RBM, &sh.full[s]);
          tma_load_2d(tiles + RSTAGES * RA_BYTES + s * RB_BYTES, &tm_w, kb * RBK, nt * RBN, &sh.full[s]);
        }
      }
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc = umma_idesc_bf16(RBM, RBN);
    uint32_t it = 0, lt = 0;
    for (int t = blockIdx.x; t < total && !warp_aborted(abort); t += gridDim.x, ++lt) {
      const uint32_t acc = lt & 1u;
      if (!warp_wait(&sh.tmem_empty[acc], ((lt >> 1) & 1u) ^ 1u, abort)) {
        if (lane == 0) rfail(sh, status, 41);
        break;
      }
      tc_fence_after();
      bool ok = true;
      for (int kb = 0; kb < kblocks; ++kb, ++it) {
        const int s = it % RSTAGES;
        if (!warp_wait(&sh.full[s], (it / RSTAGES) & 1u, abort)) {
          if (lane == 0) rfail(sh, status, 42);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t da = umma_desc_sw128(a_smem + s * RA_BYTES);
        const uint64_t db = umma_desc_sw128(b_smem + s * RB_BYTES);
#pragma unroll
        for (int k = 0; k < RBK / RUMMA_K; ++k)  // K16 step = 32 bytes = 2 in the descriptor's address field
          umma_f16_elect(tmem + acc * RBN, da + 2 * k, db + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
        umma_commit_elect(&sh.empty[s]);
      }
      if (!ok) break;
      umma_commit_elect(&sh.tmem_full[acc]);
    }
  } else {
    const int quarter = warp & 3;  // TMEM lanes 32 * quarter ... (warps 2-5 cover all four)
    uint32_t lt = 0;
    for (int t = blockIdx.x; t < total && !*abort; t += gridDim.x, ++lt) {
      const uint32_t acc = lt & 1u;
      const int mt = t / n_n, nt = t % n_n;
      if (!mbar_wait(&sh.tmem_full[acc], (lt >> 1) & 1u, abort)) {
        rfail(sh, status, 43);
        break;
      }
      tc_fence_after();
      const int row = mt * RBM + quarter * 32 + lane;
      float* dst = logits + int64_t(row) * E + nt * RBN;
      const uint32_t taddr = tmem + acc * RBN + (uint32_t(quarter * 32) << 16);
#pragma unroll 1
      for (int jc = 0; jc < RBN / 32; ++jc) {
        uint32_t v[32];
        tmem_ld_32cols(taddr + jc * 32, v);
        tmem_ld_wait();
        if (row < T) {
#pragma unroll
          for (int i = 0; i < 8; ++i) stg_f4(dst + jc * 32 + 4 * i, v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
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
    tmem_dealloc(tmem, R_TMEM_COLS);
  }
}

bool router_gemm_shape_ok(int T, int H, int E) { return T >= 256 && H % RBK == 0 && E % RBN == 0; }

void router_gemm_init_attributes() {
  cudaFuncSetAttribute(router_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, R_SMEM);
}

void launch_router_gemm(const void* tm_x, const void* tm_w, int T, int H, int E, float* logits, uint32_t* status,
                        int num_sms, cudaStream_t stream) {
  const int tiles = ((T + RBM - 1) / RBM) * (E / RBN);
  const int grid = tiles < num_sms ? tiles : num_sms;
  router_gemm_kernel<<<grid, R_THREADS, R_SMEM, stream>>>(*static_cast<const CUtensorMap*>(tm_x),
                                                          *static_cast<const CUtensorMap*>(tm_w), T, H, E, logits,
                                                          status);
}

}  // namespace wm
