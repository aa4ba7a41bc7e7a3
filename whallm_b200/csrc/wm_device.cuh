// Device helpers shared by the MoE expert-FFN kernels (sm_100a only).
//
// * number formats: bf16, E2M1 (MXFP4 nibbles), E8M0 scales, FP8 E4M3;
// * the device status word that bounded waits report into;
// * thin inline-PTX wrappers for mbarrier, TMA (cp.async.bulk.tensor) and
//   the 5th-generation tensor-core instructions (tcgen05.*).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "wm_types.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "whallm_b200 kernels are written for sm_100a only"
#endif

namespace wm {

// ------------------------------------------------------------------ status

// Device status codes (first nonzero one wins; read back by wm_sync).
enum : uint32_t {
  kStatusOk = 0,
  kStatusWaitTimeout = 1,   // an mbarrier wait in a GEMM kernel ran out of time
  kStatusBadExpert = 2,     // a route named an expert outside [0, E)
  kStatusOverflow = 3,      // sorted rows exceeded the workspace capacity
  kStatusNanCode = 4,       // an FP8 weight held a reserved NaN code
};

__device__ __forceinline__ void report_status(uint32_t* status, uint32_t code, uint32_t where) {
  if (status != nullptr && atomicCAS(status, 0u, code) == 0u) status[1] = where;
}

// ------------------------------------------------------------------ number formats

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}

__device__ __forceinline__ float bf16_round(float f) { return __uint_as_float(uint32_t(f32_to_bf16_bits(f)) << 16); }

// Two floats -> packed bf16x2 (lo in bits 0-15), round to nearest even.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float2 unpack_bf16x2(uint32_t v) {
  return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}

// E8M0 byte -> 2^(b-127) as a float; b = 0 is 0 (the Metal convention) unless
// `mlx_zero` selects the subnormal 2^-127 of the MLX decode.  b = 255 -> +inf.
__device__ __forceinline__ float e8m0_to_f32(uint32_t b, bool mlx_zero = false) {
  if (b == 0u) return mlx_zero ? __uint_as_float(0x00400000u) : 0.0f;
  return __uint_as_float(b << 23);
}

// Two E2M1 codes (the low byte of `byte2`, low nibble first) -> half2, exactly.
// Uses the sm_100a hardware conversion; E2M1 code 8 gives -0.
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte2) {
  uint32_t r;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t}"
      : "=r"(r) : "r"(byte2));
  return r;
}

// Eight E2M1 codes of one 32-bit word (nibble j = element j) -> 8 floats,
// exact.  out[j] = value of element j.
__device__ __forceinline__ void e2m1x8_to_f32(uint32_t w, float* out) {
  uint32_t h0, h1, h2, h3;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3) : "r"(w));
  float2 f;
  f = __half22float2(*reinterpret_cast<__half2*>(&h0)); out[0] = f.x; out[1] = f.y;
  f = __half22float2(*reinterpret_cast<__half2*>(&h1)); out[2] = f.x; out[3] = f.y;
  f = __half22float2(*reinterpret_cast<__half2*>(&h2)); out[4] = f.x; out[5] = f.y;
  f = __half22float2(*reinterpret_cast<__half2*>(&h3)); out[6] = f.x; out[7] = f.y;
}

// Four FP8 E4M3 bytes -> 4 floats, exactly (hardware conversion to half2).
// The reserved NaN codes 0x7F / 0xFF decode to NaN.
__device__ __forceinline__ void e4m3x4_to_f32(uint32_t w, float* out) {
  uint32_t h0, h1;
  asm("{\n\t.reg .b16 lo, hi;\n\t"
      "mov.b32 {lo, hi}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, lo;\n\t"
      "cvt.rn.f16x2.e4m3x2 %1, hi;\n\t}"
      : "=r"(h0), "=r"(h1) : "r"(w));
  float2 f;
  f = __half22float2(*reinterpret_cast<__half2*>(&h0)); out[0] = f.x; out[1] = f.y;
  f = __half22float2(*reinterpret_cast<__half2*>(&h1)); out[2] = f.x; out[3] = f.y;
}

__device__ __forceinline__ float silu_f32(float v) { return v / (1.0f + __expf(-v)); }

// SwiGLU of one gate/up pair; limit <= 0 means unclamped.
__device__ __forceinline__ float swiglu_f32(float g, float u, float limit) {
  if (limit > 0.0f) {
    g = fminf(g, limit);
    u = fminf(fmaxf(u, -limit), limit);
  }
  return silu_f32(g) * u;
}

// ------------------------------------------------------------------ global memory

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

__device__ __forceinline__ uint32_t ldg_nc_u8(const uint8_t* p) {
  uint16_t r;
  asm volatile("ld.global.nc.u8 %0, [%1];" : "=h"(r) : "l"(p));
  return r;
}

// ------------------------------------------------------------------ shared memory / mbarrier

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  // the phase token is not needed: the sink lets the warp go on without waiting for it
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking probe of a phase.  On B200 it answers in about half the time
// try_wait takes on an already-completed phase, so it is the fast path.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on an mbarrier phase.  Gives up after `timeout_ns` of wall time,
// or as soon as another role raised `*abort`, and returns false then; the
// caller reports the status and unwinds.  A healthy wait lasts microseconds.
// `sleep_ns` > 0 backs off between polls: a waiting warp then leaves the
// issue slots to the working warps of its SM instead of polling.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          uint32_t sleep_ns = 0, uint64_t timeout_ns = 2000000000ull) {
  if (mbar_test_wait(bar, parity)) return true;
  uint64_t start = global_timer_ns();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if (sleep_ns != 0u) __nanosleep(sleep_ns);
    if ((spin & 15u) == 0u) {
      if (*abort) return false;
      if (global_timer_ns() - start > timeout_ns) return false;
    }
  }
}

// mbar_wait by every lane of a converged warp; the result is warp-uniform
// (false if any lane gave up), so the warp stays converged after it.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          uint32_t sleep_ns = 0) {
  const bool ok = mbar_wait(bar, parity, abort, sleep_ns);
  return __all_sync(0xffffffffu, ok);
}

// Warp-uniform read of the abort flag.
__device__ __forceinline__ bool warp_aborted(volatile int* abort) { return __any_sync(0xffffffffu, *abort != 0); }

// ------------------------------------------------------------------ proxy fences

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy reads (tcgen05.mma operands, TMA stores).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------ TMA

// 2-D tiled bulk tensor load global -> shared, completing on `bar` (tx bytes).
// Callers keep the innermost coordinate x a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, int32_t x, int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ------------------------------------------------------------------ tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16/f16 operands, fp32 accumulate).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Warp-wide MMA issue: every lane of a converged warp calls these with the
// same arguments and one elected lane issues the instruction.  Measured on
// B200, an M128 x K16 MMA issued this way costs ~60 cycles when one warp
// issues, against ~200 cycles from a single thread inside a lane branch.
__device__ __forceinline__ void umma_f16_elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16, issued by one elected lane.
__device__ __forceinline__ void umma_f16_ts_elect(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit_elect(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

// 32 consecutive TMEM columns of this warp's 32 lanes -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld_32cols(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand tile stored with the
// 128-byte swizzle (rows of 64 bf16, 8-row atoms of 1024 bytes).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= uint64_t((smem_addr >> 4) & 0x3FFFu);   // start address
  d |= uint64_t(1u) << 16;                      // leading byte offset (unused with 128B swizzle)
  d |= uint64_t(1024u >> 4) << 32;              // stride byte offset: 8 rows x 128 B
  d |= uint64_t(1u) << 46;                      // descriptor version (sm_100)
  d |= uint64_t(2u) << 61;                      // layout: 128-byte swizzle
  return d;
}

// Instruction descriptor, kind::f16: bf16 A and B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(uint32_t M, uint32_t N) {
  return (1u << 4)            // D format: f32
         | (1u << 7)          // A format: bf16
         | (1u << 10)         // B format: bf16
         | ((N >> 3) << 17)   // N / 8
         | ((M >> 4) << 24);  // M / 16
}

}  // namespace wm
