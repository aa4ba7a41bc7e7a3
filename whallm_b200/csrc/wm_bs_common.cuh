// Device helpers shared by the block-scaled tcgen05 kernels (kind::mxf8f6f4
// with UE8M0 scale factors): TMA / bulk copies into shared memory, the
// scale-factor atom copy into TMEM, the MMA itself (one elected lane, issued
// warp-wide) and the hi / lo E4M3 split of activation rows.
//
// Scale-factor atoms: 512 bytes = 32 rows of 16 bytes; row r holds, for the
// operand rows r, r + 32, r + 64, r + 96, the UE8M0 bytes of four 32-K
// blocks (byte 4 m + kk for row r + 32 m, block kk).  tcgen05.cp.32x128b.warpx4
// copies an atom to four TMEM columns of every lane quarter; operand row n of
// an MMA then reads column c0 + n / 32, lane n % 32, byte kk (the scale-factor
// id).  Operands of 256 rows use two atoms in eight columns.
#pragma once

#include <cuda.h>

#include "wm_kernels.h"

namespace wm {
namespace {

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* tmap, int x, int y, int z, int w,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(dst),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_2d_s(uint32_t dst, const void* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dst),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory descriptor of a scale-factor atom for tcgen05.cp: 32 rows of
// 16 bytes, no swizzle, 8-row core matrices 128 bytes apart.
__device__ __forceinline__ uint64_t sf_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= uint64_t((addr >> 4) & 0x3FFFu);
  d |= uint64_t(128u >> 4) << 16;
  d |= uint64_t(128u >> 4) << 32;
  d |= uint64_t(1u) << 46;
  return d;
}

// Warp-wide issue: every lane of a converged warp executes these and one
// elected lane issues the instruction (far cheaper than a one-lane branch).
__device__ __forceinline__ void sf_copy_elect(uint32_t taddr, uint64_t desc) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;\n\t}" ::"r"(taddr),
      "l"(desc)
      : "memory");
}

__device__ __forceinline__ void bs_mma_elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t sfa, uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}

__device__ __forceinline__ void sts_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ uint32_t lds_b32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}


// ---- the hi / lo E4M3 parts

// Power-of-two scale for a 32-element block of largest magnitude `amax`: the
// smallest 2^e with amax / 2^e <= 448 (E4M3's largest finite value), as the
// UE8M0 byte e + 127 (clamped to [1, 254]; 1 for an all-zero block).
__device__ __forceinline__ uint32_t e4m3_block_scale(float amax) {
  if (!(amax > 0.0f)) return 1u;
  const int eb = int((__float_as_uint(amax) >> 23) & 0xFFu);  // biased exponent of amax
  if (eb == 0) return 1u;
  // amax in [2^(eb-127), 2^(eb-126)); with e = eb - 127 - 8, amax / 2^e in [256, 512)
  int e = eb - 127 - 8;
  if (amax > 448.0f * __uint_as_float(uint32_t(e + 127) << 23)) e += 1;
  return uint32_t(min(max(e + 127, 1), 254));
}

// Two floats -> two E4M3 bytes (round to nearest even, saturating), low byte = a.
__device__ __forceinline__ uint32_t to_e4m3x2(float a, float b) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(b), "f"(a));
  return r;
}

// 32 values -> hi and lo E4M3 bytes (32 each) and their UE8M0 scale bytes.
__device__ __forceinline__ void split_block(const float* v, uint32_t* hi, uint32_t* lo, uint32_t* shi, uint32_t* slo) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const uint32_t bh = e4m3_block_scale(amax);
  const float inv_h = __uint_as_float((254u - bh) << 23), sc_h = __uint_as_float(bh << 23);
  float r[32];
  float rmax = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    const uint32_t p01 = to_e4m3x2(v[i] * inv_h, v[i + 1] * inv_h);
    const uint32_t p23 = to_e4m3x2(v[i + 2] * inv_h, v[i + 3] * inv_h);
    hi[i / 4] = p01 | (p23 << 16);
    float q[4];
    e4m3x4_to_f32(hi[i / 4], q);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      r[i + j] = v[i + j] - q[j] * sc_h;  // exact: x and its rounded part share a binade
      rmax = fmaxf(rmax, fabsf(r[i + j]));
    }
  }
  const uint32_t bl = e4m3_block_scale(rmax);
  const float inv_l = __uint_as_float((254u - bl) << 23);
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    const uint32_t p01 = to_e4m3x2(r[i] * inv_l, r[i + 1] * inv_l);
    const uint32_t p23 = to_e4m3x2(r[i + 2] * inv_l, r[i + 3] * inv_l);
    lo[i / 4] = p01 | (p23 << 16);
  }
  *shi = bh;
  *slo = bl;
}

// Byte offset of (row n of a 32-row part image, 16-byte chunk c) in the
// 128-byte swizzled layout the MMA reads (chunk c of row n at c ^ (n % 8)).
__device__ __forceinline__ int image_off(int n, int c) { return n * 128 + ((c ^ (n & 7)) << 4); }

}  // namespace
}  // namespace wm
