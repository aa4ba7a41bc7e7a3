// Bit-exactness probe: dequantise one matrix to bf16 with the same decode
// helpers the GEMV / GEMM kernels use.
//
//   MXFP4      deepseek_v41/dequant.py:53-68 (w * 2^(s-127) in fp32, then bf16);
//              Metal convention per QwenNative/kernels.metal:701-702, 727
//   FP8 128    mimo/weights.py:17-43 (bf16(fp32(e4m3 * scale)))
//   FP8 32     deepseek_v41/dequant.py:45-50 (UE8M0 32x32 blocks)
#include <algorithm>

#include "wm_kernels.h"

namespace wm {

__global__ void __launch_bounds__(256) dequant_kernel(int format, const uint8_t* __restrict__ w,
                                                      const uint8_t* __restrict__ s, int64_t rows, int64_t cols,
                                                      int convention, uint16_t* __restrict__ out,
                                                      uint32_t* status) {
  const bool mlx = convention == WM_CONV_MLX;
  const int64_t per_row = cols / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < rows * per_row;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / per_row, c0 = (i % per_row) * 8;
    float v[8];
    if (format == WM_FORMAT_MXFP4) {
      const uint32_t word = *reinterpret_cast<const uint32_t*>(w + r * (cols / 2) + c0 / 2);
      e2m1x8_to_f32(word, v);
      const float sc = e8m0_to_f32(s[r * (cols / 32) + c0 / 32], mlx);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        // MLX's table holds +0 for code 8; the hardware decode gives -0.
        if (mlx && v[j] == 0.0f) v[j] = 0.0f;
        v[j] = v[j] * sc;
      }
    } else {
      const uint2 bytes = *reinterpret_cast<const uint2*>(w + r * cols + c0);
      e4m3x4_to_f32(bytes.x, v);
      e4m3x4_to_f32(bytes.y, v + 4);
      // The reference decode rejects the reserved NaN codes 0x7F / 0xFF.
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t b = (j < 4 ? bytes.x >> (8 * j) : bytes.y >> (8 * (j - 4))) & 0x7fu;
        if (b == 0x7fu) report_status(status, kStatusNanCode, uint32_t(r));
      }
      float sc;
      if (format == WM_FORMAT_FP8_B128) {
        sc = reinterpret_cast<const float*>(s)[(r / 128) * ((cols + 127) / 128) + c0 / 128];
      } else {
        sc = e8m0_to_f32(s[(r / 32) * ((cols + 31) / 32) + c0 / 32], true);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(v[j], sc);
    }
    uint4 o;
    o.x = pack_bf16x2(v[0], v[1]);
    o.y = pack_bf16x2(v[2], v[3]);
    o.z = pack_bf16x2(v[4], v[5]);
    o.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(out + r * cols + c0) = o;
  }
}

void launch_dequant(int format, const void* weight, const void* scale, int64_t rows, int64_t cols, int convention,
                    uint16_t* out, uint32_t* status, cudaStream_t stream) {
  const int64_t n = rows * (cols / 8);
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
  dequant_kernel<<<blocks, 256, 0, stream>>>(format, static_cast<const uint8_t*>(weight),
                                             static_cast<const uint8_t*>(scale), rows, cols, convention, out, status);
}

}  // namespace wm
