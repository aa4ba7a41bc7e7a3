// Decode path: dequantise-and-multiply GEMV over the few rows each expert gets.
//
// Restates the arithmetic of the reference's decode kernels --
// expert_linear4 (QwenNative/kernels.metal:1186-1219) and expert_group<R, K>
// (DeepSeekNative/kernels.metal:933-987): y[r, o] = sum_k x[r, k] * w[o, k],
// fp32 accumulation, each group's E8M0 scale applied to the group's partial
// sum -- for the MXFP4 blob layout, and the same for FP8 E4M3 experts with
// fp32 128x128 block scales (each weight rounded to bf16 after scaling, as
// mimo/weights.py:17-43 decodes them) or UE8M0 32x32 block scales (the same
// rounding, deepseek_v41/dequant.py:45-50).
//
// Layout of the work: one CTA per (expert with rows, slab of outputs).  Each
// CTA reads its slab of weights once with 16-byte non-allocating loads and
// multiplies it against all of its expert's rows (up to 4 at a time, staged
// as fp32 in shared memory with a 16-byte XOR swizzle so the per-lane reads
// are bank-conflict free).  The gate/up kernel computes a gate row and its up
// row together and writes silu(g) * u (bf16) -- the reference's separate
// expert_act / swiglu_pairs dispatch is fused away.
#include <algorithm>
#include <mutex>

#include "wm_kernels.h"

namespace wm {

namespace {

constexpr int kRows = 4;     // token rows per pass
constexpr int kWarps = 8;    // warps per CTA

template <int FMT>
struct Traits;

template <>
struct Traits<kFmtMxfp4> {
  static constexpr int kVals = 32;  // values per 16-byte chunk
  static constexpr int kUnits = 8;  // 4-value (16-byte fp32) units per chunk
  __host__ __device__ static int64_t row_bytes(int cols) { return cols / 2; }
};

template <>
struct Traits<kFmtFp8B128> {
  static constexpr int kVals = 16;
  static constexpr int kUnits = 4;
  __host__ __device__ static int64_t row_bytes(int cols) { return cols; }
};

template <>
struct Traits<kFmtFp8B32> : Traits<kFmtFp8B128> {};

// Shared-memory index of value k of a staged row (16-byte units XOR-swizzled
// within each chunk by the chunk index).
template <int FMT>
__device__ __forceinline__ int xs_index(int k) {
  constexpr int V = Traits<FMT>::kVals, U = Traits<FMT>::kUnits;
  const int c = k / V, u = (k % V) / 4;
  return c * V + ((u ^ (c & (U - 1))) * 4) + (k & 3);
}

// Stage rows [first, first + n) of the sorted list as fp32.  Row r's source is
// src + row_of(r) * cols (bf16).
template <int FMT, typename RowOf>
__device__ __forceinline__ void stage_rows(float* xs, const uint16_t* src, int cols, int n, RowOf row_of) {
  const int pieces = cols / 8;  // 16-byte bf16 pieces per row
  for (int i = threadIdx.x; i < n * pieces; i += blockDim.x) {
    const int r = i / pieces, c8 = i % pieces;
    const int64_t row = row_of(r);
    const uint4 v = *reinterpret_cast<const uint4*>(src + row * cols + c8 * 8);
    const float2 a = unpack_bf16x2(v.x), b = unpack_bf16x2(v.y), c = unpack_bf16x2(v.z), d = unpack_bf16x2(v.w);
    float* dst = xs + r * cols;
    const int k0 = c8 * 8;
    *reinterpret_cast<float4*>(dst + xs_index<FMT>(k0)) = make_float4(a.x, a.y, b.x, b.y);
    *reinterpret_cast<float4*>(dst + xs_index<FMT>(k0 + 4)) = make_float4(c.x, c.y, d.x, d.y);
  }
}

// Partial dot products of one 16-byte weight chunk (4 weight rows) against
// the staged rows.  part[w][r] accumulates; wq[w] are the 4 rows' chunks.
template <int FMT>
__device__ __forceinline__ void chunk_dot(const uint4* wq, const float* xs, int cols, int c, int nr,
                                          float (&part)[4][kRows], const float (&scale)[4]) {
  constexpr int V = Traits<FMT>::kVals, U = Traits<FMT>::kUnits;
  const int sw = c & (U - 1);
  float p[4][kRows];
#pragma unroll
  for (int w = 0; w < 4; ++w)
#pragma unroll
    for (int r = 0; r < kRows; ++r) p[w][r] = 0.0f;
  if constexpr (FMT == kFmtMxfp4) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float wf[4][8];
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const uint32_t word = q == 0 ? wq[w].x : q == 1 ? wq[w].y : q == 2 ? wq[w].z : wq[w].w;
        e2m1x8_to_f32(word, wf[w]);
      }
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        if (r < nr) {
          const float* row = xs + r * cols + c * V;
          const float4 lo = *reinterpret_cast<const float4*>(row + (((2 * q) ^ sw) * 4));
          const float4 hi = *reinterpret_cast<const float4*>(row + (((2 * q + 1) ^ sw) * 4));
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            float s = p[w][r];
            s = fmaf(wf[w][0], lo.x, s); s = fmaf(wf[w][1], lo.y, s);
            s = fmaf(wf[w][2], lo.z, s); s = fmaf(wf[w][3], lo.w, s);
            s = fmaf(wf[w][4], hi.x, s); s = fmaf(wf[w][5], hi.y, s);
            s = fmaf(wf[w][6], hi.z, s); s = fmaf(wf[w][7], hi.w, s);
            p[w][r] = s;
          }
        }
      }
    }
#pragma unroll
    for (int w = 0; w < 4; ++w)
#pragma unroll
      for (int r = 0; r < kRows; ++r) part[w][r] = fmaf(p[w][r], scale[w], part[w][r]);
  } else {
    // FP8: each weight is bf16(e4m3 * block_scale); the scale cannot be
    // factored out because of that rounding.
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float wf[4][4];
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const uint32_t word = q == 0 ? wq[w].x : q == 1 ? wq[w].y : q == 2 ? wq[w].z : wq[w].w;
        e4m3x4_to_f32(word, wf[w]);
#pragma unroll
        for (int j = 0; j < 4; ++j) wf[w][j] = __uint_as_float(uint32_t(f32_to_bf16_bits(wf[w][j] * scale[w])) << 16);
      }
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        if (r < nr) {
          const float* row = xs + r * cols + c * V;
          const float4 v = *reinterpret_cast<const float4*>(row + ((q ^ sw) * 4));
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            float s = p[w][r];
            s = fmaf(wf[w][0], v.x, s); s = fmaf(wf[w][1], v.y, s);
            s = fmaf(wf[w][2], v.z, s); s = fmaf(wf[w][3], v.w, s);
            p[w][r] = s;
          }
        }
      }
    }
#pragma unroll
    for (int w = 0; w < 4; ++w)
#pragma unroll
      for (int r = 0; r < kRows; ++r) part[w][r] += p[w][r];
  }
}

// Scale of chunk c of weight row `row` (of a matrix with `cols` inputs).
template <int FMT>
__device__ __forceinline__ float chunk_scale(const uint8_t* s, int64_t row, int cols, int c) {
  if constexpr (FMT == kFmtMxfp4) {
    return e8m0_to_f32(ldg_nc_u8(s + row * (cols / 32) + c));
  } else if constexpr (FMT == kFmtFp8B32) {  // UE8M0 32x32 blocks (dequant.py:45-50)
    return e8m0_to_f32(ldg_nc_u8(s + (row / 32) * ((cols + 31) / 32) + (c * 16) / 32), true);
  } else {
    const float* sf = reinterpret_cast<const float*>(s);
    return __ldg(sf + (row / 128) * ((cols + 127) / 128) + (c * 16) / 128);
  }
}

}  // namespace

// gate/up + SwiGLU.  Grid (I / (2 * kWarps), max_unique); warp w handles the
// outputs f0 = 2 * (blockIdx.x * kWarps + w) and f0 + 1.
template <int FMT>
__global__ void __launch_bounds__(256) gemv_gateup_kernel(GemvArgs a) {
  extern __shared__ __align__(16) float xs[];
  const int u = blockIdx.y;
  if (u >= *a.plan.n_unique) return;
  const int e = a.plan.unique[u];
  const int cnt = a.plan.counts[e], off = a.plan.offsets[e];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int f0 = 2 * (blockIdx.x * kWarps + warp);
  const int H = a.H, I = a.I;
  const int gate_base = a.gate_first ? 0 : I, up_base = a.gate_first ? I : 0;
  const int64_t rb = Traits<FMT>::row_bytes(H);
  const uint8_t* w = a.wts.w13_of(e);
  const uint8_t* s = a.wts.s13_of(e);
  const int64_t rows[4] = {gate_base + f0, gate_base + f0 + 1, up_base + f0, up_base + f0 + 1};
  const int chunks = int(rb / 16);
  for (int rc = 0; rc < cnt; rc += kRows) {
    const int nr = min(kRows, cnt - rc);
    __syncthreads();
    stage_rows<FMT>(xs, a.x, H, nr, [&](int r) { return (int64_t)a.plan.row_token[off + rc + r]; });
    __syncthreads();
    if (f0 >= I) continue;
    float acc[4][kRows];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int r = 0; r < kRows; ++r) acc[i][r] = 0.0f;
    for (int c = lane; c < chunks; c += 32) {
      uint4 wq[4];
      float sc[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        wq[i] = ldg_nc_v4(w + rows[i] * rb + c * 16);
        sc[i] = chunk_scale<FMT>(s, rows[i], H, c);
      }
      chunk_dot<FMT>(wq, xs, H, c, nr, acc, sc);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int r = 0; r < kRows; ++r)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[i][r] += __shfl_xor_sync(0xffffffffu, acc[i][r], o);
    if (lane < kRows && lane < nr) {
      // lane r writes row r's two activations
      float g0 = 0, g1 = 0, u0 = 0, u1 = 0;
#pragma unroll
      for (int r = 0; r < kRows; ++r)
        if (r == lane) {
          g0 = acc[0][r]; g1 = acc[1][r]; u0 = acc[2][r]; u1 = acc[3][r];
        }
      // The MLX path rounds the gate/up product to bf16 before the activation.
      g0 = bf16_round(g0); g1 = bf16_round(g1); u0 = bf16_round(u0); u1 = bf16_round(u1);
      const uint32_t packed = pack_bf16x2(swiglu_f32(g0, u0, a.limit), swiglu_f32(g1, u1, a.limit));
      *reinterpret_cast<uint32_t*>(a.act + (int64_t)(off + rc + lane) * I + f0) = packed;
    }
  }
}

// down projection.  Weight rows of I inputs; a warp covers `slots` groups of 4
// output rows when a row is at most 16 chunks, else one group with the lanes
// striding over its chunks.
template <int FMT>
__global__ void __launch_bounds__(256) gemv_down_kernel(GemvArgs a) {
  extern __shared__ __align__(16) float xs[];
  const int u = blockIdx.y;
  if (u >= *a.plan.n_unique) return;
  const int e = a.plan.unique[u];
  const int cnt = a.plan.counts[e], off = a.plan.offsets[e];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = a.H, I = a.I;
  const int64_t rb = Traits<FMT>::row_bytes(I);
  const int chunks = int(rb / 16);
  // several rows per warp when a row is a power-of-two number (<= 16) of chunks
  const bool packed = chunks <= 16 && (chunks & (chunks - 1)) == 0;
  const int slots = packed ? 32 / chunks : 1;
  const int lanes_per_slot = packed ? chunks : 32;
  const int slot = lane / lanes_per_slot, sub = lane % lanes_per_slot;
  const int h0 = ((blockIdx.x * kWarps + warp) * slots + slot) * 4;
  const uint8_t* w = a.wts.w2_of(e);
  const uint8_t* s = a.wts.s2_of(e);
  for (int rc = 0; rc < cnt; rc += kRows) {
    const int nr = min(kRows, cnt - rc);
    __syncthreads();
    stage_rows<FMT>(xs, a.act, I, nr, [&](int r) { return (int64_t)(off + rc + r); });
    __syncthreads();
    float acc[4][kRows];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int r = 0; r < kRows; ++r) acc[i][r] = 0.0f;
    const bool active = slot < slots && h0 < H;
    if (active) {
      for (int c = sub; c < chunks; c += lanes_per_slot) {
        uint4 wq[4];
        float sc[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          wq[i] = ldg_nc_v4(w + (int64_t)(h0 + i) * rb + c * 16);
          sc[i] = chunk_scale<FMT>(s, h0 + i, I, c);
        }
        chunk_dot<FMT>(wq, xs, I, c, nr, acc, sc);
      }
    }
    // reduce over the lanes of a slot (lanes_per_slot is a power of two)
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int r = 0; r < kRows; ++r)
        for (int o = lanes_per_slot >> 1; o > 0; o >>= 1) acc[i][r] += __shfl_xor_sync(0xffffffffu, acc[i][r], o);
    if (active && sub < nr) {
      float v[4] = {0, 0, 0, 0};
#pragma unroll
      for (int r = 0; r < kRows; ++r)
        if (r == sub) {
          v[0] = acc[0][r]; v[1] = acc[1][r]; v[2] = acc[2][r]; v[3] = acc[3][r];
        }
      uint2 o;
      o.x = pack_bf16x2(v[0], v[1]);
      o.y = pack_bf16x2(v[2], v[3]);
      *reinterpret_cast<uint2*>(a.routed + (int64_t)(off + rc + sub) * H + h0) = o;
    }
  }
}

// Only ever raises the current device's limit: a handle sized for large
// shapes and a later, smaller call (another handle, the allocation-free
// entry point) launch the same kernels.
void gemv_init_attributes(int max_smem) {
  static std::mutex mu;
  static int set_to[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return;
  std::lock_guard<std::mutex> lock(mu);
  if (max_smem <= set_to[dev]) return;
  set_to[dev] = max_smem;
  cudaFuncSetAttribute(gemv_gateup_kernel<kFmtMxfp4>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(gemv_down_kernel<kFmtMxfp4>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(gemv_gateup_kernel<kFmtFp8B128>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(gemv_down_kernel<kFmtFp8B128>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(gemv_gateup_kernel<kFmtFp8B32>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(gemv_down_kernel<kFmtFp8B32>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
}

size_t gemv_smem_bytes(int H, int I) { return size_t(kRows) * std::max(H, I) * sizeof(float); }

void launch_gemv(const GemvArgs& a, int fmt, int max_unique, cudaStream_t stream, Profiler* prof) {
  const size_t smem_gu = size_t(kRows) * a.H * sizeof(float);
  const size_t smem_dn = size_t(kRows) * a.I * sizeof(float);
  dim3 grid_gu((a.I / 2 + kWarps - 1) / kWarps, max_unique);
  const int64_t rb_dn = fmt == kFmtMxfp4 ? a.I / 2 : a.I;
  const int chunks_dn = int(rb_dn / 16);
  const bool packed = chunks_dn <= 16 && (chunks_dn & (chunks_dn - 1)) == 0;
  const int slots = packed ? 32 / chunks_dn : 1;
  dim3 grid_dn((a.H / 4 + kWarps * slots - 1) / (kWarps * slots), max_unique);
  if (fmt == kFmtMxfp4) {
    prof_begin(prof, kProfGemvGateUp, stream);
    gemv_gateup_kernel<kFmtMxfp4><<<grid_gu, 256, smem_gu, stream>>>(a);
    prof_end(prof, kProfGemvGateUp, stream);
    prof_begin(prof, kProfGemvDown, stream);
    gemv_down_kernel<kFmtMxfp4><<<grid_dn, 256, smem_dn, stream>>>(a);
    prof_end(prof, kProfGemvDown, stream);
  } else if (fmt == kFmtFp8B32) {
    prof_begin(prof, kProfGemvGateUp, stream);
    gemv_gateup_kernel<kFmtFp8B32><<<grid_gu, 256, smem_gu, stream>>>(a);
    prof_end(prof, kProfGemvGateUp, stream);
    prof_begin(prof, kProfGemvDown, stream);
    gemv_down_kernel<kFmtFp8B32><<<grid_dn, 256, smem_dn, stream>>>(a);
    prof_end(prof, kProfGemvDown, stream);
  } else {
    prof_begin(prof, kProfGemvGateUp, stream);
    gemv_gateup_kernel<kFmtFp8B128><<<grid_gu, 256, smem_gu, stream>>>(a);
    prof_end(prof, kProfGemvGateUp, stream);
    prof_begin(prof, kProfGemvDown, stream);
    gemv_down_kernel<kFmtFp8B128><<<grid_dn, 256, smem_dn, stream>>>(a);
    prof_end(prof, kProfGemvDown, stream);
  }
}

}  // namespace wm
