// Router: logits = x . W_r^T (bf16 operands, fp32 accumulation) and the top-k
// selection of the four router kinds of the reference.
//
//   softmax (Qwen)            qwen4_exp.py:1009-1013, 1036-1047; QwenNative/engine.mm:2085-2101
//   sqrt-softplus (V4.1)      deepseek_v41/moe.py:58-74; DeepSeekNative/engine.mm:1863-1890
//   sigmoid + bias (MiMo)     mimo/model.py:139-150
//   sigmoid, group-limited    DeepSeek-V3 "noaux_tc" selection (not in the reference)
//
// Selection ties go to the lower expert index (DeepSeekNative/engine.mm:1880);
// the reference's argpartition leaves tie order unspecified.
#include <algorithm>
#include <mutex>

#include "wm_kernels.h"
#include "wm_route.cuh"

namespace wm {

// One warp per router row (expert e, or row E = the shared-expert gate g).
// x is staged 8 tokens at a time in shared memory as bf16.
__global__ void __launch_bounds__(256) router_logits_kernel(const uint16_t* __restrict__ x,
                                                            const uint16_t* __restrict__ wr,
                                                            const uint16_t* __restrict__ sg_w, int T, int H, int E,
                                                            float* __restrict__ logits, float* __restrict__ sg) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem_raw);  // [8][H]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  const int rows_total = E + (sg_w != nullptr ? 1 : 0);
  const uint16_t* w = row < E ? wr + (int64_t)row * H : sg_w;
  for (int t0 = blockIdx.y * 8; t0 < T; t0 += 8 * gridDim.y) {
    const int nt = min(8, T - t0);
    __syncthreads();
    // stage x[t0 .. t0 + nt) (16-byte pieces)
    const int pieces = nt * H / 8;
    for (int i = threadIdx.x; i < pieces; i += blockDim.x) {
      const int r = i / (H / 8), c = i % (H / 8);
      reinterpret_cast<uint4*>(xs + r * H)[c] = reinterpret_cast<const uint4*>(x + (int64_t)(t0 + r) * H)[c];
    }
    __syncthreads();
    if (row >= rows_total) continue;
    float acc[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) acc[r] = 0.0f;
    for (int c = lane; c < H / 8; c += 32) {
      const uint4 wv = *reinterpret_cast<const uint4*>(w + c * 8);
      float wf[8];
      float2 p;
      p = unpack_bf16x2(wv.x); wf[0] = p.x; wf[1] = p.y;
      p = unpack_bf16x2(wv.y); wf[2] = p.x; wf[3] = p.y;
      p = unpack_bf16x2(wv.z); wf[4] = p.x; wf[5] = p.y;
      p = unpack_bf16x2(wv.w); wf[6] = p.x; wf[7] = p.y;
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        if (r < nt) {
          const uint4 xv = reinterpret_cast<const uint4*>(xs + r * H)[c];
          float2 a;
          float s = 0.0f;
          a = unpack_bf16x2(xv.x); s = fmaf(a.x, wf[0], s); s = fmaf(a.y, wf[1], s);
          a = unpack_bf16x2(xv.y); s = fmaf(a.x, wf[2], s); s = fmaf(a.y, wf[3], s);
          a = unpack_bf16x2(xv.z); s = fmaf(a.x, wf[4], s); s = fmaf(a.y, wf[5], s);
          a = unpack_bf16x2(xv.w); s = fmaf(a.x, wf[6], s); s = fmaf(a.y, wf[7], s);
          acc[r] += s;
        }
      }
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      float v = acc[r];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0 && r < nt) {
        if (row < E)
          logits[(int64_t)(t0 + r) * E + row] = v;
        else
          sg[t0 + r] = 1.0f / (1.0f + expf(-v));
      }
    }
  }
}

// 8 bf16 of x times the row's rstd times 8 bf16 norm weights, rounded to bf16:
// ((x * rstd) * w), the order of the reference's rms_norm kernels.
__device__ __forceinline__ uint4 rms_scale8(uint4 xv, uint4 wv, float r) {
  const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w}, ws[4] = {wv.x, wv.y, wv.z, wv.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 a = unpack_bf16x2(xs[i]), b = unpack_bf16x2(ws[i]);
    o[i] = pack_bf16x2(a.x * r * b.x, a.y * r * b.y);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Shared-expert gate of one token by one warp: sigmoid(x[t] . g), lanes over
// 8-element pieces, fp32, xor-tree reduction (shared_gate_kernel uses the same).
__device__ __forceinline__ float shared_gate_row(const uint16_t* __restrict__ xr, const uint16_t* __restrict__ g,
                                                 int H, int lane, const uint16_t* __restrict__ nw = nullptr,
                                                 float r = 1.0f) {
  float acc = 0.0f;
  for (int c = lane; c < H / 8; c += 32) {
    const uint4 wv = *reinterpret_cast<const uint4*>(g + c * 8);
    uint4 xv = *reinterpret_cast<const uint4*>(xr + c * 8);
    if (nw != nullptr) xv = rms_scale8(xv, *reinterpret_cast<const uint4*>(nw + c * 8), r);
    float2 p, a;
    float s = 0.0f;
    p = unpack_bf16x2(wv.x); a = unpack_bf16x2(xv.x); s = fmaf(a.x, p.x, s); s = fmaf(a.y, p.y, s);
    p = unpack_bf16x2(wv.y); a = unpack_bf16x2(xv.y); s = fmaf(a.x, p.x, s); s = fmaf(a.y, p.y, s);
    p = unpack_bf16x2(wv.z); a = unpack_bf16x2(xv.z); s = fmaf(a.x, p.x, s); s = fmaf(a.y, p.y, s);
    p = unpack_bf16x2(wv.w); a = unpack_bf16x2(xv.w); s = fmaf(a.x, p.x, s); s = fmaf(a.y, p.y, s);
    acc += s;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  return 1.0f / (1.0f + expf(-acc));
}

// Top-k: one warp per token, two per block, so short calls spread over SMs.
template <int EPL>
__global__ void __launch_bounds__(64) router_topk_kernel(const float* __restrict__ logits, int T, int E,
                                                          const TopkArgs tk) {
  const int t = blockIdx.x * 2 + (threadIdx.x >> 5);
  if (t >= T) return;
  topk_token<EPL>(logits + int64_t(t) * E, tk, E, t, threadIdx.x & 31);
}

constexpr int kRouterWarps = 8;
constexpr int kRouterSteps = 4;  // 64-K steps per warp per batch of loads

// Logits of short calls on warp MMAs (mma.sync.m16n8k16, bf16 operands,
// fp32 accumulation).  A CTA computes 16 tokens x 8 experts; its 8 warps split
// H into 8 slices (all of a slice's loads go out before its MMAs), and warp 0
// adds the 8 partial tiles in slice order.  Per 64-K step lane (g, t) reads 16
// contiguous K (32 bytes) of token rows g, g + 8 and of expert row g; MMA step
// j takes K offsets 16t + 4j .. 16t + 4j + 3 of them for both operands.  The
// CTA column past the experts computes the shared-expert gate, a warp per token.
//
// With a norm weight `nw` the layer input is RMSNorm(x): every CTA first forms
// the 1 / sqrt(mean(x^2) + eps) of its 16 rows the same way (lane partial sums
// over the lane's K pieces, the t lanes, then the 8 warps, in a fixed order),
// so every CTA of a token tile normalises identically; the A operands are
// bf16((x * rstd) * w), and the CTA of expert group 0 writes them to xn for
// the expert kernels (DeepSeekNative/kernels.metal:443-465, rms_norm_tg; the
// norm before the gate, engine.mm:1846; GroupRMSNorm, qwen4_exp.py:93-117).
__global__ void __launch_bounds__(32 * kRouterWarps) router_logits_mma_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ wr, const uint16_t* __restrict__ sg_w, int T, int H,
    int E, float* __restrict__ logits, float* __restrict__ sg, const uint16_t* __restrict__ nw, float eps,
    uint16_t* __restrict__ xn) {
  __shared__ float part[kRouterWarps][32][4];
  __shared__ float ssq[kRouterWarps][16];
  __shared__ float rstd_s[16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int t0 = blockIdx.y * 16;
  const int ra = min(t0 + g, T - 1), rb = min(t0 + g + 8, T - 1);  // rows past T read row T-1, not stored
  const int steps = H / 64 / kRouterWarps;                          // 64-K steps of this warp's slice
  const int64_t k0 = int64_t(warp) * steps * 8;                     // first uint4 of the slice
  const uint4* xa = reinterpret_cast<const uint4*>(x + int64_t(ra) * H) + k0 + 2 * t;
  const uint4* xb = reinterpret_cast<const uint4*>(x + int64_t(rb) * H) + k0 + 2 * t;
  const uint4* np = nw != nullptr ? reinterpret_cast<const uint4*>(nw) + k0 + 2 * t : nullptr;
  float ra_r = 1.0f, rb_r = 1.0f;
  if (nw != nullptr) {
    float sa = 0.0f, sb = 0.0f;
    for (int k = 0; k < steps; ++k)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint4 va = __ldg(xa + 8 * k + h), vb = __ldg(xb + 8 * k + h);
        const uint32_t wa[4] = {va.x, va.y, va.z, va.w}, wb[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 fa = unpack_bf16x2(wa[i]), fb = unpack_bf16x2(wb[i]);
          sa = fmaf(fa.y, fa.y, fmaf(fa.x, fa.x, sa));
          sb = fmaf(fb.y, fb.y, fmaf(fb.x, fb.x, sb));
        }
      }
    sa += __shfl_xor_sync(0xffffffffu, sa, 1);
    sb += __shfl_xor_sync(0xffffffffu, sb, 1);
    sa += __shfl_xor_sync(0xffffffffu, sa, 2);
    sb += __shfl_xor_sync(0xffffffffu, sb, 2);
    if (t == 0) {
      ssq[warp][g] = sa;
      ssq[warp][g + 8] = sb;
    }
    __syncthreads();
    if (threadIdx.x < 16) {
      float total = 0.0f;
      for (int w8 = 0; w8 < kRouterWarps; ++w8) total += ssq[w8][threadIdx.x];
      rstd_s[threadIdx.x] = 1.0f / sqrtf(total / float(H) + eps);
    }
    __syncthreads();
    ra_r = rstd_s[g];
    rb_r = rstd_s[g + 8];
  }
  if (int(blockIdx.x) * 8 >= E) {  // shared-expert gate, on the normalised rows when there is a norm
    for (int r = warp; r < 16; r += kRouterWarps) {
      if (t0 + r >= T) continue;
      const float v = shared_gate_row(x + int64_t(t0 + r) * H, sg_w, H, lane, nw, nw != nullptr ? rstd_s[r] : 1.0f);
      if (lane == 0) sg[t0 + r] = v;
    }
    return;
  }
  const int e = blockIdx.x * 8 + g;
  const uint4* wp = reinterpret_cast<const uint4*>(wr + int64_t(e) * H) + k0 + 2 * t;
  const bool write_xn = nw != nullptr && xn != nullptr && blockIdx.x == 0;
  uint4* xna = write_xn ? reinterpret_cast<uint4*>(xn + int64_t(t0 + g) * H) + k0 + 2 * t : nullptr;
  uint4* xnb = write_xn ? reinterpret_cast<uint4*>(xn + int64_t(t0 + g + 8) * H) + k0 + 2 * t : nullptr;
  float d[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
  for (int k = 0; k < steps; k += kRouterSteps) {
    uint4 a[kRouterSteps][2], b[kRouterSteps][2], w[kRouterSteps][2];
#pragma unroll
    for (int i = 0; i < kRouterSteps; ++i)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const bool in = k + i < steps;
        a[i][h] = in ? __ldg(xa + 8 * (k + i) + h) : make_uint4(0, 0, 0, 0);
        b[i][h] = in ? __ldg(xb + 8 * (k + i) + h) : make_uint4(0, 0, 0, 0);
        w[i][h] = in ? __ldg(wp + 8 * (k + i) + h) : make_uint4(0, 0, 0, 0);
      }
    if (nw != nullptr) {
#pragma unroll
      for (int i = 0; i < kRouterSteps; ++i)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (k + i >= steps) continue;
          const uint4 nv = __ldg(np + 8 * (k + i) + h);
          a[i][h] = rms_scale8(a[i][h], nv, ra_r);
          b[i][h] = rms_scale8(b[i][h], nv, rb_r);
          if (write_xn) {
            if (t0 + g < T) xna[8 * (k + i) + h] = a[i][h];
            if (t0 + g + 8 < T) xnb[8 * (k + i) + h] = b[i][h];
          }
        }
    }
#pragma unroll
    for (int i = 0; i < kRouterSteps; ++i) {
      const uint32_t av[8] = {a[i][0].x, a[i][0].y, a[i][0].z, a[i][0].w, a[i][1].x, a[i][1].y, a[i][1].z, a[i][1].w};
      const uint32_t bv[8] = {b[i][0].x, b[i][0].y, b[i][0].z, b[i][0].w, b[i][1].x, b[i][1].y, b[i][1].z, b[i][1].w};
      const uint32_t wv[8] = {w[i][0].x, w[i][0].y, w[i][0].z, w[i][0].w, w[i][1].x, w[i][1].y, w[i][1].z, w[i][1].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {  // word 2j = K 4j, 4j+1; word 2j+1 = K 4j+2, 4j+3
        float* dd = d[j & 1];
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
            "{%0, %1, %2, %3};"
            : "+f"(dd[0]), "+f"(dd[1]), "+f"(dd[2]), "+f"(dd[3])
            : "r"(av[2 * j]), "r"(bv[2 * j]), "r"(av[2 * j + 1]), "r"(bv[2 * j + 1]), "r"(wv[2 * j]),
              "r"(wv[2 * j + 1]));
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) part[warp][lane][i] = d[0][i] + d[1][i];
  __syncthreads();
  if (warp != 0) return;
  float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int w8 = 0; w8 < kRouterWarps; ++w8)
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] += part[w8][lane][i];
  const int ec = blockIdx.x * 8 + 2 * t;  // D: rows g / g + 8 = tokens, columns 2t, 2t+1 = experts
  if (t0 + g < T) *reinterpret_cast<float2*>(logits + int64_t(t0 + g) * E + ec) = make_float2(v[0], v[1]);
  if (t0 + g + 8 < T) *reinterpret_cast<float2*>(logits + int64_t(t0 + g + 8) * E + ec) = make_float2(v[2], v[3]);
}

// RMSNorm of whole rows for calls the fused kernel does not take: one CTA of
// 256 threads per token, partial sums in a fixed order (rms_norm_tg).
__global__ void __launch_bounds__(256) rmsnorm_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ nw,
                                                     int H, float eps, uint16_t* __restrict__ xn) {
  __shared__ float part[8];
  const int row = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint4* xr = reinterpret_cast<const uint4*>(x + int64_t(row) * H);
  float ss = 0.0f;
  for (int c = threadIdx.x; c < H / 8; c += 256) {
    const uint4 v = xr[c];
    const uint32_t ws[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16x2(ws[i]);
      ss = fmaf(f.y, f.y, fmaf(f.x, f.x, ss));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) part[warp] = ss;
  __syncthreads();
  float total = 0.0f;
  for (int k = 0; k < 8; ++k) total += part[k];
  const float r = 1.0f / sqrtf(total / float(H) + eps);
  uint4* out = reinterpret_cast<uint4*>(xn + int64_t(row) * H);
  const uint4* wv = reinterpret_cast<const uint4*>(nw);
  for (int c = threadIdx.x; c < H / 8; c += 256) out[c] = rms_scale8(xr[c], wv[c], r);
}

void launch_rmsnorm(const uint16_t* x, const uint16_t* nw, int T, int H, float eps, uint16_t* xn,
                    cudaStream_t stream) {
  rmsnorm_kernel<<<T, 256, 0, stream>>>(x, nw, H, eps, xn);
}

bool router_logits_fused_ok(int T, int H, int E) { return H % (64 * kRouterWarps) == 0 && E % 8 == 0 && T <= 4096; }

size_t router_smem_bytes(int H) { return size_t(8) * H * 2; }

// Only ever raises the current device's limit (see gemv_init_attributes).
void router_init_attributes(int max_hidden) {
  static std::mutex mu;
  static int set_to[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return;
  std::lock_guard<std::mutex> lock(mu);
  if (max_hidden <= set_to[dev]) return;
  set_to[dev] = max_hidden;
  cudaFuncSetAttribute(router_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       int(router_smem_bytes(max_hidden)));
}

// sg[t] = sigmoid(x[t] . g) alone, one warp per token, with the per-lane
// order and the xor reduction of router_logits_kernel's gate row (the same
// bits), for calls whose logits come from elsewhere.
__global__ void __launch_bounds__(256) shared_gate_kernel(const uint16_t* __restrict__ x,
                                                          const uint16_t* __restrict__ g, int T, int H,
                                                          float* __restrict__ sg) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  const uint16_t* xr = x + (int64_t)t * H;
  float acc = 0.0f;
  for (int c = lane; c < H / 8; c += 32) {
    const uint4 wv = *reinterpret_cast<const uint4*>(g + c * 8);
    const uint4 xv = *reinterpret_cast<const uint4*>(xr + c * 8);
    float2 p, a;
    float s = 0.0f;
    p = unpack_bf16x2(wv.x); a = unpack_bf16x2(xv.x); s = fmaf(a.x, p.x, s); s = fmaf(a.y, p.y, s);
    p = unpack_bf16x2(wv.y); a = unpack_bf16x2(xv.y); s = fmaf(a.x, p.x, s); s = fmaf(a.y, p.y, s);
    p = unpack_bf16x2(wv.z); a = unpack_bf16x2(xv.z); s = fmaf(a.x, p.x, s); s = fmaf(a.y, p.y, s);
    p = unpack_bf16x2(wv.w); a = unpack_bf16x2(xv.w); s = fmaf(a.x, p.x, s); s = fmaf(a.y, p.y, s);
    acc += s;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) sg[t] = 1.0f / (1.0f + expf(-acc));
}

void launch_shared_gate(const uint16_t* x, const uint16_t* g, int T, int H, float* sg, cudaStream_t stream) {
  shared_gate_kernel<<<(T + 7) / 8, 256, 0, stream>>>(x, g, T, H, sg);
}

void launch_router_logits(const uint16_t* x, const uint16_t* wr, const uint16_t* sg_w, int T, int H, int E,
                          float* logits, float* sg, cudaStream_t stream, const uint16_t* nw, float eps,
                          uint16_t* xn) {
  if (router_logits_fused_ok(T, H, E)) {
    const dim3 blocks(E / 8 + (sg_w != nullptr ? 1 : 0), (T + 15) / 16);
    router_logits_mma_kernel<<<blocks, 32 * kRouterWarps, 0, stream>>>(x, wr, sg_w, T, H, E, logits, sg, nw, eps,
                                                                        xn);
    return;
  }
  const int rows = E + (sg_w != nullptr ? 1 : 0);
  // experts in groups of 8 (one per warp) x token chunks of 8 (up to 64 chunks in flight)
  const dim3 blocks((rows + 7) / 8, std::min((T + 7) / 8, 64));
  const size_t smem = size_t(8) * H * 2;
  router_logits_kernel<<<blocks, 256, smem, stream>>>(x, wr, sg_w, T, H, E, logits, sg);
}

// Top-k of short calls: a block of kTopkGroupWarps warps per token, each warp
// selecting from a quarter of the experts, then one warp from their
// candidates -- the same selections and weights as router_topk_kernel, with
// the chain of selection rounds split over two shorter chains.
template <int EPL>
__global__ void __launch_bounds__(32 * kTopkGroupWarps) router_topk_group_kernel(const float* __restrict__ logits,
                                                                               int T, int E, const TopkArgs tk) {
  __shared__ TopkCands c;
  const int t = blockIdx.x, g = threadIdx.x >> 5, lane = threadIdx.x & 31;
  topk_group_local<EPL>(logits + int64_t(t) * E, tk, E, g, lane, c);
  __syncthreads();
  if (g == 0) topk_group_merge(c, tk, t, lane);
}

bool router_topk_group_ok(int T, int K, int E, int kind) {
  return T <= kTopkGroupCalls && K >= 1 && K <= kTopkGroupMaxK && E <= kTopkGroupWarps * 32 * 8 &&
         kind != WM_ROUTER_SIGMOID_GROUPED;
}

void launch_router_topk(const float* logits, int T, int E, const TopkArgs& tk, cudaStream_t stream) {
  if (router_topk_group_ok(T, tk.K, E, tk.kind)) {
    const int threads = 32 * kTopkGroupWarps;
    if (E <= kTopkGroupWarps * 64)
      router_topk_group_kernel<2><<<T, threads, 0, stream>>>(logits, T, E, tk);
    else if (E <= kTopkGroupWarps * 128)
      router_topk_group_kernel<4><<<T, threads, 0, stream>>>(logits, T, E, tk);
    else
      router_topk_group_kernel<8><<<T, threads, 0, stream>>>(logits, T, E, tk);
    return;
  }
  const int blocks = (T + 1) / 2;
  if (E <= 256)
    router_topk_kernel<8><<<blocks, 64, 0, stream>>>(logits, T, E, tk);
  else if (E <= 512)
    router_topk_kernel<16><<<blocks, 64, 0, stream>>>(logits, T, E, tk);
  else
    router_topk_kernel<32><<<blocks, 64, 0, stream>>>(logits, T, E, tk);
}

}  // namespace wm
