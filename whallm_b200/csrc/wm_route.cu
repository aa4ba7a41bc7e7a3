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

#include "wm_kernels.h"

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

// Warp-wide argmax of (key, index): larger key wins, equal keys -> lower index.
__device__ __forceinline__ void warp_argmax(float& key, int& idx) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float k2 = __shfl_xor_sync(0xffffffffu, key, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
    if (k2 > key || (k2 == key && i2 < idx)) {
      key = k2;
      idx = i2;
    }
  }
}

// One warp per token.  Lane l holds experts e = l + 32 j, j < EPL (E <= 32 EPL).
template <int EPL>
__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ logits,
                                                          const float* __restrict__ bias, int T, int E, int K,
                                                          int kind, int n_groups, int topk_groups, float route_scale,
                                                          int32_t* __restrict__ idx_out, float* __restrict__ w_out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= T) return;
  const float* row = logits + (int64_t)t * E;
  const int per_lane = (E + 31) / 32;
  float score[EPL], key[EPL];
  uint32_t taken = 0;  // bit j: slot j is selected or not eligible
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = lane + 32 * j;
    float l = (j < per_lane && e < E) ? row[e] : -INFINITY;
    // A softmax router takes `bias` as an additive logit bias (the reference's
    // Qwen router has none; the synthetic Zipf-skewed workload uses one).
    if (kind == WM_ROUTER_SOFTMAX && bias != nullptr && e < E) l += bias[e];
    float s = l;
    if (kind == WM_ROUTER_SQRTSOFTPLUS)
      s = sqrtf(fmaxf(l, 0.0f) + log1pf(expf(-fabsf(l))));
    else if (kind == WM_ROUTER_SIGMOID || kind == WM_ROUTER_SIGMOID_GROUPED)
      s = 1.0f / (1.0f + expf(-l));
    score[j] = s;
    float k = kind == WM_ROUTER_SOFTMAX ? l : s + (bias != nullptr && e < E ? bias[e] : 0.0f);
    if (!(j < per_lane && e < E)) {
      k = -INFINITY;
      taken |= 1u << j;
    }
    key[j] = k;
  }
  if (kind == WM_ROUTER_SIGMOID_GROUPED && n_groups > 1) {
    // Group score: sum of the two largest biased scores of its E / n_groups
    // contiguous experts.  The top `topk_groups` groups stay eligible.
    const int per_group = E / n_groups;
    uint32_t group_keep = 0;  // bit g (n_groups <= 32)
    float gscore_lane = -INFINITY;  // lane g holds group g's score
    for (int g = 0; g < n_groups; ++g) {
      float best = -INFINITY, second = -INFINITY;
#pragma unroll
      for (int j = 0; j < EPL; ++j) {
        const int e = lane + 32 * j;
        if (j < per_lane && e < E && e / per_group == g) {
          const float v = key[j];
          if (v > best) {
            second = best;
            best = v;
          } else if (v > second) {
            second = v;
          }
        }
      }
      // merge (best, second) across lanes
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float b2 = __shfl_xor_sync(0xffffffffu, best, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, second, o);
        const float nb = fmaxf(best, b2);
        const float ns = fmaxf(fminf(best, b2), fmaxf(second, s2));
        best = nb;
        second = ns;
      }
      if (lane == g) gscore_lane = best + second;
    }
    for (int i = 0; i < topk_groups; ++i) {
      float k = (group_keep >> lane) & 1u ? -INFINITY : gscore_lane;
      int gi = lane < n_groups ? lane : 0x7fffffff;
      if (lane >= n_groups) k = -INFINITY;
      warp_argmax(k, gi);
      group_keep |= 1u << gi;
    }
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      const int e = lane + 32 * j;
      if (j < per_lane && e < E && !((group_keep >> (e / per_group)) & 1u)) taken |= 1u << j;
    }
  }
  // top-k by key
  float sum = 0.0f, top_logit = 0.0f;
  for (int k = 0; k < K; ++k) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      const int e = lane + 32 * j;
      if (!((taken >> j) & 1u) && (key[j] > best || (key[j] == best && e < bi))) {
        best = key[j];
        bi = e;
      }
    }
    warp_argmax(best, bi);
    if (bi == 0x7fffffff) bi = 0;  // fewer eligible experts than K: cannot happen for valid shapes
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    float s_sel = 0.0f;
#pragma unroll
    for (int j = 0; j < EPL; ++j)
      if (lane + 32 * j == bi) s_sel = score[j];
    s_sel = __shfl_sync(0xffffffffu, s_sel, bi & 31);
    if (kind == WM_ROUTER_SOFTMAX) {
      if (k == 0) top_logit = s_sel;
      s_sel = expf(s_sel - top_logit);
    }
    sum += s_sel;
    if (lane == 0) {
      idx_out[(int64_t)t * K + k] = bi;
      w_out[(int64_t)t * K + k] = s_sel;
    }
  }
  __syncwarp();
  if (lane == 0) {
    for (int k = 0; k < K; ++k) {
      float v = w_out[(int64_t)t * K + k];
      if (kind == WM_ROUTER_SOFTMAX)
        v = v / sum;
      else if (K > 1)
        v = v / (sum + 1e-20f);
      w_out[(int64_t)t * K + k] = v * route_scale;
    }
  }
}

size_t router_smem_bytes(int H) { return size_t(8) * H * 2; }

void router_init_attributes(int max_hidden) {
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
                          float* logits, float* sg, cudaStream_t stream) {
  const int rows = E + (sg_w != nullptr ? 1 : 0);
  // experts in groups of 8 (one per warp) x token chunks of 8 (up to 64 chunks in flight)
  const dim3 blocks((rows + 7) / 8, std::min((T + 7) / 8, 64));
  const size_t smem = size_t(8) * H * 2;
  router_logits_kernel<<<blocks, 256, smem, stream>>>(x, wr, sg_w, T, H, E, logits, sg);
}

void launch_router_topk(const float* logits, const float* bias, int T, int E, int K, int kind, int n_groups,
                        int topk_groups, float route_scale, int32_t* idx, float* w, cudaStream_t stream) {
  const int blocks = (T + 7) / 8;
  if (E <= 256)
    router_topk_kernel<8><<<blocks, 256, 0, stream>>>(logits, bias, T, E, K, kind, n_groups, topk_groups,
                                                       route_scale, idx, w);
  else if (E <= 512)
    router_topk_kernel<16><<<blocks, 256, 0, stream>>>(logits, bias, T, E, K, kind, n_groups, topk_groups,
                                                        route_scale, idx, w);
  else
    router_topk_kernel<32><<<blocks, 256, 0, stream>>>(logits, bias, T, E, K, kind, n_groups, topk_groups,
                                                        route_scale, idx, w);
}

}  // namespace wm
