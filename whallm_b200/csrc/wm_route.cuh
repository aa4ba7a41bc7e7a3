// Top-k selection of one token by one warp, shared by the top-k kernel
// (wm_route.cu) and the small-call route/plan/quantise kernel (wm_bs_sm100.cu).
// The router kinds and their reference sources are listed in wm_route.cu.
#pragma once

#include "wm_kernels.h"

namespace wm {
namespace {

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

// Top-k of one token by one warp.  Lane l holds experts e = l + 32 j, j < EPL
// (E <= 32 EPL).  The results go to tk.idx / tk.w at [t * K + k] and, when
// idx2 is given, also to idx2 / w2 (same layout).
template <int EPL>
__device__ __forceinline__ void topk_token(const float* __restrict__ row, const TopkArgs& tk, int E, int t,
                                           int lane, int32_t* idx2 = nullptr, float* w2 = nullptr) {
  const float* __restrict__ bias = tk.bias;
  const int K = tk.K, kind = tk.kind, n_groups = tk.n_groups, topk_groups = tk.topk_groups;
  const float route_scale = tk.route_scale;
  int32_t* __restrict__ idx_out = tk.idx;
  float* __restrict__ w_out = tk.w;
  const int per_lane = (E + 31) / 32;
  float score[EPL], key[EPL], lg[EPL], bs[EPL];
  uint32_t taken = 0;  // bit j: slot j is selected or not eligible
  // every load first (branch-free, predicated), so they are in flight together
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = lane + 32 * j;
    const bool in = j < per_lane && e < E;
    lg[j] = in ? row[e] : -INFINITY;
    bs[j] = in && bias != nullptr ? __ldg(bias + e) : 0.0f;
  }
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = lane + 32 * j;
    float l = lg[j];
    // A softmax router takes `bias` as an additive logit bias (the reference's
    // Qwen router has none; the synthetic Zipf-skewed workload uses one).
    if (kind == WM_ROUTER_SOFTMAX && bias != nullptr) l += bs[j];
    float s = l;
    if (kind == WM_ROUTER_SQRTSOFTPLUS)
      s = sqrtf(fmaxf(l, 0.0f) + log1pf(expf(-fabsf(l))));
    else if (kind == WM_ROUTER_SIGMOID || kind == WM_ROUTER_SIGMOID_GROUPED)
      s = 1.0f / (1.0f + expf(-l));
    score[j] = s;
    float k = kind == WM_ROUTER_SOFTMAX ? l : s + bs[j];
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
  // top-k by key: every lane keeps its best remaining slot (ties to the
  // lower slot); each round two warp reductions find the
  // largest key and, among equal keys, the lowest expert index; only the
  // winner's lane rescans.  Lane k keeps selection k.
  float lbest = -INFINITY;
  int lidx = 0x7fffffff;
  // (a linear pass in slot order, strictly greater wins: the fewest
  // instructions, which is what long calls pay for)
  auto rescan = [&]() {
    float best = ((taken & 1u) != 0u) ? -INFINITY : key[0];
    int bj = 0;
#pragma unroll
    for (int j = 1; j < EPL; ++j) {
      const float kj = ((taken >> j) & 1u) ? -INFINITY : key[j];
      if (kj > best) {
        best = kj;
        bj = j;
      }
    }
    lbest = best;
    lidx = lane + 32 * bj;
  };
  // larger key -> larger unsigned value
  auto ordered = [](float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  };
  rescan();
  float sum = 0.0f, top_logit = 0.0f, my_w[2] = {0.0f, 0.0f};  // selections lane and lane + 32
  int my_idx[2] = {0, 0};
  for (int k = 0; k < K; ++k) {
    const uint32_t u = ordered(lbest);
    const uint32_t top = __reduce_max_sync(0xffffffffu, u);
    int bi = int(__reduce_min_sync(0xffffffffu, u == top ? uint32_t(lidx) : 0xffffffffu));
    if (bi < 0 || bi >= 32 * EPL) bi = 0;  // fewer eligible experts than K: cannot happen for valid shapes
    float s_sel = 0.0f;
    if (kind == WM_ROUTER_SOFTMAX) {
      // the score is the key itself: the winning key, back from its ordered bits
      s_sel = __uint_as_float((top & 0x80000000u) ? (top & 0x7fffffffu) : ~top);
      if ((bi & 31) == lane) {
        taken |= 1u << (bi >> 5);
        rescan();
      }
    } else {
      if ((bi & 31) == lane) {
        taken |= 1u << (bi >> 5);
#pragma unroll
        for (int j = 0; j < EPL; ++j)
          if (j == (bi >> 5)) s_sel = score[j];
        rescan();
      }
      s_sel = __shfl_sync(0xffffffffu, s_sel, bi & 31);
    }
    if (kind == WM_ROUTER_SOFTMAX) {
      if (k == 0) top_logit = s_sel;
      s_sel = expf(s_sel - top_logit);
    }
    sum += s_sel;
    if (lane == (k & 31)) {  // static register indices: selection k goes to slot k / 32
      if (k < 32) {
        my_idx[0] = bi;
        my_w[0] = s_sel;
      } else {
        my_idx[1] = bi;
        my_w[1] = s_sel;
      }
    }
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int k = lane + 32 * h;
    if (k < K) {
      float v = my_w[h];
      if (kind == WM_ROUTER_SOFTMAX)
        v = v / sum;
      else if (K > 1)
        v = v / (sum + 1e-20f);
      idx_out[(int64_t)t * K + k] = my_idx[h];
      w_out[(int64_t)t * K + k] = v * route_scale;
      if (idx2 != nullptr) {
        idx2[(int64_t)t * K + k] = my_idx[h];
        w2[(int64_t)t * K + k] = v * route_scale;
      }
    }
  }
}

}  // namespace
}  // namespace wm
