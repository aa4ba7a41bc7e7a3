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

// Selection key and score of one expert from its logit l and bias b (0 when
// the router has none).  A softmax router takes the bias as an additive logit
// bias (the reference's Qwen router has none; the synthetic Zipf-skewed
// workload uses one); the others select on score + bias.
__device__ __forceinline__ void router_key_score(int kind, float l, float b, bool has_bias, float* key,
                                                 float* score) {
  if (kind == WM_ROUTER_SOFTMAX && has_bias) l += b;
  float s = l;
  if (kind == WM_ROUTER_SQRTSOFTPLUS)
    s = sqrtf(fmaxf(l, 0.0f) + log1pf(expf(-fabsf(l))));
  else if (kind == WM_ROUTER_SIGMOID || kind == WM_ROUTER_SIGMOID_GROUPED)
    s = 1.0f / (1.0f + expf(-l));
  *score = s;
  *key = kind == WM_ROUTER_SOFTMAX ? l : s + b;
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
    float k;
    router_key_score(kind, lg[j], bs[j], bias != nullptr, &k, &score[j]);
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

// ---- top-k of one token by a group of warps (short calls)

constexpr int kTopkGroupWarps = 4;  // warps selecting one token together
constexpr int kTopkGroupMaxK = 32;

// Candidates of one token: warp g of the group writes its K best at
// [g * K, g * K + K); u = the key's order-preserving bits (0 = none).
struct TopkCands {
  uint32_t u[kTopkGroupWarps * kTopkGroupMaxK];
  int32_t idx[kTopkGroupWarps * kTopkGroupMaxK];
  float score[kTopkGroupWarps * kTopkGroupMaxK];
};

__device__ __forceinline__ uint32_t ordered_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Phase 1: warp g (< kTopkGroupWarps) of the group selects the K best of
// experts [g * 32 EPL, (g + 1) * 32 EPL) (E <= kTopkGroupWarps * 32 * EPL)
// -- largest key first, ties to the lower expert index -- into c.
template <int EPL>
__device__ __forceinline__ void topk_group_local(const float* __restrict__ row, const TopkArgs& tk, int E, int g,
                                                 int lane, TopkCands& c) {
  const float* __restrict__ bias = tk.bias;
  const int K = tk.K, kind = tk.kind, base = g * 32 * EPL;
  float score[EPL], key[EPL], lg[EPL], bs[EPL];
  uint32_t taken = 0;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = base + lane + 32 * j;
    lg[j] = e < E ? row[e] : -INFINITY;
    bs[j] = e < E && bias != nullptr ? __ldg(bias + e) : 0.0f;
  }
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    router_key_score(kind, lg[j], bs[j], bias != nullptr, &key[j], &score[j]);
    if (base + lane + 32 * j >= E) taken |= 1u << j;
  }
  const int eligible = __reduce_add_sync(0xffffffffu, EPL - __popc(taken));
  float lbest = -INFINITY;
  int lidx = 0x7fffffff;
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
    lidx = base + lane + 32 * bj;
  };
  rescan();
  for (int k = 0; k < K; ++k) {
    if (k >= eligible) {  // fewer experts in this slice than K
      if (lane == 0) {
        c.u[g * K + k] = 0u;
        c.idx[g * K + k] = 0x7fffffff;
        c.score[g * K + k] = 0.0f;
      }
      continue;
    }
    const uint32_t u = ordered_key(lbest);
    const uint32_t top = __reduce_max_sync(0xffffffffu, u);
    const int bi = int(__reduce_min_sync(0xffffffffu, u == top ? uint32_t(lidx) : 0xffffffffu));
    if (bi - base - lane >= 0 && ((bi - base) & 31) == lane) {
      const int bj = (bi - base) >> 5;
      taken |= 1u << bj;
      float s_sel = 0.0f;
#pragma unroll
      for (int j = 0; j < EPL; ++j)
        if (j == bj) s_sel = score[j];
      c.u[g * K + k] = top;
      c.idx[g * K + k] = bi;
      c.score[g * K + k] = s_sel;
      rescan();
    }
  }
}

// Phase 2 (after the group's candidates are visible): one warp selects the K
// best of the kTopkGroupWarps * K candidates and writes the routes as
// topk_token does (same selections and weights).
__device__ __forceinline__ void topk_group_merge(const TopkCands& c, const TopkArgs& tk, int t, int lane,
                                                 int32_t* idx2 = nullptr, float* w2 = nullptr) {
  constexpr int EPL = kTopkGroupWarps * kTopkGroupMaxK / 32;
  const int K = tk.K, kind = tk.kind, n = kTopkGroupWarps * K;
  uint32_t u[EPL];
  int32_t ix[EPL];
  uint32_t taken = 0;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int q = lane + 32 * j;
    u[j] = q < n ? c.u[q] : 0u;
    ix[j] = q < n ? c.idx[q] : 0x7fffffff;
    if (q >= n || u[j] == 0u) taken |= 1u << j;
  }
  uint32_t lu = 0u;
  int lx = 0x7fffffff, lj = 0;
  auto rescan = [&]() {
    lu = 0u;
    lx = 0x7fffffff;
    lj = 0;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      if ((taken >> j) & 1u) continue;
      if (u[j] > lu || (u[j] == lu && ix[j] < lx)) {
        lu = u[j];
        lx = ix[j];
        lj = j;
      }
    }
  };
  rescan();
  float sum = 0.0f, top_logit = 0.0f, my_w = 0.0f;
  int my_idx = 0;
  for (int k = 0; k < K; ++k) {
    const uint32_t top = __reduce_max_sync(0xffffffffu, lu);
    const int bi = int(__reduce_min_sync(0xffffffffu, lu == top ? uint32_t(lx) : 0xffffffffu));
    const bool win = lu == top && lx == bi;
    const int wl = __ffs(__ballot_sync(0xffffffffu, win)) - 1;
    float s_sel = 0.0f;
    if (win) {
#pragma unroll
      for (int j = 0; j < EPL; ++j)
        if (j == lj) s_sel = c.score[lane + 32 * j];
      taken |= 1u << lj;
      rescan();
    }
    if (kind == WM_ROUTER_SOFTMAX) {
      s_sel = __uint_as_float((top & 0x80000000u) ? (top & 0x7fffffffu) : ~top);
      if (k == 0) top_logit = s_sel;
      s_sel = expf(s_sel - top_logit);
    } else {
      s_sel = __shfl_sync(0xffffffffu, s_sel, wl < 0 ? 0 : wl);
    }
    sum += s_sel;
    if (lane == k) {
      my_idx = bi;
      my_w = s_sel;
    }
  }
  if (lane < K) {
    float v = my_w;
    if (kind == WM_ROUTER_SOFTMAX)
      v = v / sum;
    else if (K > 1)
      v = v / (sum + 1e-20f);
    tk.idx[(int64_t)t * K + lane] = my_idx;
    tk.w[(int64_t)t * K + lane] = v * tk.route_scale;
    if (idx2 != nullptr) {
      idx2[(int64_t)t * K + lane] = my_idx;
      w2[(int64_t)t * K + lane] = v * tk.route_scale;
    }
  }
}

}  // namespace
}  // namespace wm
