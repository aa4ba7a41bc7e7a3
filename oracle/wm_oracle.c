/*
 * wm_oracle.c -- CPU restatement of Whallm's MoE expert-FFN arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * path in whallm_b200/csrc and the timed CPU baseline of bench.py.  Only
 * tests/, __graft_entry__.smoke() and bench.py's cpu-baseline / reference arm
 * may load it.  The product library never links or calls it.
 *
 * Every function cites the reference file:line it restates (paths are inside
 * the yanun0323/Whallm project):
 *
 *   E2M1 / E8M0 decode ...... runtime/deepseek_v4_ssd/deepseek_v41/dequant.py:27-68
 *                             Native/QwenNative/kernels.metal:140-144, 701-702
 *   FP8 E4M3 decode ......... runtime/deepseek_v4_ssd/mimo/weights.py:17-43
 *                             runtime/deepseek_v4_ssd/deepseek_v41/dequant.py:45-50
 *                             Sources/DeepSeekRepack/MXFP4.swift:96-107
 *   MXFP4 quantiser ......... Sources/DeepSeekRepack/MXFP4.swift:4-131
 *   MXFP4 linear ............ runtime/deepseek_v4_ssd/model.py:504-513 (mx.quantized_matmul
 *                             mode="mxfp4", group 32), Native/QwenNative/kernels.metal:1186-1219
 *   SwiGLU .................. runtime/deepseek_v4_ssd/qwen4_exp.py:815-818 (gate rows first)
 *                             runtime/deepseek_v4_ssd/deepseek_v41/moe.py:30-43 (clamped)
 *                             runtime/deepseek_v4_ssd/model.py:452-461 (w13 = [w3; w1], up first)
 *   routers ................. qwen4_exp.py:1009-1013, 1036-1047; Native/QwenNative/engine.mm:2085-2101
 *                             deepseek_v41/moe.py:46-74; Native/DeepSeekNative/engine.mm:1863-1890
 *                             mimo/model.py:132-150
 *   combine ................. qwen4_exp.py:1049-1051; deepseek_v41/moe.py:105-112;
 *                             Native/QwenNative/kernels.metal:185-194
 *
 * Numerics of the layer restatement (wmo_moe_forward): bf16 activations in,
 * products of exact dequantised weights accumulated in double, and rounded to
 * bf16 at the points where the MLX path returns bf16 arrays (the gate/up
 * product, the SwiGLU result and each expert's output rows); the combine is an
 * fp32 sum in k order.
 * WMO_NUMERICS_FP32 keeps every intermediate in fp32 instead, as the native
 * Metal engines do.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define WMO_EXPORT __attribute__((visibility("default")))

enum { WMO_CONV_MLX = 0, WMO_CONV_METAL = 1 };
enum { WMO_LAYOUT_QWEN_GATE_UP_MXFP4 = 0, WMO_LAYOUT_DS_W13_MXFP4 = 1, WMO_LAYOUT_W13_FP8_B128 = 2, WMO_LAYOUT_W13_FP8_B32 = 3 };
enum { WMO_ROUTER_SOFTMAX = 0, WMO_ROUTER_SQRTSOFTPLUS = 1, WMO_ROUTER_SIGMOID = 2, WMO_ROUTER_SIGMOID_GROUPED = 3 };
enum { WMO_SHARED_NONE = 0, WMO_SHARED_SIGMOID_GATE = 1, WMO_SHARED_ONE = 2 };
enum { WMO_NUMERICS_BF16 = 0, WMO_NUMERICS_FP32 = 1 };

/* ------------------------------------------------------------------ scalar formats */

static inline float bf16_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* Round to nearest even; NaN stays NaN (quiet). */
static inline uint16_t f32_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

static inline float round_bf16(double v) { return bf16_f32(f32_bf16((float)v)); }

WMO_EXPORT uint16_t wmo_f32_to_bf16(float f) { return f32_bf16(f); }
WMO_EXPORT float wmo_bf16_to_f32(uint16_t b) { return bf16_f32(b); }

/* E2M1 code -> value.  dequant.py:27-28 maps code 8 to +0.0; the Metal table
   FP4_VALUES (QwenNative/kernels.metal:701-702) holds -0.0 there. */
WMO_EXPORT float wmo_e2m1(uint32_t code, int convention) {
  static const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  code &= 15u;
  float v = mag[code & 7u];
  if (code & 8u) {
    if (code == 8u) return convention == WMO_CONV_METAL ? -0.0f : 0.0f;
    return -v;
  }
  return v;
}

/* E8M0 byte -> 2^(b-127).  dequant.py:31-35 computes the power in fp32, so
   b = 0 gives the subnormal 2^-127; the Metal kernels build the float from the
   bits (as_type<float>(b << 23), QwenNative/kernels.metal:727), so b = 0 gives
   0.  b = 255 is +inf in both. */
WMO_EXPORT float wmo_e8m0(uint32_t b, int convention) {
  b &= 255u;
  if (b == 0 && convention == WMO_CONV_METAL) return 0.0f;
  if (b == 255) return INFINITY;
  return ldexpf(1.0f, (int)b - 127);
}

/* FP8 E4M3 (OCP "FN": no infinities, 0x7F/0xFF NaN), as mx.from_fp8 and
   MXFP4.swift:96-107 decode it. */
WMO_EXPORT float wmo_e4m3(uint32_t b) {
  b &= 255u;
  float sign = (b & 0x80u) ? -1.0f : 1.0f;
  int e = (int)((b >> 3) & 15u);
  int m = (int)(b & 7u);
  if (e == 0) return sign * (float)m * ldexpf(1.0f, -9);
  if (e == 15 && m == 7) return NAN;
  return sign * (1.0f + (float)m / 8.0f) * ldexpf(1.0f, e - 7);
}

/* ------------------------------------------------------------------ dequantisers */

/* Packed E2M1 [rows, cols/2] (low nibble = even column) + E8M0 [rows, cols/32]
   -> bf16 [rows, cols].  dequant.py:53-68 (w * s in fp32, then astype bf16). */
WMO_EXPORT int wmo_dequant_mxfp4(const uint8_t* w, const uint8_t* s, int64_t rows, int64_t cols,
                                 int convention, uint16_t* out) {
  if (cols % 32) return 1;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t c = 0; c < cols; ++c) {
      uint8_t byte = w[r * (cols / 2) + c / 2];
      uint32_t code = (c & 1) ? (byte >> 4) : (byte & 15u);
      float scale = wmo_e8m0(s[r * (cols / 32) + c / 32], convention);
      float v = wmo_e2m1(code, convention) * scale;
      out[r * cols + c] = f32_bf16(v);
    }
  }
  return 0;
}

/* FP8 E4M3 [rows, cols] + fp32 block scales [ceil(rows/128), ceil(cols/128)]
   -> bf16.  mimo/weights.py:17-43 with source_shards = 1: reserved NaN codes
   and negative or non-finite scales are rejected (status 2), and each value is
   bf16(fp32(e4m3 * scale)). */
WMO_EXPORT int wmo_dequant_fp8_b128(const uint8_t* w, const float* s, int64_t rows, int64_t cols, uint16_t* out) {
  int64_t scols = (cols + 127) / 128, srows = (rows + 127) / 128;
  for (int64_t i = 0; i < rows * cols; ++i)
    if ((w[i] & 127u) == 127u) return 2;
  for (int64_t i = 0; i < srows * scols; ++i)
    if (!isfinite(s[i]) || s[i] < 0.0f) return 2;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) {
      volatile float prod = wmo_e4m3(w[r * cols + c]) * s[(r / 128) * scols + c / 128];
      out[r * cols + c] = f32_bf16(prod);
    }
  return 0;
}

/* FP8 E4M3 [rows, cols] + UE8M0 [ceil(rows/32), ceil(cols/32)] -> bf16.
   dequant.py:45-50. */
WMO_EXPORT int wmo_dequant_fp8_b32(const uint8_t* w, const uint8_t* s, int64_t rows, int64_t cols, uint16_t* out) {
  int64_t scols = (cols + 31) / 32;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) {
      volatile float prod = wmo_e4m3(w[r * cols + c]) * wmo_e8m0(s[(r / 32) * scols + c / 32], WMO_CONV_MLX);
      out[r * cols + c] = f32_bf16(prod);
    }
  return 0;
}

/* ------------------------------------------------------------------ MXFP4 quantiser (MXFP4.swift) */

/* fp4Code, MXFP4.swift:109-130: nearest E2M1 magnitude of min(|v|, 6); on a
   tie the candidate with the even code wins; the sign comes from the sign bit
   (so -0 gives code 8). */
static uint8_t fp4_code(float value) {
  static const float cand[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  int negative = signbit(value) != 0;
  float mag = fabsf(value);
  if (mag > 6.0f) mag = 6.0f;
  int sel = 0;
  float dist = INFINITY;
  for (int i = 0; i < 8; ++i) {
    float d = fabsf(mag - cand[i]);
    if (d < dist || (d == dist && (i % 2) == 0)) {
      sel = i;
      dist = d;
    }
  }
  return (uint8_t)(sel | (negative ? 8 : 0));
}

/* Swift Float.exponent for a finite nonzero value: floor(log2|v|). */
static int float_exponent(float v) {
  int e;
  frexpf(v, &e);
  return e - 1;
}

static void quantize_group(const float* values, uint8_t* wout, uint8_t* sout) {
  float maximum = 0.0f;
  for (int i = 0; i < 32; ++i) {
    float a = fabsf(values[i]);
    if (a > maximum) maximum = a;
  }
  if (maximum == 0.0f) return; /* bytes stay 0 */
  int exponent = float_exponent(maximum) - 2;
  if (exponent < -127) exponent = -127;
  if (exponent > 128) exponent = 128;
  *sout = (uint8_t)(exponent + 127);
  float factor = ldexpf(1.0f, -exponent);
  for (int p = 0; p < 16; ++p) {
    uint8_t lo = fp4_code(values[2 * p] * factor);
    uint8_t hi = fp4_code(values[2 * p + 1] * factor);
    wout[p] = (uint8_t)(lo | (hi << 4));
  }
}

/* quantizeBF16, MXFP4.swift:4-40: bf16 [rows, cols] -> packed weights and scales. */
WMO_EXPORT int wmo_quantize_bf16_mxfp4(const uint16_t* src, int64_t rows, int64_t cols, uint8_t* w, uint8_t* s) {
  if (rows <= 0 || cols <= 0 || cols % 32) return 1;
  memset(w, 0, (size_t)(rows * cols / 2));
  memset(s, 0, (size_t)(rows * cols / 32));
  int64_t groups = cols / 32;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    float values[32];
    for (int64_t g = 0; g < groups; ++g) {
      for (int i = 0; i < 32; ++i) values[i] = bf16_f32(src[r * cols + g * 32 + i]);
      quantize_group(values, w + r * cols / 2 + g * 16, s + r * groups + g);
    }
  }
  return 0;
}

/* roundedBFloat16, MXFP4.swift:103-107 (no NaN special case). */
static float rounded_bf16_swift(float v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  u = (u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* quantizeFP8, MXFP4.swift:42-88: FP8 E4M3 [rows, cols] with bf16 inverse
   scales per 128x128 block -> packed weights and scales. */
WMO_EXPORT int wmo_quantize_fp8_mxfp4(const uint8_t* src, const uint16_t* inv_scales, int64_t rows, int64_t cols,
                                      uint8_t* w, uint8_t* s) {
  if (rows <= 0 || cols <= 0 || rows % 128 || cols % 128) return 1;
  memset(w, 0, (size_t)(rows * cols / 2));
  memset(s, 0, (size_t)(rows * cols / 32));
  int64_t groups = cols / 32, scols = cols / 128;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    float values[32];
    for (int64_t g = 0; g < groups; ++g) {
      float src_scale = bf16_f32(inv_scales[(r / 128) * scols + g / 4]);
      for (int i = 0; i < 32; ++i) {
        volatile float prod = wmo_e4m3(src[r * cols + g * 32 + i]) * src_scale;
        values[i] = rounded_bf16_swift(prod);
      }
      quantize_group(values, w + r * cols / 2 + g * 16, s + r * groups + g);
    }
  }
  return 0;
}

/* ------------------------------------------------------------------ expert arithmetic */

typedef struct {
  int32_t layout;
  /* one expert: the fused gate/up projection [2I, H] and the down projection [H, I] */
  const uint8_t* w13;
  const void* w13_scale; /* uint8 E8M0 [2I, H/32] or fp32 [2I/128, H/128] */
  const uint8_t* w2;
  const void* w2_scale; /* uint8 E8M0 [H, I/32] or fp32 [H/128, I/128] */
} wmo_expert;

/* One weight of row o, column k of a projection with `cols` inputs, exactly as
   dequantised (bf16-exact: every MXFP4 product with a power-of-two scale is
   representable; FP8 values are bf16-rounded as decode_fp8_blocks does). */
static inline float weight_at(int32_t layout, const uint8_t* w, const void* scale, int64_t o, int64_t k, int64_t cols,
                              int convention) {
  if (layout == WMO_LAYOUT_W13_FP8_B128) {
    const float* s = (const float*)scale;
    volatile float prod = wmo_e4m3(w[o * cols + k]) * s[(o / 128) * ((cols + 127) / 128) + k / 128];
    return bf16_f32(f32_bf16(prod));
  }
  if (layout == WMO_LAYOUT_W13_FP8_B32) { /* dequant.py:45-50, as wmo_dequant_fp8_b32 */
    const uint8_t* s = (const uint8_t*)scale;
    volatile float prod = wmo_e4m3(w[o * cols + k]) * wmo_e8m0(s[(o / 32) * ((cols + 31) / 32) + k / 32], WMO_CONV_MLX);
    return bf16_f32(f32_bf16(prod));
  }
  uint8_t byte = w[o * (cols / 2) + k / 2];
  uint32_t code = (k & 1) ? (byte >> 4) : (byte & 15u);
  return wmo_e2m1(code, convention) * wmo_e8m0(((const uint8_t*)scale)[o * (cols / 32) + k / 32], convention);
}

/* Decode a whole projection once into fp32 (bf16-exact values). */
static float* decode_projection(int32_t layout, const uint8_t* w, const void* scale, int64_t rows, int64_t cols,
                                int convention) {
  float* out = (float*)malloc((size_t)(rows * cols) * sizeof(float));
  if (!out) return NULL;
  for (int64_t o = 0; o < rows; ++o)
    for (int64_t k = 0; k < cols; ++k) out[o * cols + k] = weight_at(layout, w, scale, o, k, cols, convention);
  return out;
}

static inline double silu(double v) { return v / (1.0 + exp(-v)); }

/* SwiGLU of one gate/up pair.  Unclamped: silu(g)*u (qwen4_exp.py:817);
   clamped (limit > 0): silu(min(g, L)) * clamp(u, -L, L) (moe.py:38-43). */
static inline double swiglu(double g, double u, float limit) {
  if (limit > 0.0f) {
    if (g > limit) g = limit;
    if (u > limit) u = limit;
    if (u < -limit) u = -limit;
  }
  return silu(g) * u;
}

/* y[r, :] = down(swiglu(gate_up(x[r, :]))) for `rows` bf16 input rows, on
   pre-decoded weights.  Rows of the fused projection: gate first for the Qwen
   layout (Qwen.swift:441 / kernels.metal:175-181), up first for w13 = [w3; w1]
   (model.py:452-461). */
static void expert_rows(int32_t layout, const float* w13, const float* w2, int64_t H, int64_t I, const uint16_t* x,
                        int64_t rows, float limit, int numerics, float* out) {
  int gate_first = layout == WMO_LAYOUT_QWEN_GATE_UP_MXFP4;
  double* act = (double*)malloc((size_t)I * sizeof(double));
  float* xf = (float*)malloc((size_t)H * sizeof(float));
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t k = 0; k < H; ++k) xf[k] = bf16_f32(x[r * H + k]);
    for (int64_t i = 0; i < I; ++i) {
      const float* wg = w13 + (gate_first ? i : I + i) * H;
      const float* wu = w13 + (gate_first ? I + i : i) * H;
      double g = 0.0, u = 0.0;
      for (int64_t k = 0; k < H; ++k) {
        g += (double)xf[k] * wg[k];
        u += (double)xf[k] * wu[k];
      }
      /* MLX returns the gate/up product as a bf16 array (gather_qmm of bf16
         input); the native engines keep it in fp32. */
      double gr = numerics == WMO_NUMERICS_BF16 ? round_bf16(g) : (double)(float)g;
      double ur = numerics == WMO_NUMERICS_BF16 ? round_bf16(u) : (double)(float)u;
      double a = swiglu(gr, ur, limit);
      act[i] = numerics == WMO_NUMERICS_BF16 ? round_bf16(a) : (double)(float)a;
    }
    for (int64_t h = 0; h < H; ++h) {
      const float* wd = w2 + h * I;
      double y = 0.0;
      for (int64_t i = 0; i < I; ++i) y += act[i] * wd[i];
      out[r * H + h] = numerics == WMO_NUMERICS_BF16 ? round_bf16(y) : (float)y;
    }
  }
  free(act);
  free(xf);
}

/* Expert FFN of one expert over `rows` rows (the quantized_matmul pair of
   qwen4_exp.py:815-818 / model.py:516-523). */
WMO_EXPORT int wmo_expert_ffn(const wmo_expert* ex, int64_t H, int64_t I, const uint16_t* x, int64_t rows,
                              float swiglu_limit, int numerics, int convention, float* out) {
  float* w13 = decode_projection(ex->layout, ex->w13, ex->w13_scale, 2 * I, H, convention);
  float* w2 = decode_projection(ex->layout, ex->w2, ex->w2_scale, H, I, convention);
  if (!w13 || !w2) {
    free(w13);
    free(w2);
    return 1;
  }
  expert_rows(ex->layout, w13, w2, H, I, x, rows, swiglu_limit, numerics, out);
  free(w13);
  free(w2);
  return 0;
}

/* One MXFP4 / FP8 projection: y[r, o] = sum_k x[r, k] * w[o, k] (fp32 result of
   a double accumulation).  mx.quantized_matmul(transpose=True), model.py:504-513. */
WMO_EXPORT int wmo_linear(int32_t layout, const uint8_t* w, const void* scale, int64_t O, int64_t Kd, const uint16_t* x,
                          int64_t rows, int convention, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t o = 0; o < O; ++o) {
    for (int64_t r = 0; r < rows; ++r) {
      double acc = 0.0;
      for (int64_t k = 0; k < Kd; ++k)
        acc += (double)bf16_f32(x[r * Kd + k]) * weight_at(layout, w, scale, o, k, Kd, convention);
      out[r * O + o] = (float)acc;
    }
  }
  return 0;
}

/* ------------------------------------------------------------------ routers */

/* logits[t, e] = sum_h x[t, h] * W[e, h] with bf16 operands, accumulated in
   double and rounded to fp32 (the fp32-accumulated router of mimo/model.py:139-141
   and qwen4_exp.py:1011). */
WMO_EXPORT void wmo_router_logits(const uint16_t* x, const uint16_t* W, int64_t T, int64_t H, int64_t E, float* logits) {
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < T; ++t)
    for (int64_t e = 0; e < E; ++e) {
      double acc = 0.0;
      for (int64_t h = 0; h < H; ++h) acc += (double)bf16_f32(x[t * H + h]) * bf16_f32(W[e * H + h]);
      logits[t * E + e] = (float)acc;
    }
}

/* Top-k of `key` (descending; equal keys -> lower index first, as
   DeepSeekNative/engine.mm:1880 breaks ties). */
static void topk_desc(const double* key, int64_t E, int64_t K, const unsigned char* allowed, int32_t* out) {
  for (int64_t k = 0; k < K; ++k) {
    int64_t best = -1;
    for (int64_t e = 0; e < E; ++e) {
      if (allowed && !allowed[e]) continue;
      int taken = 0;
      for (int64_t j = 0; j < k; ++j)
        if (out[j] == e) taken = 1;
      if (taken) continue;
      if (best < 0 || key[e] > key[best]) best = e;
    }
    out[k] = (int32_t)best;
  }
}

/* Routes of one token from its fp32 logits.
   SOFTMAX (Qwen): top-k of the logits, weights exp(l - max) renormalised over
     the kept experts (QwenNative/engine.mm:2085-2101; equal to softmax followed
     by scores / scores.sum, qwen4_exp.py:1009-1013, 1036-1043).
   SQRTSOFTPLUS (DeepSeek V4.1): s = sqrt(softplus(l)); top-k of s + bias;
     weights s / (sum + 1e-20) * route_scale (moe.py:58-74, engine.mm:1863-1890).
   SIGMOID (MiMo): s = sigmoid(l); top-k of s + bias; s / (sum + 1e-20)
     (mimo/model.py:139-150), times route_scale.
   SIGMOID_GROUPED: as SIGMOID, but only the top `topk_groups` of `n_groups`
     contiguous expert groups are eligible, a group scored by the sum of its
     two largest biased scores.  Not in the reference (mimo/model.py:65 pins
     n_group = 1); restated from the DeepSeek-V3 "noaux_tc" selection. */
static void route_token(int router, const float* logits, const float* bias, int64_t E, int64_t K, int64_t n_groups,
                        int64_t topk_groups, float route_scale, int32_t* idx, float* w) {
  double* score = (double*)malloc((size_t)E * sizeof(double));
  double* key = (double*)malloc((size_t)E * sizeof(double));
  unsigned char* allowed = NULL;
  if (router == WMO_ROUTER_SOFTMAX) {
    /* an optional additive logit bias (used by the synthetic Zipf workload) */
    for (int64_t e = 0; e < E; ++e) key[e] = bias ? (double)(float)(logits[e] + bias[e]) : (double)logits[e];
    topk_desc(key, E, K, NULL, idx);
    double top = key[idx[0]], kept = 0.0;
    for (int64_t k = 0; k < K; ++k) kept += exp(key[idx[k]] - top);
    for (int64_t k = 0; k < K; ++k) w[k] = (float)(exp(key[idx[k]] - top) / kept * route_scale);
  } else {
    for (int64_t e = 0; e < E; ++e) {
      double v = logits[e];
      if (router == WMO_ROUTER_SQRTSOFTPLUS)
        score[e] = sqrt((v > 0 ? v : 0.0) + log1p(exp(-fabs(v))));
      else
        score[e] = 1.0 / (1.0 + exp(-v));
      score[e] = (float)score[e]; /* the reference holds scores in fp32 */
      key[e] = score[e] + (bias ? bias[e] : 0.0f);
      key[e] = (float)key[e];
    }
    if (router == WMO_ROUTER_SIGMOID_GROUPED && n_groups > 1) {
      int64_t per = E / n_groups;
      double* gscore = (double*)malloc((size_t)n_groups * sizeof(double));
      for (int64_t g = 0; g < n_groups; ++g) {
        double a = -INFINITY, b = -INFINITY;
        for (int64_t e = g * per; e < (g + 1) * per; ++e) {
          if (key[e] > a) {
            b = a;
            a = key[e];
          } else if (key[e] > b) {
            b = key[e];
          }
        }
        gscore[g] = (float)(a + b);
      }
      int32_t* gsel = (int32_t*)malloc((size_t)topk_groups * sizeof(int32_t));
      topk_desc(gscore, n_groups, topk_groups, NULL, gsel);
      allowed = (unsigned char*)calloc((size_t)E, 1);
      for (int64_t j = 0; j < topk_groups; ++j)
        for (int64_t e = gsel[j] * per; e < (gsel[j] + 1) * per; ++e) allowed[e] = 1;
      free(gscore);
      free(gsel);
    }
    topk_desc(key, E, K, allowed, idx);
    double sum = 0.0;
    for (int64_t k = 0; k < K; ++k) sum += score[idx[k]];
    for (int64_t k = 0; k < K; ++k) {
      double v = score[idx[k]];
      if (K > 1) v = v / (sum + 1e-20);
      w[k] = (float)(v * route_scale);
    }
  }
  free(score);
  free(key);
  free(allowed);
}

WMO_EXPORT void wmo_route(int router, const float* logits, const float* bias, int64_t T, int64_t E, int64_t K,
                          int64_t n_groups, int64_t topk_groups, float route_scale, int32_t* idx, float* w) {
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < T; ++t)
    route_token(router, logits + t * E, bias, E, K, n_groups, topk_groups, route_scale, idx + t * K, w + t * K);
}

/* ------------------------------------------------------------------ the layer */

typedef struct {
  int64_t T, H, I, E, K;
  int32_t layout;
  /* routed experts: expert e's fused projection at w13 + e * w13_stride, etc. */
  const uint8_t* w13;
  int64_t w13_stride;
  const uint8_t* w13_scale;
  int64_t w13_scale_stride;
  const uint8_t* w2;
  int64_t w2_stride;
  const uint8_t* w2_scale;
  int64_t w2_scale_stride;
  /* shared expert (one blob, same layout); NULL weights = none */
  const uint8_t* sh_w13;
  const void* sh_w13_scale;
  const uint8_t* sh_w2;
  const void* sh_w2_scale;
  int32_t shared_gate_kind;
  const uint16_t* shared_gate_weight; /* bf16 [H] */
  float swiglu_limit;
  int32_t numerics;
  int32_t convention;
} wmo_layer;

/* out[t] = sum_k w[t, k] * expert_{idx[t, k]}(x[t]) + shared_gate(t) * shared(x[t]),
   fp32 sum in k order, then bf16 (qwen4_exp.py:1049-1051, moe.py:110-112,
   QwenNative/kernels.metal:185-194).  `only_tokens` (may be NULL) restricts the
   work to a subset of tokens (their rows of `out` are written, others left). */
WMO_EXPORT int wmo_moe_forward(const wmo_layer* L, const uint16_t* x, const int32_t* idx, const float* w,
                               const int32_t* only_tokens, int64_t n_only, uint16_t* out) {
  int64_t T = L->T, H = L->H, I = L->I, E = L->E, K = L->K;
  int64_t n = only_tokens ? n_only : T;
  /* group the pairs by expert so each expert is decoded once */
  int64_t* cnt = (int64_t*)calloc((size_t)(E + 1), sizeof(int64_t));
  for (int64_t j = 0; j < n; ++j) {
    int64_t t = only_tokens ? only_tokens[j] : j;
    for (int64_t k = 0; k < K; ++k) {
      int32_t e = idx[t * K + k];
      if (e < 0 || e >= E) {
        free(cnt);
        return 2;
      }
      cnt[e]++;
    }
  }
  float* routed = (float*)calloc((size_t)(n * K * H), sizeof(float));
  int status = 0;
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t e = 0; e < E; ++e) {
    if (cnt[e] == 0) continue;
    int64_t rows = 0;
    int64_t* pairs = (int64_t*)malloc((size_t)cnt[e] * sizeof(int64_t));
    uint16_t* xr = (uint16_t*)malloc((size_t)(cnt[e] * H) * sizeof(uint16_t));
    for (int64_t j = 0; j < n; ++j) {
      int64_t t = only_tokens ? only_tokens[j] : j;
      for (int64_t k = 0; k < K; ++k)
        if (idx[t * K + k] == e) {
          pairs[rows] = j * K + k;
          memcpy(xr + rows * H, x + t * H, (size_t)H * 2);
          rows++;
        }
    }
    const void* s13 = L->w13_scale + e * L->w13_scale_stride;
    const void* s2 = L->w2_scale + e * L->w2_scale_stride;
    float* w13 = decode_projection(L->layout, L->w13 + e * L->w13_stride, s13, 2 * I, H, L->convention);
    float* w2 = decode_projection(L->layout, L->w2 + e * L->w2_stride, s2, H, I, L->convention);
    float* y = (float*)malloc((size_t)(rows * H) * sizeof(float));
    if (!w13 || !w2 || !y) {
      status = 1;
    } else {
      expert_rows(L->layout, w13, w2, H, I, xr, rows, L->swiglu_limit, L->numerics, y);
      for (int64_t r = 0; r < rows; ++r) memcpy(routed + pairs[r] * H, y + r * H, (size_t)H * sizeof(float));
    }
    free(w13);
    free(w2);
    free(y);
    free(pairs);
    free(xr);
  }
  float* shared = NULL;
  float* sg = NULL;
  if (L->sh_w13) {
    shared = (float*)calloc((size_t)(n * H), sizeof(float));
    sg = (float*)calloc((size_t)n, sizeof(float));
    float* w13 = decode_projection(L->layout, L->sh_w13, L->sh_w13_scale, 2 * I, H, L->convention);
    float* w2 = decode_projection(L->layout, L->sh_w2, L->sh_w2_scale, H, I, L->convention);
#pragma omp parallel for schedule(static)
    for (int64_t j = 0; j < n; ++j) {
      int64_t t = only_tokens ? only_tokens[j] : j;
      expert_rows(L->layout, w13, w2, H, I, x + t * H, 1, L->swiglu_limit, L->numerics, shared + j * H);
      if (L->shared_gate_kind == WMO_SHARED_SIGMOID_GATE) {
        double d = 0.0;
        for (int64_t h = 0; h < H; ++h) d += (double)bf16_f32(x[t * H + h]) * bf16_f32(L->shared_gate_weight[h]);
        sg[j] = (float)(1.0 / (1.0 + exp(-(double)(float)d)));
      } else {
        sg[j] = 1.0f;
      }
    }
    free(w13);
    free(w2);
  }
#pragma omp parallel for schedule(static)
  for (int64_t j = 0; j < n; ++j) {
    int64_t t = only_tokens ? only_tokens[j] : j;
    for (int64_t h = 0; h < H; ++h) {
      float a = 0.0f;
      for (int64_t k = 0; k < K; ++k) a += w[t * K + k] * routed[(j * K + k) * H + h];
      if (shared) a += sg[j] * shared[j * H + h];
      out[t * H + h] = f32_bf16(a);
    }
  }
  free(cnt);
  free(routed);
  free(shared);
  free(sg);
  return status;
}

/* The routed rows alone: y[t, k, :] = expert_{idx[t, k]}(x[t]) as bf16 bits
   (StreamingExperts.__call__ -> [1, T, K, H], qwen4_exp.py:853-904). */
WMO_EXPORT int wmo_expert_pairs(const wmo_layer* L, const uint16_t* x, const int32_t* idx, uint16_t* out) {
  int64_t T = L->T, H = L->H, I = L->I, E = L->E, K = L->K;
  int status = 0;
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t e = 0; e < E; ++e) {
    int64_t rows = 0;
    for (int64_t p = 0; p < T * K; ++p) rows += idx[p] == e;
    if (!rows) continue;
    int64_t* pairs = (int64_t*)malloc((size_t)rows * sizeof(int64_t));
    uint16_t* xr = (uint16_t*)malloc((size_t)(rows * H) * 2);
    int64_t r = 0;
    for (int64_t p = 0; p < T * K; ++p)
      if (idx[p] == e) {
        pairs[r] = p;
        memcpy(xr + r * H, x + (p / K) * H, (size_t)H * 2);
        r++;
      }
    float* w13 = decode_projection(L->layout, L->w13 + e * L->w13_stride, L->w13_scale + e * L->w13_scale_stride,
                                   2 * I, H, L->convention);
    float* w2 = decode_projection(L->layout, L->w2 + e * L->w2_stride, L->w2_scale + e * L->w2_scale_stride, H, I,
                                  L->convention);
    float* y = (float*)malloc((size_t)(rows * H) * sizeof(float));
    if (!w13 || !w2 || !y) {
      status = 1;
    } else {
      expert_rows(L->layout, w13, w2, H, I, xr, rows, L->swiglu_limit, L->numerics, y);
      for (int64_t i = 0; i < rows; ++i)
        for (int64_t h = 0; h < H; ++h) out[pairs[i] * H + h] = f32_bf16(y[i * H + h]);
    }
    free(w13);
    free(w2);
    free(y);
    free(pairs);
    free(xr);
  }
  return status;
}

/* Threads of later parallel regions of the calling thread (launchers such as
   torchrun set OMP_NUM_THREADS=1 for every process). */
WMO_EXPORT void wmo_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

WMO_EXPORT int wmo_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
