// C ABI of libwhallm_moe.so: handle, workspace, validation and the
// stream-ordered orchestration of the expert-FFN kernels.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>

#include "wm_kernels.h"
#include "wm_profile.h"

struct wm_ctx {
  int device = 0;
  int num_sms = 148;
  wm_options opt{};
  std::string err;
  wm_counters counters{};
  void* ws = nullptr;
  size_t ws_bytes = 0;
  wm::Plan plan{};
  uint16_t* xs = nullptr;      // sorted input rows (GEMM path)
  uint16_t* act = nullptr;     // sorted SwiGLU rows
  uint16_t* routed = nullptr;  // sorted expert output rows
  float* logits = nullptr;
  int32_t* idx = nullptr;
  float* w = nullptr;
  float* sg = nullptr;
  uint32_t* status = nullptr;  // [4]
  uint16_t* act16 = nullptr;   // [rows, I] f16 activation rows (decode path)
  float* rowscale = nullptr;   // [rows] prescale of the f16 x rows (decode path)
  float* actscale = nullptr;   // [rows] prescale of the f16 act rows (decode path)
  uint32_t* rowmax = nullptr;  // [rows] per-row |act| maxima (decode path)
  uint16_t* xn = nullptr;      // [T, H] normalised input rows (pre-MoE RMSNorm)
  uint8_t* xss = nullptr;      // block-scaled GEMM: the sorted x rows' UE8M0 scale rows (hi, lo)
  uint8_t* bs_img_x = nullptr;    // block-scaled decode / GEMM: token tile images (hi / lo E4M3 + scale atoms)
  uint8_t* bs_img_act = nullptr;  // ... and the act tile images
  uint32_t* tile_done = nullptr;  // fused decode launch: per-tile counts (max_mtiles + 1, zero between calls)
  int max_rows = 0, max_mtiles = 0, max_chunks = 0;
  PFN_cuTensorMapEncodeTiled_v12000 encode_tiled = nullptr;
  wm::Profiler prof;
};

namespace {

class DeviceGuard {
 public:
  explicit DeviceGuard(int device) {
    cudaGetDevice(&prev_);
    if (prev_ != device) cudaSetDevice(device);
  }
  ~DeviceGuard() { cudaSetDevice(prev_); }

 private:
  int prev_ = 0;
};

int fail(wm_ctx* ctx, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  ctx->err = buf;
  return WM_ERROR;
}

int check_launch(wm_ctx* ctx, const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(ctx, "%s: CUDA launch failed: %s", what, cudaGetErrorString(e));
  return WM_OK;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int fmt_of(int layout) {
  return layout == WM_LAYOUT_W13_FP8_B128 ? wm::kFmtFp8B128
         : layout == WM_LAYOUT_W13_FP8_B32 ? wm::kFmtFp8B32
                                           : wm::kFmtMxfp4;
}

bool is_fp8(int layout) { return layout == WM_LAYOUT_W13_FP8_B128 || layout == WM_LAYOUT_W13_FP8_B32; }

// The pre-MoE RMSNorm fields (x checked by the caller).
int validate_norm(wm_ctx* ctx, const wm_moe_args* a) {
  if (a->norm_weight == nullptr) return WM_OK;
  if (!aligned(a->norm_weight, 16)) return fail(ctx, "norm_weight must be a 16-byte aligned device pointer");
  if (!(a->norm_eps >= 0.0f) || !std::isfinite(a->norm_eps)) return fail(ctx, "norm_eps must be finite and >= 0");
  if (a->x_norm != nullptr) {
    if (!aligned(a->x_norm, 16)) return fail(ctx, "x_norm must be 16-byte aligned");
    const uintptr_t x0 = uintptr_t(a->x), n0 = uintptr_t(a->x_norm), bytes = uintptr_t(a->T) * a->H * 2;
    if (n0 < x0 + bytes && x0 < n0 + bytes) return fail(ctx, "x_norm must not overlap x");
  }
  return WM_OK;
}

// Where a call with a norm weight keeps its normalised rows.
uint16_t* norm_rows(wm_ctx* ctx, const wm_moe_args* a) {
  return static_cast<uint16_t*>(a->x_norm != nullptr ? a->x_norm : ctx->xn);
}

// Normalises x into norm_rows (a call whose router does not fuse the norm).
void run_rmsnorm(wm_ctx* ctx, const wm_moe_args* a, cudaStream_t s) {
  wm::prof_begin(&ctx->prof, wm::kProfNorm, s);
  wm::launch_rmsnorm(static_cast<const uint16_t*>(a->x), static_cast<const uint16_t*>(a->norm_weight), a->T, a->H,
                     a->norm_eps, norm_rows(ctx, a), s);
  wm::prof_end(&ctx->prof, wm::kProfNorm, s);
  ctx->counters.launches += 1;
}

// Validates the shape / pointer contract shared by every expert call.
int validate_experts(wm_ctx* ctx, const wm_moe_args* a, bool need_router) {
  const wm_options& o = ctx->opt;
  if (a == nullptr) return fail(ctx, "args is NULL");
  if (a->T < 0) return fail(ctx, "T must be >= 0 (got %d)", a->T);
  if (a->T > o.max_tokens) return fail(ctx, "T = %d exceeds the handle's max_tokens %lld", a->T, (long long)o.max_tokens);
  if (a->H <= 0 || a->H > o.max_hidden) return fail(ctx, "H = %d outside (0, max_hidden %d]", a->H, o.max_hidden);
  if (a->I <= 0 || a->I > o.max_inter) return fail(ctx, "I = %d outside (0, max_inter %d]", a->I, o.max_inter);
  if (a->E <= 0 || a->E > o.max_experts) return fail(ctx, "E = %d outside (0, max_experts %d]", a->E, o.max_experts);
  if (a->K <= 0 || a->K > o.max_topk || a->K > a->E)
    return fail(ctx, "K = %d outside (0, min(E, max_topk %d)]", a->K, o.max_topk);
  if (a->H % 64 || a->I % 64) return fail(ctx, "H (%d) and I (%d) must be multiples of 64", a->H, a->I);
  if (a->layout < WM_LAYOUT_QWEN_GATE_UP_MXFP4 || a->layout > WM_LAYOUT_W13_FP8_B32)
    return fail(ctx, "unknown expert layout %d", a->layout);
  if (a->T == 0) return WM_OK;  // nothing is read or written
  if (a->x == nullptr || !aligned(a->x, 16)) return fail(ctx, "x must be a 16-byte aligned device pointer");
  if (int rc = validate_norm(ctx, a)) return rc;
  const wm_matrix* ms[2] = {&a->w13, &a->w2};
  for (const wm_matrix* m : ms) {
    if (m->weight == nullptr || m->scale == nullptr) return fail(ctx, "expert weights and scales must be given");
    if (!aligned(m->weight, 16) || m->weight_stride % 16)
      return fail(ctx, "expert weight regions must start on 16-byte boundaries (pointer and per-expert stride)");
    if (a->layout == WM_LAYOUT_W13_FP8_B128 && (!aligned(m->scale, 4) || m->scale_stride % 4))
      return fail(ctx, "FP8 block scales must be 4-byte aligned");
    if (a->layout == WM_LAYOUT_W13_FP8_B32 && (!aligned(m->scale, 2) || m->scale_stride % 2))
      return fail(ctx, "UE8M0 block scales must be 2-byte aligned");
  }
  if (a->shared_gate != WM_SHARED_NONE) {
    if (a->shared_gate != WM_SHARED_SIGMOID_GATE && a->shared_gate != WM_SHARED_ONE)
      return fail(ctx, "unknown shared_gate %d", a->shared_gate);
    if (a->shared_w13.weight == nullptr || a->shared_w2.weight == nullptr || a->shared_w13.scale == nullptr ||
        a->shared_w2.scale == nullptr)
      return fail(ctx, "shared expert weights and scales must be given");
    if (!aligned(a->shared_w13.weight, 16) || !aligned(a->shared_w2.weight, 16))
      return fail(ctx, "shared expert weights must be 16-byte aligned");
    const size_t sal = a->layout == WM_LAYOUT_W13_FP8_B128 ? 4 : a->layout == WM_LAYOUT_W13_FP8_B32 ? 2 : 1;
    if (!aligned(a->shared_w13.scale, sal) || !aligned(a->shared_w2.scale, sal))
      return fail(ctx, "shared expert block scales must be %zu-byte aligned", sal);
    if (a->shared_gate == WM_SHARED_SIGMOID_GATE && (a->shared_gate_weight == nullptr || !aligned(a->shared_gate_weight, 16)))
      return fail(ctx, "the sigmoid shared gate needs a 16-byte aligned bf16 [H] weight");
  }
  if (need_router) {
    if (a->router_weight != nullptr) {
      if (!aligned(a->router_weight, 16)) return fail(ctx, "router_weight must be 16-byte aligned");
      if (a->router < WM_ROUTER_SOFTMAX || a->router > WM_ROUTER_SIGMOID_GROUPED)
        return fail(ctx, "unknown router kind %d", a->router);
      if (a->E > 1024) return fail(ctx, "the router supports at most 1024 experts");
      if (a->router == WM_ROUTER_SIGMOID_GROUPED) {
        if (a->n_groups < 1 || a->n_groups > 32 || a->E % a->n_groups)
          return fail(ctx, "n_groups must divide E and be in [1, 32]");
        if (a->topk_groups < 1 || a->topk_groups > a->n_groups) return fail(ctx, "topk_groups outside [1, n_groups]");
        if (a->K > a->topk_groups * (a->E / a->n_groups))
          return fail(ctx, "K exceeds the experts of the kept groups");
      }
    } else if (a->routes_idx == nullptr || a->routes_w == nullptr) {
      return fail(ctx, "give router_weight or routes_idx and routes_w");
    }
  }
  if (a->layout == WM_LAYOUT_W13_FP8_B128 && (a->H % 128 || a->I % 128))
    return fail(ctx, "FP8 128x128 experts need H and I multiples of 128");
  return WM_OK;
}

wm::ExpertWeights weights_of(const wm_moe_args* a, bool with_shared) {
  wm::ExpertWeights w{};
  w.w13 = static_cast<const uint8_t*>(a->w13.weight);
  w.w13_stride = a->w13.weight_stride;
  w.s13 = static_cast<const uint8_t*>(a->w13.scale);
  w.s13_stride = a->w13.scale_stride;
  w.w2 = static_cast<const uint8_t*>(a->w2.weight);
  w.w2_stride = a->w2.weight_stride;
  w.s2 = static_cast<const uint8_t*>(a->w2.scale);
  w.s2_stride = a->w2.scale_stride;
  if (with_shared) {
    w.sh_w13 = static_cast<const uint8_t*>(a->shared_w13.weight);
    w.sh_s13 = static_cast<const uint8_t*>(a->shared_w13.scale);
    w.sh_w2 = static_cast<const uint8_t*>(a->shared_w2.weight);
    w.sh_s2 = static_cast<const uint8_t*>(a->shared_w2.scale);
  }
  w.E = a->E;
  return w;
}

// Router logits + top-k into idx / w (and sg for the sigmoid shared gate).
bool encode_2d_bf16(wm_ctx* ctx, CUtensorMap* map, const void* base, int cols, int rows, int box_rows);

// With a norm weight the router sees the normalised rows, which it leaves in
// norm_rows: short calls normalise inside the logits kernel, long calls (and
// shapes that kernel does not take) run the RMSNorm kernel first.
// With select false only the logits (and the shared gate) are computed: the
// caller runs the selection itself (the small-call kernel).
int run_router(wm_ctx* ctx, const wm_moe_args* a, float* logits, int32_t* idx, float* w, cudaStream_t s,
               bool select = true) {
  const wm::TopkArgs tk{a->router_bias, a->K, a->router, a->n_groups, a->topk_groups, a->route_scale, idx, w};
  const uint16_t* sg_w =
      a->shared_gate == WM_SHARED_SIGMOID_GATE ? static_cast<const uint16_t*>(a->shared_gate_weight) : nullptr;
  const bool norm = a->norm_weight != nullptr;
  const uint16_t* x = static_cast<const uint16_t*>(a->x);
  CUtensorMap mx, mw;
  const bool gemm = wm::router_gemm_shape_ok(a->T, a->H, a->E) && aligned(a->router_weight, 16) &&
                    encode_2d_bf16(ctx, &mw, a->router_weight, a->H, a->E, 128);
  if (norm && (gemm || !wm::router_logits_fused_ok(a->T, a->H, a->E))) {
    run_rmsnorm(ctx, a, s);
    x = norm_rows(ctx, a);
  }
  wm::prof_begin(&ctx->prof, wm::kProfRouter, s);
  if (gemm && encode_2d_bf16(ctx, &mx, x, a->H, a->T, 128)) {
    // long calls: the logits GEMM on the tensor cores, the shared gate (one row) on the CUDA cores
    wm::launch_router_gemm(&mx, &mw, a->T, a->H, a->E, logits, ctx->status, ctx->num_sms, s);
    if (sg_w != nullptr) {
      wm::launch_shared_gate(x, sg_w, a->T, a->H, ctx->sg, s);
      ctx->counters.launches += 1;
    }
  } else {
    const bool fused = norm && x == a->x;
    wm::launch_router_logits(x, static_cast<const uint16_t*>(a->router_weight), sg_w, a->T, a->H, a->E, logits,
                             ctx->sg, s, fused ? static_cast<const uint16_t*>(a->norm_weight) : nullptr,
                             a->norm_eps, fused ? norm_rows(ctx, a) : nullptr);
  }
  wm::prof_end(&ctx->prof, wm::kProfRouter, s);
  ctx->counters.launches += 1;
  if (!select) return check_launch(ctx, "router");
  wm::prof_begin(&ctx->prof, wm::kProfTopk, s);
  wm::launch_router_topk(logits, a->T, a->E, tk, s);
  wm::prof_end(&ctx->prof, wm::kProfTopk, s);
  ctx->counters.launches += 1;
  return check_launch(ctx, "router");
}

// TMA descriptor of a sorted-row buffer: bf16 [max_rows, kdim], 64 x 128
// boxes with the 128-byte swizzle the MMA operand layout expects.
bool encode_rows_box(wm_ctx* ctx, CUtensorMap* map, const void* base, int kdim, CUtensorMapDataType dtype,
                     int box_rows) {
  if (ctx->encode_tiled == nullptr) return false;
  cuuint64_t dims[2] = {cuuint64_t(kdim), cuuint64_t(ctx->max_rows)};
  cuuint64_t strides[1] = {cuuint64_t(kdim) * 2};
  cuuint32_t box[2] = {64, cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = ctx->encode_tiled(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// TMA descriptor of a caller's bf16 matrix [rows, cols] (row-major), boxes
// of 64 columns x box_rows rows with the 128-byte swizzle.
bool encode_2d_bf16(wm_ctx* ctx, CUtensorMap* map, const void* base, int cols, int rows, int box_rows) {
  if (ctx->encode_tiled == nullptr) return false;
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(cols) * 2};
  cuuint32_t box[2] = {64, cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = ctx->encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                                 box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Expert rows per expert (on average) above which a call takes the grouped
// GEMM: its 128-row tiles read each expert's weights once, the decode
// kernels' 16-row tiles once per 16 rows.
constexpr int64_t kDecodeMaxRowsPerExpert = 32;

// Whether a call takes the tcgen05 grouped GEMM (else the decode kernels).
// gemv_max_tokens: -1 always, > 0 above that many tokens, 0 by rows per expert.
bool use_gemm(const wm_ctx* ctx, const wm_moe_args* a) {
  const int g = ctx->opt.gemv_max_tokens;
  bool gemm;
  if (g < 0)
    gemm = true;
  else if (g > 0)
    gemm = a->T > g;
  else
    gemm = (a->T * int64_t(a->K) + a->E - 1) / a->E > kDecodeMaxRowsPerExpert;
  return gemm && wm::gemm_shape_ok(a->H, a->I) && ctx->encode_tiled != nullptr;
}

enum Path { kPathGemv = 0, kPathGemm = 2, kPathDecodeMma = 3, kPathBsDecode = 4, kPathBsGemm = 5, kPathFp8Gemm = 6 };

// The block-scaled decode kernel's TMA operands: packed weights 32-byte
// aligned with 32-byte multiple strides (16U4_ALIGN16B), E8M0 rows 16-byte
// aligned with 16-byte multiple strides.
bool bs_operands_ok(const wm_ctx* ctx, const wm_moe_args* a, bool has_shared) {
  if (ctx->encode_tiled == nullptr || is_fp8(a->layout) || !wm::bs_shape_ok(a->H, a->I)) return false;
  const wm_matrix* ms[4] = {&a->w13, &a->w2, &a->shared_w13, &a->shared_w2};
  for (int i = 0; i < (has_shared ? 4 : 2); ++i) {
    if (!aligned(ms[i]->weight, 32) || !aligned(ms[i]->scale, 16)) return false;
    if (i < 2 && (ms[i]->weight_stride % 32 || ms[i]->scale_stride % 16)) return false;
  }
  return true;
}

// Which expert kernels a call takes: for long calls the block-scaled tcgen05
// grouped GEMM (MXFP4 experts whose shapes and regions its TMA operands take,
// unless WM_FLAG_F16_GEMM), else the kind::f16 tcgen05 grouped GEMM; for short
// calls the block-scaled tcgen05 decode kernel (MXFP4 experts whose
// shapes and regions its TMA operands take, unless WM_FLAG_MMA_DECODE), else
// the register-direct decode kernel where 16-byte loads are possible (MXFP4
// and FP8), else the CUDA-core GEMV.
// The FP8 grouped GEMM's TMA operands: E4M3 weights 16-byte aligned with
// 16-byte multiple strides (fp32 128 x 128 block scales, read directly).
bool fp8g_operands_ok(const wm_ctx* ctx, const wm_moe_args* a, bool has_shared) {
  if (ctx->encode_tiled == nullptr || a->layout != WM_LAYOUT_W13_FP8_B128 || !wm::fp8g_shape_ok(a->H, a->I))
    return false;
  const wm_matrix* ms[4] = {&a->w13, &a->w2, &a->shared_w13, &a->shared_w2};
  for (int i = 0; i < (has_shared ? 4 : 2); ++i) {
    if (!aligned(ms[i]->weight, 16) || !aligned(ms[i]->scale, 4)) return false;
    if (i < 2 && (ms[i]->weight_stride % 16 || ms[i]->scale_stride % 4)) return false;
  }
  return true;
}

Path expert_path(const wm_ctx* ctx, const wm_moe_args* a, bool has_shared) {
  if (use_gemm(ctx, a)) {
    if (ctx->opt.flags & WM_FLAG_F16_GEMM) return kPathGemm;
    if (bs_operands_ok(ctx, a, has_shared)) return kPathBsGemm;
    return fp8g_operands_ok(ctx, a, has_shared) ? kPathFp8Gemm : kPathGemm;
  }
  if (ctx->encode_tiled == nullptr) return kPathGemv;
  const wm_matrix* ms[4] = {&a->w13, &a->w2, &a->shared_w13, &a->shared_w2};
  for (int i = 0; i < (has_shared ? 4 : 2); ++i)
    if (!aligned(ms[i]->scale, 16) || (i < 2 && ms[i]->scale_stride % 16)) return kPathGemv;
  if (!is_fp8(a->layout) && !(ctx->opt.flags & WM_FLAG_MMA_DECODE) && bs_operands_ok(ctx, a, has_shared))
    return kPathBsDecode;
  for (int i = 0; i < (has_shared ? 4 : 2); ++i)
    if (!aligned(ms[i]->weight, 16) || (i < 2 && ms[i]->weight_stride % 16)) return kPathGemv;
  return wm::decode_mma_shape_ok(a->H, a->I, fmt_of(a->layout)) ? kPathDecodeMma : kPathGemv;
}

// Rows each expert's group is padded to: the GEMMs' 128-row tiles, the
// block-scaled decode kernel's 16-token tiles, else none.
int plan_align(Path path) {
  return path == kPathGemm || path == kPathBsGemm || path == kPathFp8Gemm ? wm::kTileM
                                                                           : path == kPathBsDecode ? 16 : 1;
}

// Plan fields of the expert kernels of `path`.
void plan_for_path(const wm_ctx* ctx, Path path, wm::Plan* plan) {
  if (path == kPathDecodeMma || path == kPathGemm) plan->rowmax = ctx->rowmax;
  if (path == kPathDecodeMma) plan->tile_rows = 8;
}

// The register-direct decode path: per-token prescale, gate/up (+SwiGLU), down.
// MXFP4 experts multiply f16 copies of the rows prescaled by 2^k (gather_f16,
// act_f16); FP8 experts the bf16 rows themselves (gather_rows, the bf16 act).
int run_decode_mma(wm_ctx* ctx, const wm_moe_args* a, const wm::ExpertWeights& wts, cudaStream_t s) {
  const int H = a->H, I = a->I;
  const int fmt = fmt_of(a->layout);
  const bool fp4 = fmt == wm::kFmtMxfp4;
  const CUtensorMapDataType dt = fp4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  uint16_t* xh = ctx->xs;                       // [max_rows, H] token rows
  uint16_t* acth = fp4 ? ctx->act16 : ctx->act;  // [max_rows, I] act rows
  CUtensorMap bx, bact;
  if (!encode_rows_box(ctx, &bx, xh, H, dt, 8) || !encode_rows_box(ctx, &bact, acth, I, dt, 8))
    return fail(ctx, "cuTensorMapEncodeTiled failed for the activation rows");
  wm::Plan plan = ctx->plan;
  plan_for_path(ctx, kPathDecodeMma, &plan);
  wm::DecodeArgs d{};
  d.plan = plan;
  d.wts = wts;
  d.act = ctx->act;
  d.routed = ctx->routed;
  d.H = H;
  d.I = I;
  d.gate_first = a->layout == WM_LAYOUT_QWEN_GATE_UP_MXFP4 ? 1 : 0;
  d.limit = a->swiglu_limit;
  d.status = ctx->status;
  wm::prof_begin(&ctx->prof, wm::kProfGather, s);
  if (fp4)
    wm::launch_gather_f16(static_cast<const uint16_t*>(a->x), plan, a->E, H, xh, ctx->rowscale, ctx->num_sms, s);
  else
    wm::launch_gather_rows(static_cast<const uint16_t*>(a->x), plan, a->E, H, xh, ctx->num_sms, s);
  wm::prof_end(&ctx->prof, wm::kProfGather, s);
  d.bscale = fp4 ? ctx->rowscale : nullptr;
  // 8-token tiles of the call, about: one per routed expert hit (at most
  // min(E, T * K)), more where an expert gets over 8 rows, plus the shared expert's
  const int64_t pairs = int64_t(a->T) * a->K;
  const int64_t has_sh = a->shared_gate != WM_SHARED_NONE ? 1 : 0;
  const int tiles = int(std::min<int64_t>(a->E, pairs) + (a->T > 8 ? pairs / 8 : 0) + has_sh * ((a->T + 7) / 8));
  wm::prof_begin(&ctx->prof, wm::kProfDecodeGateUp, s);
  const int ks0 = wm::decode_mma_split(0, H, I, tiles, ctx->num_sms, fmt);
  const int ks1 = wm::decode_mma_split(1, H, I, tiles, ctx->num_sms, fmt);
  d.nbuf = wm::decode_mma_buffers(0, H, I, ks0, tiles, ctx->num_sms, fmt);
  wm::launch_decode_mma(d, 0, &bx, ctx->num_sms, s, ks0, fmt);
  wm::prof_end(&ctx->prof, wm::kProfDecodeGateUp, s);
  if (fp4) {
    wm::prof_begin(&ctx->prof, wm::kProfActF16, s);
    wm::launch_act_f16(ctx->act, plan, a->E, I, acth, ctx->actscale, ctx->num_sms, s);
    wm::prof_end(&ctx->prof, wm::kProfActF16, s);
    ctx->counters.launches += 1;
  }
  d.bscale = fp4 ? ctx->actscale : nullptr;
  wm::prof_begin(&ctx->prof, wm::kProfDecodeDown, s);
  d.nbuf = wm::decode_mma_buffers(1, H, I, ks1, tiles, ctx->num_sms, fmt);
  wm::launch_decode_mma(d, 1, &bact, ctx->num_sms, s, ks1, fmt);
  wm::prof_end(&ctx->prof, wm::kProfDecodeDown, s);
  ctx->counters.launches += 3;
  ctx->counters.decode_calls += 1;
  return check_launch(ctx, "expert decode");
}

// TMA descriptor over one projection's packed E2M1 weights as the block-scaled
// MMA reads them: [experts][rows][K] 4-bit elements (16U4_ALIGN16B: every 8
// packed bytes land in 16 bytes of shared memory), boxes of 128 K x box_rows,
// 128-byte swizzle.
// halves = 2: the matrix is split into two halves of rows / 2 rows (w13's
// gate and up halves), a 4-D map whose boxes take box_rows rows of both.
bool encode_fp4_weights(wm_ctx* ctx, CUtensorMap* map, const void* base, int64_t K, int64_t rows, int64_t experts,
                        int64_t expert_stride, int box_rows, int halves) {
  if (ctx->encode_tiled == nullptr) return false;
  const int64_t hr = rows / halves;
  const int64_t estride = experts > 1 ? expert_stride : K / 2 * rows;
  cuuint64_t dims[4] = {cuuint64_t(K), cuuint64_t(hr), cuuint64_t(halves), cuuint64_t(experts)};
  cuuint64_t strides[3] = {cuuint64_t(K / 2), cuuint64_t(K / 2 * hr), cuuint64_t(estride)};
  cuuint32_t box[4] = {128, cuuint32_t(box_rows), cuuint32_t(halves), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  if (halves == 1) {  // 3-D: [experts][rows][K]
    dims[2] = cuuint64_t(experts);
    strides[1] = cuuint64_t(estride);
    box[2] = 1;
  }
  CUresult r = ctx->encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, halves == 1 ? 3 : 4,
                                 const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                 CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// E4M3 weights [experts][halves][rows / halves][K] as uint8, boxes of 128
// bytes x box_rows (x halves), 128-byte swizzle (the FP8 grouped GEMM's B).
bool encode_fp8_weights(wm_ctx* ctx, CUtensorMap* map, const void* base, int64_t K, int64_t rows, int64_t experts,
                        int64_t expert_stride, int box_rows, int halves) {
  if (ctx->encode_tiled == nullptr) return false;
  const int64_t hr = rows / halves;
  const int64_t estride = experts > 1 ? expert_stride : K * rows;
  cuuint64_t dims[4] = {cuuint64_t(K), cuuint64_t(hr), cuuint64_t(halves), cuuint64_t(experts)};
  cuuint64_t strides[3] = {cuuint64_t(K), cuuint64_t(K * hr), cuuint64_t(estride)};
  cuuint32_t box[4] = {128, cuuint32_t(box_rows), cuuint32_t(halves), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  if (halves == 1) {  // 3-D: [experts][rows][K]
    dims[2] = cuuint64_t(experts);
    strides[1] = cuuint64_t(estride);
    box[2] = 1;
  }
  return ctx->encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, halves == 1 ? 3 : 4, const_cast<void*>(base), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// E8M0 rows [experts][halves][rows / halves][S] as uint8, boxes of 16 bytes x
// box_rows (x halves), no swizzle.
bool encode_scale_rows(wm_ctx* ctx, CUtensorMap* map, const void* base, int64_t S, int64_t rows, int64_t experts,
                       int64_t expert_stride, int box_rows, int halves) {
  if (ctx->encode_tiled == nullptr) return false;
  const int64_t hr = rows / halves;
  const int64_t estride = experts > 1 ? expert_stride : S * rows;
  cuuint64_t dims[4] = {cuuint64_t(S), cuuint64_t(hr), cuuint64_t(halves), cuuint64_t(experts)};
  cuuint64_t strides[3] = {cuuint64_t(S), cuuint64_t(S * hr), cuuint64_t(estride)};
  cuuint32_t box[4] = {16, cuuint32_t(box_rows), cuuint32_t(halves), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  if (halves == 1) {
    dims[2] = cuuint64_t(experts);
    strides[1] = cuuint64_t(estride);
    box[2] = 1;
  }
  CUresult r = ctx->encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, halves == 1 ? 3 : 4, const_cast<void*>(base),
                                 dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// The block-scaled decode path: hi / lo E4M3 token tiles, gate/up (+SwiGLU,
// act tiles), down.  The plan's groups are padded to 16 rows.
int run_bs_decode(wm_ctx* ctx, const wm_moe_args* a, const wm::ExpertWeights& wts, bool has_shared, cudaStream_t s,
                  const wm::EpReturn* ret, bool images_ready) {
  const int H = a->H, I = a->I;
  CUtensorMap w13, w13s, w2, w2s, s13, s13s, s2, s2s;
  bool ok = encode_fp4_weights(ctx, &w13, a->w13.weight, H, 2 * I, a->E, a->w13.weight_stride, 64, 2) &&
            encode_fp4_weights(ctx, &w2, a->w2.weight, I, H, a->E, a->w2.weight_stride, 128, 1) &&
            encode_scale_rows(ctx, &s13, a->w13.scale, H / 32, 2 * I, a->E, a->w13.scale_stride, 64, 2) &&
            encode_scale_rows(ctx, &s2, a->w2.scale, I / 32, H, a->E, a->w2.scale_stride, 128, 1);
  if (has_shared)
    ok = ok && encode_fp4_weights(ctx, &w13s, a->shared_w13.weight, H, 2 * I, 1, 0, 64, 2) &&
         encode_fp4_weights(ctx, &w2s, a->shared_w2.weight, I, H, 1, 0, 128, 1) &&
         encode_scale_rows(ctx, &s13s, a->shared_w13.scale, H / 32, 2 * I, 1, 0, 64, 2) &&
         encode_scale_rows(ctx, &s2s, a->shared_w2.scale, I / 32, H, 1, 0, 128, 1);
  if (!ok) return fail(ctx, "cuTensorMapEncodeTiled failed for the block-scaled expert operands");
  uint8_t* ximg = ctx->bs_img_x;    // rows / 16 x H / 128 images of 4608 bytes
  uint8_t* aimg = ctx->bs_img_act;  // the same for the act rows (K = I)
  wm::BsArgs b{};
  b.plan = ctx->plan;
  b.wts = wts;
  b.H = H;
  b.I = I;
  b.gate_first = a->layout == WM_LAYOUT_QWEN_GATE_UP_MXFP4 ? 1 : 0;
  b.limit = a->swiglu_limit;
  b.status = ctx->status;
  b.act_img = aimg;
  b.routed = ctx->routed;
  if (!images_ready) {
    wm::prof_begin(&ctx->prof, wm::kProfGather, s);
    wm::launch_bs_quant_rows(static_cast<const uint16_t*>(a->x), b.plan, a->E, H, ximg, ctx->num_sms, s);
    wm::prof_end(&ctx->prof, wm::kProfGather, s);
    ctx->counters.launches += 1;
  }
  b.img = ximg;
  if ((ctx->opt.flags & WM_FLAG_FUSED_DECODE) && ret == nullptr) {
    // both expert kernels in one persistent launch (not on the expert-parallel
    // owner path, whose side-stream kernels could hold SMs the launch waits on)
    b.tile_done = ctx->tile_done;
    b.max_tiles = ctx->max_mtiles;
    const void* maps[8] = {&w13, has_shared ? &w13s : &w13, &s13, has_shared ? &s13s : &s13,
                           &w2,  has_shared ? &w2s : &w2,   &s2,  has_shared ? &s2s : &s2};
    wm::prof_begin(&ctx->prof, wm::kProfDecodeFused, s);
    wm::launch_bs_decode_fused(b, maps, ctx->num_sms, s);
    wm::prof_end(&ctx->prof, wm::kProfDecodeFused, s);
    ctx->counters.launches += 1;
    ctx->counters.decode_calls += 1;
    return check_launch(ctx, "block-scaled expert decode (one launch)");
  }
  wm::prof_begin(&ctx->prof, wm::kProfDecodeGateUp, s);
  const void* maps0[4] = {&w13, has_shared ? &w13s : &w13, &s13, has_shared ? &s13s : &s13};
  wm::launch_bs_decode(b, 0, maps0, ctx->num_sms, s);
  wm::prof_end(&ctx->prof, wm::kProfDecodeGateUp, s);
  b.img = aimg;
  if (ret != nullptr) b.ret = *ret;
  wm::prof_begin(&ctx->prof, wm::kProfDecodeDown, s);
  const void* maps1[4] = {&w2, has_shared ? &w2s : &w2, &s2, has_shared ? &s2s : &s2};
  wm::launch_bs_decode(b, 1, maps1, ctx->num_sms, s);
  wm::prof_end(&ctx->prof, wm::kProfDecodeDown, s);
  ctx->counters.launches += 2;
  ctx->counters.decode_calls += 1;
  return check_launch(ctx, "block-scaled expert decode");
}

// The x rows a call's plan may reference: rows [0, rows); with counts, rows
// are expert-parallel slots and block r = row / capacity holds counts[r].
struct XRows {
  int64_t rows;
  const int32_t* counts;
  int capacity;
};

// 2-D uint8 map [rows][cols] with boxes of box_cols x box_rows.
bool encode_bytes_2d(wm_ctx* ctx, CUtensorMap* map, const void* base, int64_t cols, int64_t rows, int box_cols,
                     int box_rows, CUtensorMapSwizzle swizzle) {
  if (ctx->encode_tiled == nullptr) return false;
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(cols)};
  cuuint32_t box[2] = {cuuint32_t(box_cols), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  return ctx->encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The block-scaled grouped GEMM path: every x row quantised once (hi / lo
// E4M3 + UE8M0 scales) and written to each sorted row that holds it, gate/up
// (+SwiGLU, act tile images), down.  The plan's groups are padded to 128
// rows.
int run_bs_gemm(wm_ctx* ctx, const wm_moe_args* a, const wm::ExpertWeights& wts, bool has_shared, cudaStream_t s,
                const wm::EpReturn* ret, const XRows& xr, bool fp8) {
  const int H = a->H, I = a->I;
  CUtensorMap w13, w13s, w2, w2s, s13, s13s, s2, s2s;
  bool ok;
  if (fp8) {  // E4M3 bytes; the fp32 block scales are read by the kernel itself
    ok = encode_fp8_weights(ctx, &w13, a->w13.weight, H, 2 * I, a->E, a->w13.weight_stride, 64, 2) &&
         encode_fp8_weights(ctx, &w2, a->w2.weight, I, H, a->E, a->w2.weight_stride, 128, 1);
    if (has_shared)
      ok = ok && encode_fp8_weights(ctx, &w13s, a->shared_w13.weight, H, 2 * I, 1, 0, 64, 2) &&
           encode_fp8_weights(ctx, &w2s, a->shared_w2.weight, I, H, 1, 0, 128, 1);
  } else {
    ok = encode_fp4_weights(ctx, &w13, a->w13.weight, H, 2 * I, a->E, a->w13.weight_stride, 64, 2) &&
         encode_fp4_weights(ctx, &w2, a->w2.weight, I, H, a->E, a->w2.weight_stride, 128, 1) &&
         encode_scale_rows(ctx, &s13, a->w13.scale, H / 32, 2 * I, a->E, a->w13.scale_stride, 64, 2) &&
         encode_scale_rows(ctx, &s2, a->w2.scale, I / 32, H, a->E, a->w2.scale_stride, 128, 1);
    if (has_shared)
      ok = ok && encode_fp4_weights(ctx, &w13s, a->shared_w13.weight, H, 2 * I, 1, 0, 64, 2) &&
           encode_fp4_weights(ctx, &w2s, a->shared_w2.weight, I, H, 1, 0, 128, 1) &&
           encode_scale_rows(ctx, &s13s, a->shared_w13.scale, H / 32, 2 * I, 1, 0, 64, 2) &&
           encode_scale_rows(ctx, &s2s, a->shared_w2.scale, I / 32, H, 1, 0, 128, 1);
  }
  if (!ok) return fail(ctx, "cuTensorMapEncodeTiled failed for the block-scaled expert operands");
  // sorted rows' parts: hi, lo [max_rows][H] in the f16 row block, scale rows [max_rows][H / 32]
  const int64_t mr = ctx->max_rows;
  uint8_t* xh = reinterpret_cast<uint8_t*>(ctx->xs);
  uint8_t* xl = xh + mr * H;
  uint8_t* xsh = ctx->xss;
  uint8_t* xsl = xsh + ((mr * (H / 32) + 255) & ~int64_t(255));
  CUtensorMap mxh, mxl, mxsh, mxsl;
  ok = encode_bytes_2d(ctx, &mxh, xh, H, mr, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B) &&
       encode_bytes_2d(ctx, &mxl, xl, H, mr, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B) &&
       encode_bytes_2d(ctx, &mxsh, xsh, H / 32, mr, 16, 128, CU_TENSOR_MAP_SWIZZLE_NONE) &&
       encode_bytes_2d(ctx, &mxsl, xsl, H / 32, mr, 16, 128, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!ok) return fail(ctx, "cuTensorMapEncodeTiled failed for the sorted-row operands");
  wm::BsArgs b{};
  b.plan = ctx->plan;
  b.wts = wts;
  b.H = H;
  b.I = I;
  b.gate_first = a->layout == WM_LAYOUT_QWEN_GATE_UP_MXFP4 ? 1 : 0;
  b.limit = a->swiglu_limit;
  b.status = ctx->status;
  b.act_img = ctx->bs_img_act;
  b.routed = ctx->routed;
  wm::prof_begin(&ctx->prof, wm::kProfGather, s);
  wm::launch_bsg_quant_scatter(static_cast<const uint16_t*>(a->x), int(xr.rows), H, b.plan, a->K, has_shared, a->E,
                               xr.counts, xr.capacity, xh, xl, xsh, xsl, ctx->num_sms, s);
  wm::prof_end(&ctx->prof, wm::kProfGather, s);
  wm::prof_begin(&ctx->prof, wm::kProfGemmGateUp, s);
  if (fp8) {
    const void* maps0[6] = {&w13, has_shared ? &w13s : &w13, &mxh, &mxl, &mxsh, &mxsl};
    wm::launch_fp8g(b, 0, maps0, ctx->num_sms, s);
  } else {
    const void* maps0[8] = {&w13, has_shared ? &w13s : &w13, &s13, has_shared ? &s13s : &s13,
                            &mxh, &mxl, &mxsh, &mxsl};
    wm::launch_bsg(b, 0, maps0, ctx->num_sms, s);
  }
  wm::prof_end(&ctx->prof, wm::kProfGemmGateUp, s);
  b.img = ctx->bs_img_act;
  if (ret != nullptr) b.ret = *ret;
  wm::prof_begin(&ctx->prof, wm::kProfGemmDown, s);
  if (fp8) {
    const void* maps1[2] = {&w2, has_shared ? &w2s : &w2};
    wm::launch_fp8g(b, 1, maps1, ctx->num_sms, s);
  } else {
    const void* maps1[4] = {&w2, has_shared ? &w2s : &w2, &s2, has_shared ? &s2s : &s2};
    wm::launch_bsg(b, 1, maps1, ctx->num_sms, s);
  }
  wm::prof_end(&ctx->prof, wm::kProfGemmDown, s);
  ctx->counters.launches += 3;
  ctx->counters.gemm_calls += 1;
  ctx->counters.bs_gemm_calls += 1;
  return check_launch(ctx, "block-scaled expert GEMM");
}

// Runs the experts of a plan already built on `s` (rows in ctx->routed, or,
// with `ret`, the down rows stored straight into the senders' back blocks:
// the grouped GEMMs and the block-scaled decode path only).
int run_experts(wm_ctx* ctx, const wm_moe_args* a, bool has_shared, Path path, cudaStream_t s,
                const wm::EpReturn* ret = nullptr, const XRows* xr = nullptr, bool images_ready = false) {
  const wm::ExpertWeights wts = weights_of(a, has_shared);
  const int gate_first = a->layout == WM_LAYOUT_QWEN_GATE_UP_MXFP4 ? 1 : 0;
  if (path == kPathDecodeMma) return run_decode_mma(ctx, a, wts, s);
  if (path == kPathBsDecode) return run_bs_decode(ctx, a, wts, has_shared, s, ret, images_ready);
  if (path == kPathBsGemm || path == kPathFp8Gemm)
    return run_bs_gemm(ctx, a, wts, has_shared, s, ret, xr ? *xr : XRows{a->T, nullptr, 0}, path == kPathFp8Gemm);
  if (path == kPathGemv) {
    wm::GemvArgs g{};
    g.plan = ctx->plan;
    g.wts = wts;
    g.x = static_cast<const uint16_t*>(a->x);
    g.act = ctx->act;
    g.routed = ctx->routed;
    g.H = a->H;
    g.I = a->I;
    g.gate_first = gate_first;
    g.limit = a->swiglu_limit;
    const int max_unique = std::min(a->E, a->T * a->K) + (has_shared ? 1 : 0);
    wm::launch_gemv(g, fmt_of(a->layout), max_unique, s, &ctx->prof);
    ctx->counters.launches += 2;
    ctx->counters.gemv_calls += 1;
    return check_launch(ctx, "expert GEMV");
  }
  // Grouped GEMM: gather the sorted rows, then gate/up (+SwiGLU) and down on
  // tcgen05.  MXFP4 runs on f16 rows scaled by 2^k per row (gather_f16, and
  // act_f16 between the two GEMMs), FP8 on bf16 rows.
  const bool f16 = fmt_of(a->layout) == wm::kFmtMxfp4;
  wm::Plan plan = ctx->plan;
  plan_for_path(ctx, kPathGemm, &plan);
  wm::prof_begin(&ctx->prof, wm::kProfGather, s);
  if (f16)
    wm::launch_gather_f16(static_cast<const uint16_t*>(a->x), plan, a->E, a->H, ctx->xs, ctx->rowscale, ctx->num_sms,
                          s);
  else
    wm::launch_gather_rows(static_cast<const uint16_t*>(a->x), plan, a->E, a->H, ctx->xs, ctx->num_sms, s);
  wm::prof_end(&ctx->prof, wm::kProfGather, s);
  CUtensorMap map_x, map_act;
  const CUtensorMapDataType dt = f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (!encode_rows_box(ctx, &map_x, ctx->xs, a->H, dt, 128) ||
      !encode_rows_box(ctx, &map_act, f16 ? ctx->act16 : ctx->act, a->I, dt, 128))
    return fail(ctx, "cuTensorMapEncodeTiled failed for the sorted-row buffers");
  wm::GemmArgs g{};
  g.plan = plan;
  g.wts = wts;
  g.I = a->I;
  g.gate_first = gate_first;
  g.limit = a->swiglu_limit;
  g.fmt = fmt_of(a->layout);
  g.status = ctx->status;
  g.out = ctx->act;
  g.Kdim = a->H;
  g.N = 2 * a->I;
  g.ascale = f16 ? ctx->rowscale : nullptr;
  g.rowmax = f16 ? ctx->rowmax : nullptr;
  {
    const wm_matrix* ms[4] = {&a->w13, &a->w2, &a->shared_w13, &a->shared_w2};
    g.w32 = 1;
    for (int i = 0; i < (has_shared ? 4 : 2); ++i)
      if (!aligned(ms[i]->weight, 32) || (i < 2 && ms[i]->weight_stride % 32)) g.w32 = 0;
  }
  wm::prof_begin(&ctx->prof, wm::kProfGemmGateUp, s);
  wm::launch_gemm(g, 0, &map_x, ctx->num_sms, s);
  wm::prof_end(&ctx->prof, wm::kProfGemmGateUp, s);
  if (f16) {
    wm::prof_begin(&ctx->prof, wm::kProfActF16, s);
    wm::launch_act_f16(ctx->act, plan, a->E, a->I, ctx->act16, ctx->actscale, ctx->num_sms, s);
    wm::prof_end(&ctx->prof, wm::kProfActF16, s);
    ctx->counters.launches += 1;
  }
  g.out = ctx->routed;
  g.Kdim = a->I;
  g.N = a->H;
  g.ascale = f16 ? ctx->actscale : nullptr;
  g.rowmax = nullptr;
  if (ret != nullptr) g.ret = *ret;
  wm::prof_begin(&ctx->prof, wm::kProfGemmDown, s);
  wm::launch_gemm(g, 1, &map_act, ctx->num_sms, s);
  wm::prof_end(&ctx->prof, wm::kProfGemmDown, s);
  ctx->counters.launches += 3;
  ctx->counters.gemm_calls += 1;
  return check_launch(ctx, "expert GEMM");
}

}  // namespace

extern "C" {

WM_EXPORT wm_ctx* wm_create(int32_t device, const wm_options* options, char* error, size_t error_size) {
  auto report = [&](const char* msg) {
    if (error && error_size) snprintf(error, error_size, "%s", msg);
  };
  if (options == nullptr) {
    report("options is NULL");
    return nullptr;
  }
  wm_options o = *options;
  if (o.flags & ~int32_t(WM_FLAG_SKIP_NEGATIVE_ROUTES | WM_FLAG_MMA_DECODE | WM_FLAG_F16_GEMM |
                        WM_FLAG_SPLIT_SMALL_CALLS | WM_FLAG_FUSED_DECODE)) {
    report("unknown flags");
    return nullptr;
  }
  if (o.max_tokens <= 0 || o.max_hidden <= 0 || o.max_inter <= 0 || o.max_experts <= 0 || o.max_topk <= 0) {
    report("every max_* option must be positive");
    return nullptr;
  }
  if (o.max_experts > 1024 || o.max_topk > 64) {
    report("max_experts must be <= 1024 and max_topk <= 64");
    return nullptr;
  }
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
    report("no such CUDA device");
    return nullptr;
  }
  DeviceGuard guard(device);
  cudaDeviceProp prop{};
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
    report("cudaGetDeviceProperties failed");
    return nullptr;
  }
  if (prop.major != 10) {
    report("libwhallm_moe needs an sm_100 (B200-class) GPU");
    return nullptr;
  }
  wm_ctx* ctx = new (std::nothrow) wm_ctx();
  if (ctx == nullptr) {
    report("out of host memory");
    return nullptr;
  }
  ctx->device = device;
  ctx->num_sms = prop.multiProcessorCount;
  ctx->opt = o;
  const int64_t T = o.max_tokens, K = o.max_topk, E = o.max_experts, H = o.max_hidden, I = o.max_inter;
  const int64_t rows = T * K + T + int64_t(wm::kTileM) * (E + 1);
  ctx->max_rows = int(rows);
  ctx->max_mtiles = int(std::max(rows / wm::kTileM + E + 2, (T * K + T) / 8 + E + 2));
  ctx->max_chunks = 1024;
  // workspace layout
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t at = off;
    off = align_up(off + bytes, 256);
    return at;
  };
  const size_t o_counts = take((E + 1) * 4), o_offsets = take((E + 2) * 4), o_pair = take(T * K * 4),
               o_rowtok = take(rows * 4), o_unique = take((E + 1) * 4), o_nunique = take(4),
               o_mtiles = take(size_t(ctx->max_mtiles) * 8), o_nm = take(4),
               o_hist = take(size_t(ctx->max_chunks) * (E + 1) * 4), o_xs = take(rows * H * 2),
               o_act = take(rows * I * 2), o_routed = take(rows * H * 2), o_logits = take(T * E * 4),
               o_idx = take(T * K * 4), o_w = take(T * K * 4), o_sg = take(T * 4), o_status = take(16),
               o_act16 = take(rows * I * 2), o_rowscale = take(rows * 4), o_actscale = take(rows * 4),
               o_rowmax = take(rows * 4), o_xn = take(T * H * 2), o_xss = take(rows * (H / 32 + 1) * 2 + 1024),
               // tile images: the decode kernel's 16-row tiles (x and act) or the GEMM's 128-row act tiles
               o_imgx = take(rows * H * 9 / 4),
               o_imga = take(std::max<size_t>(rows * I * 9 / 4, wm::bsg_image_bytes(rows / wm::kTileM + 2, int(I)))),
               o_tiledone = take((size_t(ctx->max_mtiles) + 1) * 4);
  ctx->ws_bytes = off;
  if (cudaMalloc(&ctx->ws, ctx->ws_bytes) != cudaSuccess) {
    cudaGetLastError();
    char msg[160];
    snprintf(msg, sizeof(msg), "cudaMalloc of the %.1f MB workspace failed", ctx->ws_bytes / 1e6);
    report(msg);
    delete ctx;
    return nullptr;
  }
  uint8_t* base = static_cast<uint8_t*>(ctx->ws);
  ctx->plan.counts = reinterpret_cast<int32_t*>(base + o_counts);
  ctx->plan.offsets = reinterpret_cast<int32_t*>(base + o_offsets);
  ctx->plan.pair_pos = reinterpret_cast<int32_t*>(base + o_pair);
  ctx->plan.row_token = reinterpret_cast<int32_t*>(base + o_rowtok);
  ctx->plan.unique = reinterpret_cast<int32_t*>(base + o_unique);
  ctx->plan.n_unique = reinterpret_cast<int32_t*>(base + o_nunique);
  ctx->plan.mtiles = reinterpret_cast<int32_t*>(base + o_mtiles);
  ctx->plan.n_mtiles = reinterpret_cast<int32_t*>(base + o_nm);
  ctx->plan.hist = reinterpret_cast<int32_t*>(base + o_hist);
  ctx->xs = reinterpret_cast<uint16_t*>(base + o_xs);
  ctx->act = reinterpret_cast<uint16_t*>(base + o_act);
  ctx->routed = reinterpret_cast<uint16_t*>(base + o_routed);
  ctx->logits = reinterpret_cast<float*>(base + o_logits);
  ctx->idx = reinterpret_cast<int32_t*>(base + o_idx);
  ctx->w = reinterpret_cast<float*>(base + o_w);
  ctx->sg = reinterpret_cast<float*>(base + o_sg);
  ctx->status = reinterpret_cast<uint32_t*>(base + o_status);
  ctx->act16 = reinterpret_cast<uint16_t*>(base + o_act16);
  ctx->rowscale = reinterpret_cast<float*>(base + o_rowscale);
  ctx->actscale = reinterpret_cast<float*>(base + o_actscale);
  ctx->rowmax = reinterpret_cast<uint32_t*>(base + o_rowmax);
  ctx->xn = reinterpret_cast<uint16_t*>(base + o_xn);
  ctx->xss = base + o_xss;
  ctx->bs_img_x = base + o_imgx;
  ctx->bs_img_act = base + o_imga;
  ctx->tile_done = reinterpret_cast<uint32_t*>(base + o_tiledone);
  // the whole workspace starts at zero (status word included); padding rows of
  // the f16 row blocks are never written afterwards, so they hold zeros or an
  // earlier call's finite rows
  if (cudaMemset(ctx->ws, 0, ctx->ws_bytes) != cudaSuccess) {
    cudaGetLastError();
    report("clearing the workspace failed");
    cudaFree(ctx->ws);
    delete ctx;
    return nullptr;
  }
  const size_t gemv_smem = wm::gemv_smem_bytes(int(H), int(I));
  if (gemv_smem > size_t(prop.sharedMemPerBlockOptin)) {
    report("max_hidden is too large for the decode GEMV's shared-memory staging");
    cudaFree(ctx->ws);
    delete ctx;
    return nullptr;
  }
  wm::gemv_init_attributes(int(gemv_smem));
  wm::gemm_init_attributes();
  wm::decode_mma_init_attributes(int(H), int(I));
  wm::bs_init_attributes();
  wm::bsg_init_attributes();
  wm::fp8g_init_attributes();
  wm::router_init_attributes(int(H));
  wm::router_gemm_init_attributes();
  cudaDriverEntryPointQueryResult q{};
  void* fn = nullptr;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    ctx->encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  if (cudaDeviceSynchronize() != cudaSuccess) {
    report("device initialisation failed");
    cudaFree(ctx->ws);
    delete ctx;
    return nullptr;
  }
  return ctx;
}

WM_EXPORT void wm_destroy(wm_ctx* ctx) {
  if (ctx == nullptr) return;
  {
    DeviceGuard guard(ctx->device);
    cudaFree(ctx->ws);
  }
  delete ctx;
}

WM_EXPORT const char* wm_error(const wm_ctx* ctx) { return ctx ? ctx->err.c_str() : "no handle"; }

WM_EXPORT void wm_counters_get(const wm_ctx* ctx, wm_counters* out) {
  if (ctx && out) *out = ctx->counters;
}

WM_EXPORT int wm_sync(wm_ctx* ctx, void* stream) {
  if (ctx == nullptr) return WM_ERROR;
  DeviceGuard guard(ctx->device);
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(ctx, "stream synchronisation failed: %s", cudaGetErrorString(e));
  uint32_t st[2] = {0, 0};
  e = cudaMemcpy(st, ctx->status, sizeof(st), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(ctx, "reading the device status failed: %s", cudaGetErrorString(e));
  if (st[0] == wm::kStatusOk) return WM_OK;
  cudaMemset(ctx->status, 0, 16);
  switch (st[0]) {
    case wm::kStatusBadExpert:
      return fail(ctx, "expert ID is outside the model (pair %u)", st[1]);
    case wm::kStatusOverflow:
      return fail(ctx, "sorted rows exceeded the workspace (%u)", st[1]);
    case wm::kStatusWaitTimeout:
      if (st[1] >= 60u * 16u && st[1] < 62u * 16u)
        return fail(ctx, "an expert-parallel %s wait timed out (peer %u never signalled); results are invalid",
                    st[1] < 61u * 16u ? "dispatch" : "return", st[1] % 16u);
      return fail(ctx, "a GEMM pipeline wait timed out (role %u); results are invalid", st[1]);
    case wm::kStatusNanCode:
      return fail(ctx, "FP8 weights contain reserved NaN codes (row %u)", st[1]);
    default:
      return fail(ctx, "device status %u (%u)", st[0], st[1]);
  }
}

WM_EXPORT int wm_dequant(wm_ctx* ctx, int32_t format, const void* weight, const void* scale, int64_t rows,
                         int64_t cols, int32_t convention, void* out_bf16, void* stream) {
  if (ctx == nullptr) return WM_ERROR;
  if (format < WM_FORMAT_MXFP4 || format > WM_FORMAT_FP8_B32) return fail(ctx, "unknown format %d", format);
  if (rows < 0 || cols <= 0 || cols % 32) return fail(ctx, "cols must be a positive multiple of 32");
  if (rows == 0) return WM_OK;
  if (!weight || !scale || !out_bf16) return fail(ctx, "weight, scale and out must be device pointers");
  if (!aligned(weight, 8) || !aligned(out_bf16, 16)) return fail(ctx, "weight must be 8-byte and out 16-byte aligned");
  if (format == WM_FORMAT_FP8_B128 && !aligned(scale, 4)) return fail(ctx, "fp32 block scales must be 4-byte aligned");
  DeviceGuard guard(ctx->device);
  wm::launch_dequant(format, weight, scale, rows, cols, convention, static_cast<uint16_t*>(out_bf16), ctx->status,
                     static_cast<cudaStream_t>(stream));
  ctx->counters.calls_dequant += 1;
  ctx->counters.launches += 1;
  return check_launch(ctx, "dequant");
}

WM_EXPORT int wm_route(wm_ctx* ctx, const wm_moe_args* a, float* logits, int32_t* idx, float* w, void* stream) {
  if (ctx == nullptr) return WM_ERROR;
  if (a == nullptr) return fail(ctx, "args is NULL");
  if (a->router_weight == nullptr) return fail(ctx, "wm_route needs router_weight");
  if (idx == nullptr || w == nullptr) return fail(ctx, "idx and w outputs must be given");
  wm_moe_args b = *a;
  b.shared_gate = WM_SHARED_NONE;
  // only the router part of the contract applies
  const wm_options& o = ctx->opt;
  if (b.T < 0 || b.T > o.max_tokens) return fail(ctx, "T = %d outside [0, max_tokens]", b.T);
  if (b.E <= 0 || b.E > std::min(o.max_experts, 1024)) return fail(ctx, "E = %d outside (0, max_experts]", b.E);
  if (b.K <= 0 || b.K > b.E || b.K > o.max_topk) return fail(ctx, "K = %d outside (0, min(E, max_topk)]", b.K);
  if (b.H <= 0 || b.H % 8 || b.H > o.max_hidden) return fail(ctx, "H = %d must be a multiple of 8 within max_hidden", b.H);
  if (!b.x || !aligned(b.x, 16) || !aligned(b.router_weight, 16)) return fail(ctx, "x and router_weight must be 16-byte aligned");
  if (int rc = validate_norm(ctx, &b)) return rc;
  if (b.router < WM_ROUTER_SOFTMAX || b.router > WM_ROUTER_SIGMOID_GROUPED) return fail(ctx, "unknown router kind %d", b.router);
  if (b.router == WM_ROUTER_SIGMOID_GROUPED &&
      (b.n_groups < 1 || b.n_groups > 32 || b.E % b.n_groups || b.topk_groups < 1 || b.topk_groups > b.n_groups ||
       b.K > b.topk_groups * (b.E / b.n_groups)))
    return fail(ctx, "invalid group-limited routing shape");
  if (b.T == 0) return WM_OK;
  DeviceGuard guard(ctx->device);
  ctx->counters.calls_route += 1;
  return run_router(ctx, &b, logits ? logits : ctx->logits, idx, w, static_cast<cudaStream_t>(stream));
}

WM_EXPORT int wm_expert_pairs(wm_ctx* ctx, const wm_moe_args* a, void* routed, void* stream) {
  if (ctx == nullptr) return WM_ERROR;
  wm_moe_args b = *a;
  b.shared_gate = WM_SHARED_NONE;
  b.router_weight = nullptr;
  if (int rc = validate_experts(ctx, &b, false)) return rc;
  if (b.T == 0) return WM_OK;
  if (b.routes_idx == nullptr) return fail(ctx, "wm_expert_pairs needs routes_idx");
  if (routed == nullptr || !aligned(routed, 16)) return fail(ctx, "routed must be a 16-byte aligned device pointer");
  DeviceGuard guard(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (b.norm_weight != nullptr) {  // the experts read the normalised rows
    run_rmsnorm(ctx, &b, s);
    b.x = norm_rows(ctx, &b);
    b.norm_weight = nullptr;
  }
  const Path path = expert_path(ctx, &b, false);
  wm::Plan plan = ctx->plan;
  plan_for_path(ctx, path, &plan);
  plan.skip_negative = (ctx->opt.flags & WM_FLAG_SKIP_NEGATIVE_ROUTES) ? 1 : 0;
  int launches = 0;
  wm::prof_begin(&ctx->prof, wm::kProfPlan, s);
  wm::launch_plan(b.routes_idx, b.T, b.K, b.E, false, plan_align(path), plan, ctx->max_rows,
                  ctx->max_mtiles, ctx->max_chunks, ctx->status, s, &launches);
  wm::prof_end(&ctx->prof, wm::kProfPlan, s);
  ctx->counters.launches += launches;
  if (int rc = check_launch(ctx, "plan")) return rc;
  if (int rc = run_experts(ctx, &b, false, path, s)) return rc;
  wm::launch_unpermute(ctx->routed, ctx->plan, b.T * b.K, b.H, static_cast<uint16_t*>(routed), ctx->num_sms, s);
  ctx->counters.launches += 1;
  ctx->counters.calls_pairs += 1;
  return check_launch(ctx, "unpermute");
}

WM_EXPORT int wm_combine(wm_ctx* ctx, int64_t T, int32_t H, int32_t K, const void* pairs, const int32_t* pair_pos,
                         const float* w, const void* shared, int32_t shared_gate, const void* x,
                         const void* shared_gate_weight, void* out, void* stream) {
  if (ctx == nullptr) return WM_ERROR;
  if (T < 0 || T > ctx->opt.max_tokens) return fail(ctx, "T out of range for this handle");
  if (T == 0) return WM_OK;
  if (H <= 0 || H % 8 != 0 || H > ctx->opt.max_hidden) return fail(ctx, "H must be a positive multiple of 8 within max_hidden");
  if (K <= 0 || K > ctx->opt.max_topk) return fail(ctx, "K out of range for this handle");
  if (shared_gate != WM_SHARED_NONE && shared_gate != WM_SHARED_SIGMOID_GATE && shared_gate != WM_SHARED_ONE)
    return fail(ctx, "unknown shared_gate");
  if (pairs == nullptr || !aligned(pairs, 16) || out == nullptr || !aligned(out, 16) || w == nullptr)
    return fail(ctx, "pairs and out must be 16-byte aligned device pointers, w non-null");
  if (shared_gate != WM_SHARED_NONE && (shared == nullptr || !aligned(shared, 16)))
    return fail(ctx, "the shared term needs 16-byte aligned shared rows");
  if (shared_gate == WM_SHARED_SIGMOID_GATE && (x == nullptr || shared_gate_weight == nullptr))
    return fail(ctx, "the sigmoid shared gate needs x and shared_gate_weight");
  DeviceGuard guard(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (shared_gate == WM_SHARED_SIGMOID_GATE) {
    wm::launch_shared_gate(static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(shared_gate_weight), int(T),
                           H, ctx->sg, s);
    ctx->counters.launches += 1;
  }
  wm::prof_begin(&ctx->prof, wm::kProfCombine, s);
  wm::launch_combine_dense(static_cast<const uint16_t*>(pairs), pair_pos, w, ctx->sg, shared_gate, int(T), H, K,
                           static_cast<const uint16_t*>(shared), static_cast<uint16_t*>(out), s);
  wm::prof_end(&ctx->prof, wm::kProfCombine, s);
  ctx->counters.launches += 1;
  return check_launch(ctx, "combine");
}

WM_EXPORT int wm_ep_plan(wm_ctx* ctx, int64_t T, int32_t K, int32_t experts_per_rank, int32_t world,
                         int32_t capacity, const int32_t* idx, const void* x, int32_t H, int32_t* send_counts,
                         int32_t* pair_pos, int32_t* send_eid, void* send_x, void* stream) {
  if (ctx == nullptr) return WM_ERROR;
  if (T < 0 || T > ctx->opt.max_tokens) return fail(ctx, "T out of range for this handle");
  if (K <= 0 || K > ctx->opt.max_topk) return fail(ctx, "K out of range for this handle");
  if (world <= 0 || world > ctx->opt.max_experts || experts_per_rank <= 0)
    return fail(ctx, "world must be in [1, max_experts] and experts_per_rank positive");
  if (H <= 0 || H % 8 != 0 || H > ctx->opt.max_hidden) return fail(ctx, "H must be a positive multiple of 8 within max_hidden");
  if (capacity != 0 && capacity < T * K) return fail(ctx, "capacity below T * K could drop pairs");
  if (T == 0) return WM_OK;
  if (idx == nullptr || x == nullptr || send_counts == nullptr || pair_pos == nullptr || send_eid == nullptr ||
      send_x == nullptr || !aligned(x, 16) || !aligned(send_x, 16))
    return fail(ctx, "wm_ep_plan needs device buffers (x and send_x 16-byte aligned)");
  DeviceGuard guard(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int P = int(T) * K;
  int launches = 0;
  wm::launch_ep_owner(idx, P, experts_per_rank, world, ctx->idx, ctx->status, ctx->num_sms, s);
  wm::Plan plan = ctx->plan;
  plan.rowmax = nullptr;
  wm::launch_plan(ctx->idx, int(T), K, world, false, 1, plan, ctx->max_rows, ctx->max_mtiles, ctx->max_chunks,
                  ctx->status, s, &launches);
  wm::launch_ep_finish(idx, plan, int(T), K, experts_per_rank, world, capacity, send_counts, pair_pos, send_eid,
                       static_cast<const uint16_t*>(x), H, static_cast<uint16_t*>(send_x), ctx->num_sms, s);
  if (capacity == 0)
    wm::launch_gather_rows(static_cast<const uint16_t*>(x), plan, world, H, static_cast<uint16_t*>(send_x),
                           ctx->num_sms, s);
  ctx->counters.launches += launches + (capacity == 0 ? 3 : 2);
  return check_launch(ctx, "expert-parallel plan");
}

// ---------------------------------------------------------------- expert parallelism over peer memory

struct wm_ep {
  int device = 0, world = 0, rank = 0, H = 0;
  int64_t capacity = 0;
  void* base = nullptr;  // this rank's exchange buffer (one cudaMalloc, exported through IPC)
  size_t bytes = 0;
  uint8_t* peer[wm::kMaxEpRanks] = {};  // every rank's buffer in this address space (own one included)
  size_t o_recv_x = 0, o_recv_e = 0, o_back = 0, o_flags = 0, o_counts = 0, o_ticket = 0, o_epoch = 0;
};

namespace {

bool ep_ready(const wm_ep* ep) {
  for (int r = 0; r < ep->world; ++r)
    if (ep->peer[r] == nullptr) return false;
  return true;
}

// The blocks this rank writes in every rank's buffer for exchange `which`
// (0: rows and ids to the owners' recv blocks, 1: results to the senders' back blocks).
wm::EpPeers ep_peers(const wm_ep* ep, int which) {
  wm::EpPeers pe{};
  const int64_t blk = int64_t(ep->rank) * ep->capacity;
  for (int r = 0; r < ep->world; ++r) {
    uint8_t* b = ep->peer[r];
    pe.rows[r] = reinterpret_cast<uint16_t*>(b + (which == 0 ? ep->o_recv_x : ep->o_back)) + blk * ep->H;
    pe.ids[r] = reinterpret_cast<int32_t*>(b + ep->o_recv_e) + blk;
    pe.flag[r] = reinterpret_cast<uint32_t*>(b + ep->o_flags) + which * ep->world + ep->rank;
    pe.count[r] = reinterpret_cast<int32_t*>(b + ep->o_counts) + ep->rank;
  }
  uint8_t* own = static_cast<uint8_t*>(ep->base);
  pe.ticket = reinterpret_cast<uint32_t*>(own + ep->o_ticket) + which;
  pe.epoch = reinterpret_cast<const uint32_t*>(own + ep->o_epoch);
  return pe;
}

}  // namespace

WM_EXPORT wm_ep* wm_ep_create(int32_t device, int32_t world, int32_t rank, int64_t capacity, int32_t H, char* error,
                              size_t error_size) {
  auto report = [&](const char* msg) {
    if (error != nullptr && error_size > 0) snprintf(error, error_size, "%s", msg);
  };
  if (world < 1 || world > wm::kMaxEpRanks || rank < 0 || rank >= world) {
    report("world must be in [1, 8] and rank in [0, world)");
    return nullptr;
  }
  if (capacity <= 0 || H <= 0 || H % 8) {
    report("capacity must be positive and H a positive multiple of 8");
    return nullptr;
  }
  wm_ep* ep = new (std::nothrow) wm_ep();
  if (ep == nullptr) {
    report("out of host memory");
    return nullptr;
  }
  ep->device = device;
  ep->world = world;
  ep->rank = rank;
  ep->capacity = capacity;
  ep->H = H;
  const size_t slots = size_t(world) * size_t(capacity);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes, 256);
    return at;
  };
  ep->o_recv_x = take(slots * H * 2);
  ep->o_recv_e = take(slots * 4);
  ep->o_back = take(slots * H * 2);
  ep->o_flags = take(size_t(2 * world) * 4);
  ep->o_counts = take(size_t(world) * 4);
  ep->o_ticket = take(8);
  ep->o_epoch = take(4);
  ep->bytes = off;
  DeviceGuard guard(device);
  if (cudaMalloc(&ep->base, ep->bytes) != cudaSuccess) {
    cudaGetLastError();
    report("cudaMalloc of the exchange buffer failed");
    delete ep;
    return nullptr;
  }
  uint8_t* b = static_cast<uint8_t*>(ep->base);
  if (cudaMemset(b + ep->o_flags, 0, off - ep->o_flags) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    report("initialising the exchange buffer failed");
    cudaFree(ep->base);
    delete ep;
    return nullptr;
  }
  ep->peer[rank] = b;
  return ep;
}

WM_EXPORT void wm_ep_destroy(wm_ep* ep) {
  if (ep == nullptr) return;
  {
    DeviceGuard guard(ep->device);
    for (int r = 0; r < ep->world; ++r)
      if (r != ep->rank && ep->peer[r] != nullptr) cudaIpcCloseMemHandle(ep->peer[r]);
    cudaFree(ep->base);
  }
  delete ep;
}

WM_EXPORT int wm_ep_ipc_handle(wm_ep* ep, void* handle64) {
  if (ep == nullptr || handle64 == nullptr) return WM_ERROR;
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handles are 64 bytes");
  DeviceGuard guard(ep->device);
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ep->base) != cudaSuccess) {
    cudaGetLastError();
    return WM_ERROR;
  }
  memcpy(handle64, &h, sizeof(h));
  return WM_OK;
}

WM_EXPORT int wm_ep_open_peer(wm_ep* ep, int32_t peer, const void* handle64) {
  if (ep == nullptr || handle64 == nullptr || peer < 0 || peer >= ep->world || peer == ep->rank) return WM_ERROR;
  if (ep->peer[peer] != nullptr) return WM_OK;
  DeviceGuard guard(ep->device);
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return WM_ERROR;
  }
  ep->peer[peer] = static_cast<uint8_t*>(p);
  return WM_OK;
}

WM_EXPORT void* wm_ep_buffer(wm_ep* ep, int32_t which) {
  if (ep == nullptr) return nullptr;
  uint8_t* b = static_cast<uint8_t*>(ep->base);
  switch (which) {
    case 0: return b + ep->o_recv_x;
    case 1: return b + ep->o_recv_e;
    case 2: return b + ep->o_back;
    default: return nullptr;
  }
}

WM_EXPORT int wm_ep_dispatch(wm_ctx* ctx, wm_ep* ep, int64_t T, int32_t K, int32_t experts_per_rank,
                             const int32_t* idx, const void* x, int32_t* pair_pos, void* stream) {
  if (ctx == nullptr) return WM_ERROR;
  if (ep == nullptr || !ep_ready(ep)) return fail(ctx, "the exchange buffer has unopened peers");
  if (ep->device != ctx->device) return fail(ctx, "the exchange buffer lives on another device");
  if (T < 0 || T > ctx->opt.max_tokens) return fail(ctx, "T out of range for this handle");
  if (K <= 0 || K > ctx->opt.max_topk || experts_per_rank <= 0) return fail(ctx, "K or experts_per_rank out of range");
  if (T * K > ep->capacity) return fail(ctx, "T * K = %lld exceeds the exchange capacity %lld", (long long)(T * K),
                                        (long long)ep->capacity);
  if (ep->world > ctx->opt.max_experts) return fail(ctx, "world exceeds the handle's max_experts");
  if (idx == nullptr || x == nullptr || pair_pos == nullptr || !aligned(x, 16))
    return fail(ctx, "wm_ep_dispatch needs device idx, pair_pos and 16-byte aligned x");
  DeviceGuard guard(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* own = static_cast<uint8_t*>(ep->base);
  wm::prof_begin(&ctx->prof, wm::kProfEpSend, s);
  const int P = int(T) * K;
  if (P > 0 && wm::ep_dispatch_small_ok(P, ep->world, int(ep->capacity))) {  // decode-sized: one launch
    wm::launch_ep_dispatch_small(idx, int(T), K, experts_per_rank, ep->world, int(ep->capacity), pair_pos,
                                 static_cast<const uint16_t*>(x), ep->H, ep_peers(ep, 0),
                                 reinterpret_cast<uint32_t*>(own + ep->o_epoch), ctx->status, ctx->num_sms, s);
    wm::prof_end(&ctx->prof, wm::kProfEpSend, s);
    ctx->counters.launches += 1;
    return check_launch(ctx, "expert-parallel dispatch");
  }
  wm::launch_ep_begin(reinterpret_cast<uint32_t*>(own + ep->o_epoch), s);
  int launches = 0;
  wm::Plan plan = ctx->plan;
  plan.rowmax = nullptr;
  if (P > 0) {
    wm::launch_ep_owner(idx, P, experts_per_rank, ep->world, ctx->idx, ctx->status, ctx->num_sms, s);
    wm::launch_plan(ctx->idx, int(T), K, ep->world, false, 1, plan, ctx->max_rows, ctx->max_mtiles, ctx->max_chunks,
                    ctx->status, s, &launches);
    launches += 1;
  } else {
    cudaMemsetAsync(plan.counts, 0, sizeof(int32_t) * (ep->world + 1), s);  // every block is padding
  }
  wm::launch_ep_send(idx, plan, int(T), K, experts_per_rank, ep->world, int(ep->capacity), pair_pos,
                     static_cast<const uint16_t*>(x), ep->H, ep_peers(ep, 0), ctx->num_sms, s);
  wm::prof_end(&ctx->prof, wm::kProfEpSend, s);
  ctx->counters.launches += launches + 2;
  return check_launch(ctx, "expert-parallel dispatch");
}

WM_EXPORT int wm_ep_return(wm_ctx* ctx, wm_ep* ep, const void* y, void* stream) {
  if (ctx == nullptr) return WM_ERROR;
  if (ep == nullptr || !ep_ready(ep)) return fail(ctx, "the exchange buffer has unopened peers");
  if (y == nullptr || !aligned(y, 16)) return fail(ctx, "y must be a 16-byte aligned device pointer");
  DeviceGuard guard(ctx->device);
  const uint8_t* own = static_cast<const uint8_t*>(ep->base);
  wm::prof_begin(&ctx->prof, wm::kProfEpReturn, static_cast<cudaStream_t>(stream));
  wm::launch_ep_return(static_cast<const uint16_t*>(y), reinterpret_cast<const int32_t*>(own + ep->o_recv_e),
                       ep->world, int(ep->capacity), ep->H, ep_peers(ep, 1), ctx->num_sms,
                       static_cast<cudaStream_t>(stream));
  wm::prof_end(&ctx->prof, wm::kProfEpReturn, static_cast<cudaStream_t>(stream));
  ctx->counters.launches += 1;
  return check_launch(ctx, "expert-parallel return");
}

WM_EXPORT int wm_ep_wait(wm_ctx* ctx, wm_ep* ep, int32_t which, void* stream) {
  if (ctx == nullptr) return WM_ERROR;
  if (ep == nullptr || which < 0 || which > 1) return fail(ctx, "wm_ep_wait: bad buffer or exchange");
  DeviceGuard guard(ctx->device);
  const uint8_t* own = static_cast<const uint8_t*>(ep->base);
  const int slot = which == 0 ? wm::kProfEpWaitDispatch : wm::kProfEpWaitReturn;
  wm::prof_begin(&ctx->prof, slot, static_cast<cudaStream_t>(stream));
  wm::launch_ep_wait(reinterpret_cast<const uint32_t*>(own + ep->o_flags) + which * ep->world, ep->world,
                     reinterpret_cast<const uint32_t*>(own + ep->o_epoch), ctx->status, 60 + which,
                     static_cast<cudaStream_t>(stream));
  wm::prof_end(&ctx->prof, slot, static_cast<cudaStream_t>(stream));
  ctx->counters.launches += 1;
  return check_launch(ctx, "expert-parallel wait");
}

WM_EXPORT int wm_ep_experts(wm_ctx* ctx, wm_ep* ep, const wm_moe_args* args, void* stream) {
  if (ctx == nullptr) return WM_ERROR;
  if (ep == nullptr || !ep_ready(ep)) return fail(ctx, "the exchange buffer has unopened peers");
  if (ep->device != ctx->device) return fail(ctx, "the exchange buffer lives on another device");
  if (args == nullptr) return fail(ctx, "args is NULL");
  const int64_t slots = int64_t(ep->world) * ep->capacity;
  if (slots > ctx->opt.max_tokens)
    return fail(ctx, "the exchange buffer's %lld slots exceed the handle's max_tokens", (long long)slots);
  if (args->H != ep->H) return fail(ctx, "H = %d differs from the exchange buffer's %d", args->H, ep->H);
  if (args->T < 1 || args->T > slots) return fail(ctx, "T (the rows expected) must lie in [1, %lld]", (long long)slots);
  uint8_t* own = static_cast<uint8_t*>(ep->base);
  // the experts read the received rows as x, one route per slot
  wm_moe_args b = *args;
  b.K = 1;
  b.x = own + ep->o_recv_x;
  b.routes_idx = reinterpret_cast<const int32_t*>(own + ep->o_recv_e);
  b.shared_gate = WM_SHARED_NONE;
  b.router_weight = nullptr;
  b.norm_weight = nullptr;
  if (int rc = validate_experts(ctx, &b, false)) return rc;
  DeviceGuard guard(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the kernels are picked by the rows expected (b.T); the GEMV sizes its grid
  // by T, so it takes every slot
  const Path path = expert_path(ctx, &b, false);
  if (path == kPathGemv) b.T = int32_t(slots);
  wm::Plan plan = ctx->plan;
  plan_for_path(ctx, path, &plan);
  const int32_t* counts = reinterpret_cast<const int32_t*>(own + ep->o_counts);
  int launches = 0;
  wm::prof_begin(&ctx->prof, wm::kProfPlan, s);
  wm::launch_plan_blocks(b.routes_idx, counts, ep->world, int(ep->capacity), b.E, plan_align(path),
                         plan, ctx->max_rows, ctx->max_mtiles, ctx->max_chunks, ctx->status, s, &launches);
  wm::prof_end(&ctx->prof, wm::kProfPlan, s);
  ctx->counters.launches += launches;
  if (int rc = check_launch(ctx, "plan")) return rc;
  // the grouped GEMM and the block-scaled decode kernel store the down rows
  // straight into the senders' back blocks (the return overlaps the math);
  // the other kernels leave them sorted and a copy kernel returns them
  const wm::EpPeers back = ep_peers(ep, 1);
  const bool fused = path == kPathGemm || path == kPathBsGemm || path == kPathFp8Gemm || path == kPathBsDecode;
  wm::EpReturn ret{};
  if (fused) {
    for (int r = 0; r < ep->world; ++r) ret.rows[r] = back.rows[r];
    ret.capacity = int(ep->capacity);
  }
  const XRows xr{slots, counts, int(ep->capacity)};  // the x rows are the recv slots
  if (int rc = run_experts(ctx, &b, false, path, s, fused ? &ret : nullptr, &xr)) return rc;
  wm::prof_begin(&ctx->prof, wm::kProfEpReturn, s);
  if (fused)
    wm::launch_ep_signal(back, ep->world, s);
  else
    wm::launch_ep_return_sorted(ctx->routed, ctx->plan.pair_pos, counts, ep->world, int(ep->capacity), ep->H,
                                back, ctx->num_sms, s);
  wm::prof_end(&ctx->prof, wm::kProfEpReturn, s);
  ctx->counters.launches += 1;
  ctx->counters.calls_pairs += 1;
  return check_launch(ctx, "expert-parallel experts and return");
}

WM_EXPORT int wm_moe_forward(wm_ctx* ctx, const wm_moe_args* args, void* stream) {
  if (ctx == nullptr) return WM_ERROR;
  if (int rc = validate_experts(ctx, args, true)) return rc;
  if (args->T == 0) return WM_OK;
  if (args->out == nullptr || !aligned(args->out, 16)) return fail(ctx, "out must be a 16-byte aligned device pointer");
  DeviceGuard guard(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // With a pre-MoE norm, everything after the router reads the normalised
  // rows: the router writes them (or the RMSNorm kernel does, without one).
  wm_moe_args na = *args;
  const wm_moe_args* a = &na;
  if (args->norm_weight != nullptr) {
    na.x = norm_rows(ctx, args);
    na.norm_weight = nullptr;
    if (args->router_weight == nullptr) run_rmsnorm(ctx, args, s);
  }
  const bool has_shared = a->shared_gate != WM_SHARED_NONE;
  const Path path = expert_path(ctx, a, has_shared);
  wm::Plan plan = ctx->plan;
  plan_for_path(ctx, path, &plan);
  plan.skip_negative = (ctx->opt.flags & WM_FLAG_SKIP_NEGATIVE_ROUTES) ? 1 : 0;
  const int32_t* idx;
  const float* w;
  const int align = plan_align(path);
  // Small router calls on the block-scaled decode path select, plan and
  // quantise the token rows in one launch after the logits.
  const bool small = a->router_weight != nullptr && path == kPathBsDecode &&
                     !(ctx->opt.flags & WM_FLAG_SPLIT_SMALL_CALLS) &&
                     wm::bs_route_plan_quant_ok(a->T, a->K, a->E, a->router);
  if (a->router_weight != nullptr) {
    int32_t* di = a->out_idx ? a->out_idx : ctx->idx;
    float* dw = a->out_w ? a->out_w : ctx->w;
    if (int rc = run_router(ctx, args, ctx->logits, di, dw, s, !small)) return rc;
    idx = di;
    w = dw;
    if (small) {
      const wm::TopkArgs tk{a->router_bias, a->K, a->router, a->n_groups, a->topk_groups, a->route_scale, di, dw};
      wm::prof_begin(&ctx->prof, wm::kProfRoutePlanQuant, s);
      wm::launch_bs_route_plan_quant(ctx->logits, a->T, a->E, tk, has_shared, plan, ctx->max_rows, ctx->max_mtiles,
                                     ctx->status, static_cast<const uint16_t*>(a->x), a->H, ctx->bs_img_x, s);
      wm::prof_end(&ctx->prof, wm::kProfRoutePlanQuant, s);
      ctx->counters.launches += 1;
      if (int rc = check_launch(ctx, "route, plan and quantise")) return rc;
    }
  } else {
    idx = a->routes_idx;
    w = a->routes_w;
    if (a->shared_gate == WM_SHARED_SIGMOID_GATE) {
      wm::launch_shared_gate(static_cast<const uint16_t*>(a->x),
                             static_cast<const uint16_t*>(a->shared_gate_weight), a->T, a->H, ctx->sg, s);
      ctx->counters.launches += 1;
    }
  }
  // Calls of up to 64 tokens (after the top-k or with given routes) plan and
  // quantise the token rows in one launch.
  const bool mid = !small && path == kPathBsDecode && !(ctx->opt.flags & WM_FLAG_SPLIT_SMALL_CALLS) &&
                   wm::bs_plan_quant_ok(a->T, a->K, a->E);
  if (mid) {
    wm::prof_begin(&ctx->prof, wm::kProfRoutePlanQuant, s);
    wm::launch_bs_plan_quant(idx, a->T, a->K, a->E, has_shared, plan, ctx->max_rows, ctx->max_mtiles, ctx->status,
                             static_cast<const uint16_t*>(a->x), a->H, ctx->bs_img_x, s);
    wm::prof_end(&ctx->prof, wm::kProfRoutePlanQuant, s);
    ctx->counters.launches += 1;
    if (int rc = check_launch(ctx, "plan and quantise")) return rc;
  } else if (!small) {
    int launches = 0;
    wm::prof_begin(&ctx->prof, wm::kProfPlan, s);
    wm::launch_plan(idx, a->T, a->K, a->E, has_shared, align, plan, ctx->max_rows, ctx->max_mtiles, ctx->max_chunks,
                    ctx->status, s, &launches);
    wm::prof_end(&ctx->prof, wm::kProfPlan, s);
    ctx->counters.launches += launches;
    if (int rc = check_launch(ctx, "plan")) return rc;
  }
  if (int rc = run_experts(ctx, a, has_shared, path, s, nullptr, nullptr, small || mid)) return rc;
  wm::prof_begin(&ctx->prof, wm::kProfCombine, s);
  wm::launch_combine(ctx->routed, ctx->plan, w, ctx->sg, a->shared_gate, a->T, a->H, a->E, a->K,
                     static_cast<uint16_t*>(a->out), s);
  wm::prof_end(&ctx->prof, wm::kProfCombine, s);
  ctx->counters.launches += 1;
  ctx->counters.calls_forward += 1;
  return check_launch(ctx, "combine");
}

WM_EXPORT int wm_profile_enable(wm_ctx* ctx, int32_t enable) {
  if (ctx == nullptr) return WM_ERROR;
  DeviceGuard guard(ctx->device);
  ctx->prof.collect();
  ctx->prof.enabled = enable != 0;
  return WM_OK;
}

WM_EXPORT int32_t wm_profile_read(wm_ctx* ctx, wm_profile_entry* out, int32_t max_entries) {
  if (ctx == nullptr || out == nullptr) return 0;
  DeviceGuard guard(ctx->device);
  ctx->prof.collect();
  int32_t n = 0;
  for (int sl = 0; sl < wm::kProfSlots && n < max_entries; ++sl) {
    if (ctx->prof.launches[sl] == 0) continue;
    snprintf(out[n].name, sizeof(out[n].name), "%s", wm::prof_name(sl));
    out[n].launches = ctx->prof.launches[sl];
    out[n].total_ms = ctx->prof.total_ms[sl];
    ++n;
  }
  return n;
}

WM_EXPORT void wm_profile_reset(wm_ctx* ctx) {
  if (ctx == nullptr) return;
  DeviceGuard guard(ctx->device);
  ctx->prof.reset();
}

}  // extern "C"
