// wm_moe_forward_noalloc: the decode MoE block with no device allocation.
//
// Every other entry point works through a handle whose workspace wm_create
// obtains with cudaMalloc.  Some callers cannot do that: a serving loop whose
// GPU memory is fixed when the process starts (a cudaMalloc mid-run also
// waits for the whole device), or a host framework that owns all device
// memory through its own allocator and forbids other allocations.  For them
// this entry point runs the same kernels as wm_moe_forward's decode path
// (router, sort, expert GEMVs, shared expert, combine) with all scratch in
// one file-scope device array of kScratchBytes per GPU, which the CUDA
// runtime reserves when it loads this file's module on that GPU and keeps
// until the process exits.
//
// * The first call on a device sets that device up: it looks up the array's
//   device address with cudaGetSymbolAddress, which is also when the runtime
//   loads the module and reserves the array (CUDA loads modules lazily by
//   default).  Make that first call -- or a call of
//   wm_moe_forward_noalloc_status -- at start-up, before device memory is
//   fixed and before any stream capture, or run with CUDA_MODULE_LOADING=EAGER.
// * All calls share the one array and it keeps the last call's contents:
//   calls that may overlap on the GPU (on different streams, or from several
//   host threads) race with each other.  Serialise them.
// * Sizes whose scratch would exceed the array are rejected with an error.
// * Errors the kernels find on the device (an expert id outside [0, E)) are
//   recorded in the array's status words; wm_moe_forward_noalloc_status waits
//   for the stream and reports them.  A route with a bad expert id
//   contributes nothing to its token's output.  FP8 NaN codes are not checked
//   on this path (wm_moe_forward reports them).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <mutex>

#include "wm_kernels.h"

namespace wm {
namespace {

constexpr size_t kScratchBytes = size_t(8) << 20;  // 8 MiB per GPU

static __device__ __align__(256) uint8_t g_scratch[kScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};
int g_major[kMaxDevices] = {};          // compute capability, 0 = not looked up
int g_smem_optin[kMaxDevices] = {};     // largest opt-in shared memory per block


int report(char* error, size_t n, const char* msg) {
  if (error != nullptr && n > 0) snprintf(error, n, "%s", msg);
  return WM_ERROR;
}

size_t up256(size_t v) { return (v + 255) / 256 * 256; }

// The array's device address and the device's limits, looked up once per
// device (the current one).  The status words sit at the array's start.
constexpr size_t kStatusBytes = 256;

bool device_setup(int* dev_out, char* msg, size_t n) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    snprintf(msg, n, "no current CUDA device");
    return false;
  }
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess || p == nullptr) {
      snprintf(msg, n, "cudaGetSymbolAddress of the scratch array failed: %s", cudaGetErrorString(e));
      return false;
    }
    g_scratch_ptr[dev] = p;
  }
  // device queries once per device: a cudaGetDeviceProperties per call costs
  // milliseconds of host time
  if (g_major[dev] == 0) {
    int major = 0, optin = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) {
      snprintf(msg, n, "CUDA device attributes could not be read");
      return false;
    }
    g_major[dev] = major;
    g_smem_optin[dev] = optin;
  }
  if (g_major[dev] != 10) {
    snprintf(msg, n, "needs an sm_100 (B200-class) GPU");
    return false;
  }
  *dev_out = dev;
  return true;
}

}  // namespace
}  // namespace wm

extern "C" WM_EXPORT int wm_moe_forward_noalloc(const wm_moe_args* a, void* stream, char* error, size_t error_size) {
  using namespace wm;
  char msg[256];
  if (a == nullptr) return report(error, error_size, "args is NULL");
  if (a->T < 0 || a->H <= 0 || a->I <= 0 || a->E <= 0 || a->K <= 0 || a->K > a->E)
    return report(error, error_size, "invalid shape (T >= 0, H, I, E, K > 0, K <= E)");
  if (a->E > 1024 || a->K > 64) return report(error, error_size, "at most 1024 experts and top-64 routing");
  if (a->H % 64 || a->I % 64) return report(error, error_size, "H and I must be multiples of 64");
  if (a->layout < WM_LAYOUT_QWEN_GATE_UP_MXFP4 || a->layout > WM_LAYOUT_W13_FP8_B32)
    return report(error, error_size, "unknown expert layout");
  if (a->layout == WM_LAYOUT_W13_FP8_B128 && (a->H % 128 || a->I % 128))
    return report(error, error_size, "FP8 128x128 experts need H and I multiples of 128");
  if (a->T == 0) return WM_OK;
  auto al = [](const void* p, size_t n) { return p != nullptr && reinterpret_cast<uintptr_t>(p) % n == 0; };
  if (!al(a->x, 16) || !al(a->out, 16)) return report(error, error_size, "x and out must be 16-byte aligned device pointers");
  if (!al(a->w13.weight, 16) || !al(a->w2.weight, 16) || a->w13.weight_stride % 16 || a->w2.weight_stride % 16 ||
      a->w13.scale == nullptr || a->w2.scale == nullptr)
    return report(error, error_size, "expert weights must be 16-byte aligned regions with scales");
  const bool has_shared = a->shared_gate != WM_SHARED_NONE;
  if (has_shared && (!al(a->shared_w13.weight, 16) || !al(a->shared_w2.weight, 16) || a->shared_w13.scale == nullptr ||
                     a->shared_w2.scale == nullptr ||
                     (a->shared_gate == WM_SHARED_SIGMOID_GATE && !al(a->shared_gate_weight, 16))))
    return report(error, error_size, "shared expert weights, scales (and sigmoid gate weight) must be given, aligned");
  const bool norm = a->norm_weight != nullptr;
  if (norm) {
    if (!al(a->norm_weight, 16) || !al(a->x_norm, 16))
      return report(error, error_size, "a norm weight needs 16-byte aligned norm_weight and x_norm (the caller's rows)");
    const uintptr_t x0 = uintptr_t(a->x), n0 = uintptr_t(a->x_norm), bytes = uintptr_t(a->T) * a->H * 2;
    if (n0 < x0 + bytes && x0 < n0 + bytes) return report(error, error_size, "x_norm must not overlap x");
    if (!(a->norm_eps >= 0.0f) || a->norm_eps > 3.0e38f) return report(error, error_size, "norm_eps must be finite and >= 0");
  }
  const bool route_here = a->router_weight != nullptr;
  if (!route_here && (a->routes_idx == nullptr || a->routes_w == nullptr))
    return report(error, error_size, "give router_weight or routes_idx and routes_w");
  if (route_here && a->router == WM_ROUTER_SIGMOID_GROUPED &&
      (a->n_groups < 1 || a->n_groups > 32 || a->E % a->n_groups || a->topk_groups < 1 ||
       a->topk_groups > a->n_groups || a->K > a->topk_groups * (a->E / a->n_groups)))
    return report(error, error_size, "invalid group-limited routing shape");
  const int64_t T = a->T, K = a->K, E = a->E, H = a->H, I = a->I;
  if (T * K > 8192) return report(error, error_size, "at most 8192 (token, expert) pairs per call");

  // scratch layout (GEMV path: no row padding)
  const int64_t rows = T * K + T;
  // unpadded groups are cut into 16-row tiles: at most rows / 16 + one partial tile per group
  const int max_mtiles = int(rows / 16 + E + 2);
  size_t off = kStatusBytes;  // the status words come first
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = up256(off + bytes);
    return at;
  };
  const size_t o_counts = take((E + 1) * 4), o_offsets = take((E + 2) * 4), o_pair = take(T * K * 4),
               o_rowtok = take(rows * 4), o_unique = take((E + 1) * 4), o_nu = take(4),
               o_mt = take(size_t(max_mtiles) * 8), o_nm = take(4), o_act = take(rows * I * 2),
               o_routed = take(rows * H * 2), o_logits = take(T * E * 4), o_idx = take(T * K * 4),
               o_w = take(T * K * 4), o_sg = take(T * 4);
  if (off > kScratchBytes) {
    snprintf(msg, sizeof(msg), "this call needs %.2f MiB of scratch; the allocation-free entry point has %.0f MiB",
             off / 1048576.0, kScratchBytes / 1048576.0);
    return report(error, error_size, msg);
  }
  const size_t gemv_smem = gemv_smem_bytes(int(H), int(I)), router_smem = router_smem_bytes(int(H));

  // once per device: the array's device address
  int dev = 0;
  if (!device_setup(&dev, msg, sizeof(msg))) return report(error, error_size, msg);
  if (gemv_smem > size_t(g_smem_optin[dev]) || router_smem > size_t(g_smem_optin[dev]))
    return report(error, error_size, "H is too large for the decode kernels' shared-memory staging");
  gemv_init_attributes(int(gemv_smem));  // raise-only, cheap after the first call
  router_init_attributes(int(H));

  uint8_t* base = static_cast<uint8_t*>(g_scratch_ptr[dev]);
  Plan p{};
  p.counts = reinterpret_cast<int32_t*>(base + o_counts);
  p.offsets = reinterpret_cast<int32_t*>(base + o_offsets);
  p.pair_pos = reinterpret_cast<int32_t*>(base + o_pair);
  p.row_token = reinterpret_cast<int32_t*>(base + o_rowtok);
  p.unique = reinterpret_cast<int32_t*>(base + o_unique);
  p.n_unique = reinterpret_cast<int32_t*>(base + o_nu);
  p.mtiles = reinterpret_cast<int32_t*>(base + o_mt);
  p.n_mtiles = reinterpret_cast<int32_t*>(base + o_nm);
  p.hist = nullptr;
  uint16_t* act = reinterpret_cast<uint16_t*>(base + o_act);
  uint16_t* routed = reinterpret_cast<uint16_t*>(base + o_routed);
  float* logits = reinterpret_cast<float*>(base + o_logits);
  float* sg = reinterpret_cast<float*>(base + o_sg);
  uint32_t* status = reinterpret_cast<uint32_t*>(base);
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  // the status words start at zero; everything else is written before it is read
  cudaMemsetAsync(status, 0, 16, s);
  const int32_t* idx = a->routes_idx;
  const float* w = a->routes_w;
  const uint16_t* x = static_cast<const uint16_t*>(a->x);
  const uint16_t* sg_w =
      a->shared_gate == WM_SHARED_SIGMOID_GATE ? static_cast<const uint16_t*>(a->shared_gate_weight) : nullptr;
  // the pre-MoE RMSNorm: fused into the router's logits kernel where it takes the shape
  uint16_t* xn = static_cast<uint16_t*>(a->x_norm);
  const uint16_t* nw = static_cast<const uint16_t*>(a->norm_weight);
  const bool fused = norm && route_here && router_logits_fused_ok(int(T), int(H), int(E));
  if (norm && !fused) {
    launch_rmsnorm(x, nw, int(T), int(H), a->norm_eps, xn, s);
    x = xn;
  }
  if (route_here) {
    int32_t* di = a->out_idx ? a->out_idx : reinterpret_cast<int32_t*>(base + o_idx);
    float* dw = a->out_w ? a->out_w : reinterpret_cast<float*>(base + o_w);
    launch_router_logits(x, static_cast<const uint16_t*>(a->router_weight), sg_w, int(T), int(H), int(E), logits, sg, s,
                         fused ? nw : nullptr, a->norm_eps, fused ? xn : nullptr);
    if (fused) x = xn;
    launch_router_topk(logits, int(T), int(E),
                       TopkArgs{a->router_bias, int(K), a->router, a->n_groups, a->topk_groups, a->route_scale, di, dw},
                       s);
    idx = di;
    w = dw;
  } else if (sg_w != nullptr) {
    launch_router_logits(x, nullptr, sg_w, int(T), int(H), 0, nullptr, sg, s);
  }
  int launches = 0;
  launch_plan(idx, int(T), int(K), int(E), has_shared, 1, p, int(rows), max_mtiles, 1, status, s, &launches);
  GemvArgs g{};
  g.plan = p;
  g.wts.w13 = static_cast<const uint8_t*>(a->w13.weight);
  g.wts.w13_stride = a->w13.weight_stride;
  g.wts.s13 = static_cast<const uint8_t*>(a->w13.scale);
  g.wts.s13_stride = a->w13.scale_stride;
  g.wts.w2 = static_cast<const uint8_t*>(a->w2.weight);
  g.wts.w2_stride = a->w2.weight_stride;
  g.wts.s2 = static_cast<const uint8_t*>(a->w2.scale);
  g.wts.s2_stride = a->w2.scale_stride;
  if (has_shared) {
    g.wts.sh_w13 = static_cast<const uint8_t*>(a->shared_w13.weight);
    g.wts.sh_s13 = static_cast<const uint8_t*>(a->shared_w13.scale);
    g.wts.sh_w2 = static_cast<const uint8_t*>(a->shared_w2.weight);
    g.wts.sh_s2 = static_cast<const uint8_t*>(a->shared_w2.scale);
  }
  g.wts.E = int(E);
  g.x = x;
  g.act = act;
  g.routed = routed;
  g.H = int(H);
  g.I = int(I);
  g.gate_first = a->layout == WM_LAYOUT_QWEN_GATE_UP_MXFP4 ? 1 : 0;
  g.limit = a->swiglu_limit;
  const int max_unique = int(std::min<int64_t>(E, T * K)) + (has_shared ? 1 : 0);
  launch_gemv(g,
              a->layout == WM_LAYOUT_W13_FP8_B128  ? kFmtFp8B128
              : a->layout == WM_LAYOUT_W13_FP8_B32 ? kFmtFp8B32
                                                   : kFmtMxfp4,
              max_unique, s, nullptr);
  launch_combine(routed, p, w, sg, a->shared_gate, int(T), int(H), int(E), int(K), static_cast<uint16_t*>(a->out), s);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    snprintf(msg, sizeof(msg), "CUDA launch failed: %s", cudaGetErrorString(e));
    return report(error, error_size, msg);
  }
  return WM_OK;
}

extern "C" WM_EXPORT int wm_moe_forward_noalloc_status(void* stream, char* error, size_t error_size) {
  using namespace wm;
  char msg[256];
  int dev = 0;
  if (!device_setup(&dev, msg, sizeof(msg))) return report(error, error_size, msg);
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    snprintf(msg, sizeof(msg), "stream synchronisation failed: %s", cudaGetErrorString(e));
    return report(error, error_size, msg);
  }
  uint32_t st[2] = {0, 0};
  e = cudaMemcpy(st, g_scratch_ptr[dev], sizeof(st), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    snprintf(msg, sizeof(msg), "reading the status words failed: %s", cudaGetErrorString(e));
    return report(error, error_size, msg);
  }
  switch (st[0]) {
    case kStatusOk:
      return WM_OK;
    case kStatusBadExpert:
      snprintf(msg, sizeof(msg), "expert ID is outside the model (pair %u)", st[1]);
      break;
    case kStatusOverflow:
      snprintf(msg, sizeof(msg), "sorted rows exceeded the scratch array (%u)", st[1]);
      break;
    case kStatusNanCode:
      snprintf(msg, sizeof(msg), "FP8 weights contain reserved NaN codes (row %u)", st[1]);
      break;
    default:
      snprintf(msg, sizeof(msg), "device status %u (%u)", st[0], st[1]);
  }
  return report(error, error_size, msg);
}
