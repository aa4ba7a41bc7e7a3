/*
 * whallm_moe.h -- C ABI of the B200 MoE expert-FFN library (libwhallm_moe.so).
 *
 * Replaces the expert arithmetic that Whallm's Python runtime reaches through
 * MLX and its native engines reach through Metal:
 *
 *   mx.gather_qmm / mx.quantized_matmul(mode="mxfp4", group_size=32)
 *       runtime/deepseek_v4_ssd/model.py:435-513, qwen4_exp.py:774-783, 853-904
 *   router + top-k        qwen4_exp.py:1009-1047, deepseek_v41/moe.py:46-74,
 *                         mimo/model.py:132-150, Native/QwenNative/engine.mm:2085-2101,
 *                         Native/DeepSeekNative/engine.mm:1863-1890
 *   sort / permute        qwen_expert_waves.py:23-51, Native/QwenNative/engine.mm:2105-2127
 *   SwiGLU + combine      qwen4_exp.py:815-818, 1049-1051; deepseek_v41/moe.py:30-43, 105-112;
 *                         Native/QwenNative/kernels.metal:175-194, 756-765
 *   shared expert         qwen4_exp.py:1046, deepseek_v41/moe.py:77-93
 *
 * Conventions follow the reference's native C ABI (Native/QwenNative/capi.h:1-5):
 * an opaque handle; functions returning int return 0 on success, 1 on an error
 * (text from wm_error) and 2 when a call was cancelled; calls on one handle
 * come from one host thread at a time.  Unlike the reference, a failed call
 * leaves the handle usable.
 *
 * Every pointer named "device" is CUDA device memory of the handle's GPU
 * (the caller owns it; PyTorch tensors in practice).  Every call is enqueued
 * on the caller's CUDA stream (`stream`, a cudaStream_t; NULL = the legacy
 * default stream) and returns without waiting for the GPU; wm_sync waits and
 * reports errors that kernels recorded on the device.
 *
 * Expert weights are used in place, in the reference's on-disk blob layout
 * (runtime/deepseek_v4_ssd/expert_layout.py:8-166): a projection of expert e
 * starts at `weight + e * weight_stride`, its scales at
 * `scale + e * scale_stride`.  This covers both the slot-major arena and the
 * region-major layer buffer of batched_layer_layout (expert_layout.py:83-119),
 * whose (base, stride, inner) triple becomes weight = buffer + base + inner,
 * weight_stride = stride.
 */
#ifndef WHALLM_MOE_H
#define WHALLM_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
#define WM_EXPORT __attribute__((visibility("default")))
extern "C" {
#else
#define WM_EXPORT __attribute__((visibility("default")))
#endif

#define WM_OK 0
#define WM_ERROR 1
#define WM_CANCELLED 2

typedef struct wm_ctx wm_ctx;

/* Expert blob layouts (the weights of one expert). */
enum wm_layout {
  /* Qwen: gate_up.weight | gate_up.scale | down.weight | down.scale;
     gate rows [0, I) then up rows [I, 2I) (Sources/DeepSeekRepack/Qwen.swift:51-65). */
  WM_LAYOUT_QWEN_GATE_UP_MXFP4 = 0,
  /* DeepSeek / MiMo: w3 | w1 | w2 | w3.s | w1.s | w2.s, w13 = [w3; w1]:
     up rows first (expert_layout.py:8-63, model.py:452-461). */
  WM_LAYOUT_DS_W13_MXFP4 = 1,
  /* FP8 E4M3 experts with fp32 128x128 block scales: w13.weight | w2.weight |
     w13.scale | w2.scale, w13 = [w3; w1] (up rows first).  New layout: the
     reference decodes this format only for resident tensors
     (mimo/weights.py:17-43). */
  WM_LAYOUT_W13_FP8_B128 = 2,
  /* FP8 E4M3 experts with UE8M0 32x32 block scales (the V4.1 dense FP8
     format, dequant.py:45-50): w13 = [w3; w1] (up rows first) E4M3 [2I, H]
     with scales [2I/32, H/32] bytes, w2 E4M3 [H, I] with scales [H/32, I/32];
     scale rows 2-byte aligned.  For the V4.1 shared expert and dense FP8
     FFNs (one expert, every token routed to it).  New layout: the reference
     keeps this format only for resident tensors. */
  WM_LAYOUT_W13_FP8_B32 = 3,
};

/* Weight formats for wm_dequant. */
enum wm_format {
  WM_FORMAT_MXFP4 = 0,     /* packed E2M1 [rows, cols/2] + E8M0 [rows, cols/32] */
  WM_FORMAT_FP8_B128 = 1,  /* E4M3 [rows, cols] + fp32 [ceil(rows/128), ceil(cols/128)] */
  WM_FORMAT_FP8_B32 = 2,   /* E4M3 [rows, cols] + UE8M0 [ceil(rows/32), ceil(cols/32)] */
};

/* Decode conventions where the reference's two decoders differ. */
enum wm_convention {
  WM_CONV_MLX = 0,    /* E2M1 code 8 -> +0; E8M0 byte 0 -> 2^-127 (deepseek_v41/dequant.py:27-35) */
  WM_CONV_METAL = 1,  /* code 8 -> -0; byte 0 -> 0 (Native/QwenNative/kernels.metal:701-702, 727) */
};

enum wm_router_kind {
  WM_ROUTER_SOFTMAX = 0,         /* Qwen: softmax, top-k, renormalised (qwen4_exp.py:1009-1047) */
  WM_ROUTER_SQRTSOFTPLUS = 1,    /* DeepSeek V4.1: sqrt(softplus), bias selects (moe.py:58-74) */
  WM_ROUTER_SIGMOID = 2,         /* MiMo: sigmoid + correction bias (mimo/model.py:139-150) */
  WM_ROUTER_SIGMOID_GROUPED = 3, /* sigmoid + bias, group-limited selection (not in the reference) */
};

enum wm_shared_gate {
  WM_SHARED_NONE = 0,          /* no shared expert */
  WM_SHARED_SIGMOID_GATE = 1,  /* Qwen: sigmoid(x . g) * shared(x) (qwen4_exp.py:1046) */
  WM_SHARED_ONE = 2,           /* DeepSeek: shared(x) added as is (moe.py:110-112) */
};

/* Sizes that bound every later call; wm_create reserves the device workspace. */
typedef struct {
  int64_t max_tokens;       /* largest T of any call */
  int32_t max_hidden;       /* largest H */
  int32_t max_inter;        /* largest I */
  int32_t max_experts;      /* largest E (routed experts) */
  int32_t max_topk;         /* largest K */
  int32_t gemv_max_tokens;  /* T up to this runs the decode kernels; -1 = never; 0 = automatic: the
                               decode kernels while the expert rows average <= 32 per expert */
  int32_t flags;            /* WM_FLAG_* bits, else 0 */
} wm_options;

/* Routes with a negative expert id are padding: they get no row and a zero
   output row (wm_expert_pairs), instead of an error.  For fixed-capacity
   exchange buffers (the expert-parallel path). */
#define WM_FLAG_SKIP_NEGATIVE_ROUTES 1

/* Short MXFP4 calls take the register-direct warp-MMA decode kernel (weights
   dequantised to exact f16 in registers) instead of the default block-scaled
   tcgen05 kernel.  The default: the E2M1 weights go from the blob to the
   tensor cores by TMA with their E8M0 scales as the MMA's scale factors
   (kind::mxf8f6f4), and each token row enters as two E4M3 parts (hi + lo,
   power-of-two scales per 32 values; within 2^-8 of every element, layer
   outputs within ~1e-3 of max|y|); it needs H and I multiples of 512,
   32-byte aligned weight regions and 16-byte aligned scale regions. */
#define WM_FLAG_MMA_DECODE 4

/* Long MXFP4 and FP8 (128 x 128 fp32 block scales) calls take the kind::f16
   tcgen05 grouped GEMM (weights dequantised by producer warps: MXFP4 to exact
   f16, FP8 to bf16(e4m3 * scale) as the reference rounds them) instead of the
   default block-scaled one.  The default: the blob's E2M1 or E4M3 weights by
   TMA into kind::mxf8f6f4 MMAs, MXFP4's E8M0 scales as the MMA's scale
   factors, FP8's fp32 block scales applied to each 128-K block's partial sum
   in registers (the weights stay exact, so FP8 results differ from the
   reference's bf16-rounded weights by up to ~1e-2 of max|y|: 5-8.5e-3 on the
   benchmark weights, against 2-4.3e-3 for the kind::f16 GEMM); token and act
   rows as hi + lo E4M3 parts (as for WM_FLAG_MMA_DECODE's default); H and I
   multiples of 512 and the block-scaled decode kernel's alignment needs. */
#define WM_FLAG_F16_GEMM 8

/* Decode calls of up to 64 tokens (T * K <= 1024, E <= 512) on the
   block-scaled decode path run the plan and the token-row quantisation -- and
   router calls of up to 4 tokens the top-k too -- as separate launches
   instead of one.  Both give the same routes, plan and output bits; the one
   launch saves one or two kernel boundaries per layer. */
#define WM_FLAG_SPLIT_SMALL_CALLS 16

/* The block-scaled decode path's gate/up and down kernels run as one
   persistent launch: a down item waits (bounded, 2 s, then an error through
   wm_sync) until the gate/up items of its 16-token tile have written the act
   rows, so the down weights stream while the last gate/up items finish.  Not
   on the expert-parallel owner path.  Off by default: not yet measured. */
#define WM_FLAG_FUSED_DECODE 32

/* One projection of every expert: expert e's matrix at weight + e * weight_stride
   bytes, its scales at scale + e * scale_stride bytes (device pointers). */
typedef struct {
  const void* weight;
  int64_t weight_stride;
  const void* scale;
  int64_t scale_stride;
} wm_matrix;

typedef struct {
  int32_t T, H, I, E, K;
  int32_t layout;                 /* enum wm_layout */
  wm_matrix w13;                  /* fused gate/up projection, [2I, H] per expert */
  wm_matrix w2;                   /* down projection, [H, I] per expert */
  wm_matrix shared_w13;           /* the shared expert (strides ignored); weight NULL = none */
  wm_matrix shared_w2;
  int32_t shared_gate;            /* enum wm_shared_gate */
  const void* shared_gate_weight; /* bf16 [H] for WM_SHARED_SIGMOID_GATE */
  const void* x;                  /* bf16 [T, H] */
  /* Routing: router weights, or (router_weight NULL) precomputed routes. */
  int32_t router;                 /* enum wm_router_kind */
  const void* router_weight;      /* bf16 [E, H] */
  const float* router_bias;       /* fp32 [E] selection bias, or NULL */
  int32_t n_groups, topk_groups;  /* WM_ROUTER_SIGMOID_GROUPED only */
  float route_scale;              /* multiplies the routing weights (1.0 for Qwen / MiMo) */
  const int32_t* routes_idx;      /* int32 [T, K] expert ids (when router_weight is NULL) */
  const float* routes_w;          /* fp32 [T, K] routing weights */
  float swiglu_limit;             /* > 0: silu(min(g, L)) * clamp(u, -L, L); else silu(g) * u */
  void* out;                      /* bf16 [T, H] combined output */
  int32_t* out_idx;               /* optional int32 [T, K]: routes used */
  float* out_w;                   /* optional fp32 [T, K] */
  /* Pre-MoE RMSNorm (optional): with norm_weight set, the block's input is
       xn[t] = bf16((x[t] * (1 / sqrt(mean_h(x[t, h]^2) + norm_eps))) * norm_weight)
     (fp32 sums of squares, bf16 output), computed once and used by the router,
     the shared-expert gate and the experts -- the post_attention_layernorm that
     the reference runs right before the gate (engine.mm:1846 with
     kernels.metal:443-465, rms_norm_tg; GroupRMSNorm, qwen4_exp.py:93-117).
     Short calls fuse it into the router kernel.  x_norm (optional, bf16
     [T, H], must not overlap x) receives xn; when NULL it stays in the
     handle's workspace.  wm_moe_forward_noalloc requires x_norm. */
  const void* norm_weight;        /* bf16 [H], or NULL: x is used as given */
  float norm_eps;                 /* >= 0, e.g. 1e-6 */
  void* x_norm;                   /* bf16 [T, H] output of xn, or NULL */
} wm_moe_args;

typedef struct {
  int64_t calls_forward, calls_pairs, calls_route, calls_dequant;
  int64_t launches;            /* kernels enqueued by this handle */
  int64_t gemv_calls, gemm_calls;
  int64_t decode_calls;        /* calls that took the decode kernels (block-scaled tcgen05 by default,
                                  WM_FLAG_MMA_DECODE selects the register-direct one) */
  int64_t bs_gemm_calls;       /* the gemm_calls that took a block-scaled grouped GEMM (the default for
                                  MXFP4 and 128 x 128 FP8; WM_FLAG_F16_GEMM selects the kind::f16 one) */
} wm_counters;

typedef struct {
  char name[32];      /* kernel group: router, plan, gather_rows, gemv_gate_up, ... */
  int64_t launches;   /* timed launches since the last reset */
  double total_ms;    /* summed CUDA-event durations */
} wm_profile_entry;

/* Creates a handle on CUDA device `device`.  NULL on failure, with a message in
   error[0 .. error_size).  Replaces wq_open's engine set-up
   (Native/QwenNative/capi.h:41) for the expert path only. */
WM_EXPORT wm_ctx* wm_create(int32_t device, const wm_options* options, char* error, size_t error_size);
WM_EXPORT void wm_destroy(wm_ctx* ctx);
/* The message of the last failed call (Native/QwenNative/capi.h:43). */
WM_EXPORT const char* wm_error(const wm_ctx* ctx);
/* Waits for `stream`; returns 1 if a kernel recorded an error since the last
   wm_sync (e.g. an expert id out of range), with the text in wm_error. */
WM_EXPORT int wm_sync(wm_ctx* ctx, void* stream);
WM_EXPORT void wm_counters_get(const wm_ctx* ctx, wm_counters* out);

/* Dequantise one matrix to bf16 [rows, cols] (device): the decode of
   deepseek_v41/dequant.py:53-68 (MXFP4), mimo/weights.py:17-43 (FP8 128x128)
   and dequant.py:45-50 (FP8 32x32 UE8M0), bit for bit. */
WM_EXPORT int wm_dequant(wm_ctx* ctx, int32_t format, const void* weight, const void* scale, int64_t rows,
                         int64_t cols, int32_t convention, void* out_bf16, void* stream);

/* Router logits and top-k: logits (optional, fp32 [T, E]), idx int32 [T, K],
   w fp32 [T, K] (SparseMoE.route/_gates, qwen4_exp.py:1009-1047; Gate,
   deepseek_v41/moe.py:58-74; Router, mimo/model.py:139-150).  Uses
   args->{T, H, E, K, x, router, router_weight, router_bias, n_groups,
   topk_groups, route_scale}. */
WM_EXPORT int wm_route(wm_ctx* ctx, const wm_moe_args* args, float* logits, int32_t* idx, float* w, void* stream);

/* Routed expert rows without the combine: routed bf16 [T, K, H] with row
   (t, k) = expert idx[t, k] applied to x[t] -- the output of
   StreamingExperts.__call__ (qwen4_exp.py:853-904) and
   _StreamingSwitchGLU.__call__ (model.py:325-501).  Uses args->routes_idx. */
WM_EXPORT int wm_expert_pairs(wm_ctx* ctx, const wm_moe_args* args, void* routed, void* stream);

/* Weighted combine of expert rows given in (token, k) order -- the step that
   closes the MoE block (_route_reduce, model.py:545-546; MoE.__call__,
   deepseek_v41/moe.py:110-112; moe_combine, QwenNative/kernels.metal:185-194):
     out[t] = sum_k w[t, k] * pairs[t * K + k] + g_t * shared[t]   (bf16 out)
   summed in fp32 in k order with the same arithmetic as wm_moe_forward's
   combine, where g_t = sigmoid(x[t] . shared_gate_weight) for
   WM_SHARED_SIGMOID_GATE, 1 for WM_SHARED_ONE, and no shared term for
   WM_SHARED_NONE.  pairs bf16 [T * K, H], w fp32 [T, K], shared bf16 [T, H];
   T <= the handle's max_tokens.  pair_pos int32 [T * K] (optional): pair
   (t, k) is row pair_pos[t * K + k] of `pairs` instead of row t * K + k.
   Used by the expert-parallel path, where the expert rows come back from
   other GPUs in send order. */
WM_EXPORT int wm_combine(wm_ctx* ctx, int64_t T, int32_t H, int32_t K, const void* pairs, const int32_t* pair_pos,
                         const float* w, const void* shared, int32_t shared_gate, const void* x,
                         const void* shared_gate_weight, void* out, void* stream);

/* Expert-parallel dispatch plan for T tokens with routes idx int32 [T, K]
   over `world` ranks that hold `experts_per_rank` consecutive experts each:
   orders the pairs by owning rank (stable: (t, k) order within a rank) and
   writes send_counts int32 [world] (pairs per rank), pair_pos int32 [T * K]
   (slot of pair (t, k)), send_eid int32 (expert id local to its owner, per
   slot) and send_x bf16 [slots, H] (x[t] per slot).  capacity 0: the slots
   are packed, T * K of them.  capacity C >= T * K: rank r's pairs take slots
   [r * C, r * C + count_r) of world * C slots, unused slots get expert id -1
   (fixed-size exchanges, no host round trip; see
   WM_FLAG_SKIP_NEGATIVE_ROUTES).  No counterpart in the reference, whose
   experts run on one device. */
WM_EXPORT int wm_ep_plan(wm_ctx* ctx, int64_t T, int32_t K, int32_t experts_per_rank, int32_t world,
                         int32_t capacity, const int32_t* idx, const void* x, int32_t H, int32_t* send_counts,
                         int32_t* pair_pos, int32_t* send_eid, void* send_x, void* stream);

/* Expert-parallel exchanges over NVLink peer memory, without a collective
   library: one process per GPU, `world` <= 8 ranks on distinct GPUs of one
   box.  wm_ep_create reserves this rank's exchange buffer (recv_x bf16
   [world * capacity, H], recv_e int32 [world * capacity], back bf16
   [world * capacity, H], flags); each rank passes wm_ep_ipc_handle's 64 bytes
   to every peer (e.g. an all-gather), which maps it with wm_ep_open_peer.
   One layer step, every rank in the same order:
     wm_ep_dispatch   routes idx int32 [T, K] (T * K <= capacity) of x bf16
                      [T, H]: each pair's row and owner-local expert id go
                      straight into its owner's recv block for this rank;
                      pair_pos int32 [T, K] receives each pair's slot
                      (owner * capacity + j) in `back`;
     wm_ep_wait(0)    until every peer's rows have arrived;
     wm_expert_pairs  on recv_x / recv_e (WM_FLAG_SKIP_NEGATIVE_ROUTES handle),
                      giving y bf16 [world * capacity, H];
     wm_ep_return     each valid row of y back to the rank that sent it;
     wm_ep_wait(1)    until every peer's rows are back; then wm_combine reads
                      `back` at pair_pos.
   Waits are bounded (2 s, then a timeout in wm_sync's status); the step
   number lives on the device, so the sequence can be captured in a CUDA
   graph.  Destroy only after every peer has finished its last step.  No
   counterpart in the reference, whose experts run on one device. */
typedef struct wm_ep wm_ep;
WM_EXPORT wm_ep* wm_ep_create(int32_t device, int32_t world, int32_t rank, int64_t capacity, int32_t H, char* error,
                              size_t error_size);
WM_EXPORT void wm_ep_destroy(wm_ep* ep);
WM_EXPORT int wm_ep_ipc_handle(wm_ep* ep, void* handle64);
WM_EXPORT int wm_ep_open_peer(wm_ep* ep, int32_t peer, const void* handle64);
/* 0: recv_x, 1: recv_e, 2: back (device pointers into this rank's buffer) */
WM_EXPORT void* wm_ep_buffer(wm_ep* ep, int32_t which);
WM_EXPORT int wm_ep_dispatch(wm_ctx* ctx, wm_ep* ep, int64_t T, int32_t K, int32_t experts_per_rank,
                             const int32_t* idx, const void* x, int32_t* pair_pos, void* stream);
WM_EXPORT int wm_ep_return(wm_ctx* ctx, wm_ep* ep, const void* y, void* stream);
WM_EXPORT int wm_ep_wait(wm_ctx* ctx, wm_ep* ep, int32_t which, void* stream);
/* The owner's half of a step, in place of wm_expert_pairs + wm_ep_return
   (call it after wm_ep_wait(0)): this rank's experts applied to the rows its
   peers dispatched to it -- only the real ones, each sender records how many
   it sent -- and every result row stored into its sender's `back` block (by
   the down kernel's epilogue itself on the grouped GEMM and the block-scaled
   decode kernel, so the return overlaps the math; from the sorted rows by a
   copy kernel otherwise), then the return flags raised (wait with
   wm_ep_wait(1)).  args gives this rank's experts (E = experts_per_rank,
   layout, H equal to the buffer's, I, w13, w2, swiglu_limit); x, routes,
   router, norm and shared fields are ignored; args->T is the number of rows
   this rank expects to receive, in [1, world * capacity], which picks the
   expert kernels as for a call of T single routes (decode kernels or grouped
   GEMM).  The handle must hold world * capacity tokens.  No counterpart in
   the reference, whose experts run on one device. */
WM_EXPORT int wm_ep_experts(wm_ctx* ctx, wm_ep* ep, const wm_moe_args* args, void* stream);

/* The whole MoE block: route, sort, experts, shared expert, combine
   (SparseMoE.__call__, qwen4_exp.py:1015-1051; _streaming_moe, model.py:526-546;
   MoE.__call__, deepseek_v41/moe.py:105-112). */
WM_EXPORT int wm_moe_forward(wm_ctx* ctx, const wm_moe_args* args, void* stream);

/* The decode MoE block (router if router_weight is set, sort, expert GEMVs,
   shared expert, combine -- the same kernels as wm_moe_forward's decode
   path) for callers that cannot allocate device memory: there is no handle,
   and all scratch lives in one static device array of 8 MiB per GPU, which
   the CUDA runtime reserves when it loads the library's module on that GPU
   and keeps until the process exits.  CUDA loads modules lazily by default,
   so that happens during the first call on a device (which also looks up the
   array's device address): make the first call, or a call of
   wm_moe_forward_noalloc_status, at start-up, before device memory is fixed
   and before any stream capture, or set CUDA_MODULE_LOADING=EAGER.  A call
   whose scratch would exceed the array (roughly: (T*K + T) * (H + I) * 2
   bytes plus routing arrays) fails with status 1 and a message in
   error[0 .. error_size).  Calls share the array: calls that overlap on the
   GPU race, so serialise them.  Expert ids of caller-given routes are checked
   on the device, not the host: a route outside [0, E) adds nothing to its
   token's output and is recorded in the array's status words, which
   wm_moe_forward_noalloc_status reports (FP8 NaN codes are not checked on
   this path; wm_moe_forward reports them).  This entry point has
   no counterpart in the reference. */
WM_EXPORT int wm_moe_forward_noalloc(const wm_moe_args* args, void* stream, char* error, size_t error_size);
/* Waits for `stream`, then reports the errors that the kernels of the last
   wm_moe_forward_noalloc call on the current device recorded: 0 when none,
   1 with the message in error[0 .. error_size) otherwise (an expert id
   outside [0, E)).  Each call clears the record when it starts.  Allocates nothing; no counterpart in the reference. */
WM_EXPORT int wm_moe_forward_noalloc_status(void* stream, char* error, size_t error_size);

/* Per-kernel-group timing with CUDA events recorded on the calls' streams
   (the counterpart of the native engines' gpu_seconds counters,
   Native/QwenNative/capi.h:28-35).  Off by default; while on, calls must not
   be captured into CUDA graphs. */
WM_EXPORT int wm_profile_enable(wm_ctx* ctx, int32_t enable);
/* Waits for the timed work, then copies up to max_entries accumulated groups;
   returns the number copied. */
WM_EXPORT int32_t wm_profile_read(wm_ctx* ctx, wm_profile_entry* out, int32_t max_entries);
WM_EXPORT void wm_profile_reset(wm_ctx* ctx);

#ifdef __cplusplus
}
#endif
#endif /* WHALLM_MOE_H */
