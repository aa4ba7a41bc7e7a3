// Kernel launchers of the MoE expert-FFN library (host-callable, stream-ordered).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

#include "../../include/whallm_moe.h"
#include "wm_device.cuh"
#include "wm_types.h"

namespace wm {

constexpr int kMaxDevices = 64;  // per-device state of the attribute setters

// ---- optional per-kernel timing with CUDA events (wm_profile_*)
enum ProfSlot : int {
  kProfRouter = 0,
  kProfTopk,
  kProfPlan,
  kProfActF16,
  kProfGather,
  kProfGemvGateUp,
  kProfGemvDown,
  kProfGemmGateUp,
  kProfGemmDown,
  kProfCombine,
  kProfDecodeGateUp,
  kProfDecodeDown,
  kProfNorm,
  kProfEpSend,          // expert-parallel dispatch: owner plan + peer stores of the rows
  kProfEpWaitDispatch,  // waiting for every peer's rows
  kProfEpReturn,        // result rows back to their senders
  kProfEpWaitReturn,    // waiting for every peer's result rows
  kProfRoutePlanQuant,  // small router calls: top-k, plan and token images in one launch
  kProfDecodeFused,     // block-scaled decode: gate/up and down in one launch (WM_FLAG_FUSED_DECODE)
  kProfSlots
};
struct Profiler;  // defined in wm_profile.cu
void prof_begin(Profiler* p, int slot, cudaStream_t s);
void prof_end(Profiler* p, int slot, cudaStream_t s);

// ---- dequant probe (wm_dequant.cu)
void launch_dequant(int format, const void* weight, const void* scale, int64_t rows, int64_t cols, int convention,
                    uint16_t* out, uint32_t* status, cudaStream_t stream);

// ---- router (wm_route.cu)
size_t router_smem_bytes(int H);
void router_init_attributes(int max_hidden);
// Top-k selection: parameters and outputs idx int32 / w fp32 [T, K].
struct TopkArgs {
  const float* bias;  // fp32 [E] or null
  int K, kind, n_groups, topk_groups;
  float route_scale;
  int32_t* idx;
  float* w;
};


// With nw (bf16 [H] RMSNorm weight) a call that router_logits_fused_ok takes
// routes bf16((x * rstd) * nw) and writes those rows to xn (when non-null);
// other calls ignore nw -- normalise first with launch_rmsnorm.
void launch_router_logits(const uint16_t* x, const uint16_t* wr, const uint16_t* sg_w, int T, int H, int E,
                          float* logits, float* sg, cudaStream_t stream, const uint16_t* nw = nullptr,
                          float eps = 0.0f, uint16_t* xn = nullptr);
bool router_logits_fused_ok(int T, int H, int E);
// xn[t] = bf16((x[t] * rsqrt(mean(x[t]^2) + eps)) * nw), H % 8 == 0
void launch_rmsnorm(const uint16_t* x, const uint16_t* nw, int T, int H, float eps, uint16_t* xn,
                    cudaStream_t stream);
void launch_shared_gate(const uint16_t* x, const uint16_t* g, int T, int H, float* sg, cudaStream_t stream);
void launch_router_topk(const float* logits, int T, int E, const TopkArgs& tk, cudaStream_t stream);
// Calls of up to kTopkGroupCalls tokens select with a block of warps per token
// (K <= 32, E <= 1024, every router kind but the group-limited one); measured
// slower than a warp per token from 8 tokens up (config 1: 10.6 against 9.3 us
// at 8 tokens, 10.5 against 9.6 us at 64).
constexpr int kTopkGroupCalls = 4;
bool router_topk_group_ok(int T, int K, int E, int kind);

// ---- router logits on tcgen05 for long calls (wm_router_sm100.cu); tm_x / tm_w
// point to CUtensorMaps of x [T, H] and W_r [E, H] (bf16, 64 x 128 boxes, 128B swizzle)
bool router_gemm_shape_ok(int T, int H, int E);
void router_gemm_init_attributes();
void launch_router_gemm(const void* tm_x, const void* tm_w, int T, int H, int E, float* logits, uint32_t* status,
                        int num_sms, cudaStream_t stream);

// ---- sort / permute / combine (wm_plan.cu)
void launch_plan(const int32_t* idx, int T, int K, int E, bool has_shared, int align, const Plan& p, int max_rows,
                 int max_mtiles, int max_chunks, uint32_t* status, cudaStream_t stream, int* launches);
void launch_gather_rows(const uint16_t* x, const Plan& p, int E, int H, uint16_t* xs, int num_sms,
                        cudaStream_t stream);
void launch_combine(const uint16_t* routed, const Plan& p, const float* w, const float* sg, int shared_kind, int T,
                    int H, int E, int K, uint16_t* out, cudaStream_t stream);
// The same sum over pairs at rows pair_pos[t * K + k] (t * K + k when null)
// and shared rows [T, H].
void launch_combine_dense(const uint16_t* pairs, const int32_t* pair_pos, const float* w, const float* sg,
                          int shared_kind, int T, int H, int K, const uint16_t* shared_rows, uint16_t* out,
                          cudaStream_t stream);
// Expert-parallel dispatch plan: owners of the pairs, then (after a plan over
// owners) slots, owner-local expert ids and per-owner counts.
void launch_ep_owner(const int32_t* idx, int P, int per_rank, int world, int32_t* owner, uint32_t* status,
                     int num_sms, cudaStream_t stream);
void launch_ep_finish(const int32_t* idx, const Plan& p, int T, int K, int per_rank, int world, int capacity,
                      int32_t* send_counts, int32_t* pair_pos, int32_t* send_eid, const uint16_t* x, int H,
                      uint16_t* send_x, int num_sms, cudaStream_t stream);
// ---- expert-parallel exchanges over peer memory (wm_ep_p2p.cu)
constexpr int kMaxEpRanks = 8;
// The blocks this rank writes in every rank's exchange buffer (peer r's
// address space mapped here), and this rank's own step state.
// Down-projection rows of an expert-parallel owner stored straight into the
// senders' `back` blocks: sorted row r holds slot s = plan.row_token[r] (s <
// 0: padding), which goes to rows[s / capacity] + (s % capacity) * H.
struct EpReturn {
  uint16_t* rows[kMaxEpRanks];  // every rank's back block for this rank; rows[0] == nullptr: off
  int capacity;
};

struct EpPeers {
  uint16_t* rows[kMaxEpRanks];  // rank r's recv_x (dispatch) or back (return) block for this rank
  int32_t* ids[kMaxEpRanks];    // rank r's recv_e block for this rank (dispatch)
  uint32_t* flag[kMaxEpRanks];  // rank r's flag for this rank
  int32_t* count[kMaxEpRanks];  // rank r's count of the pairs this rank sent it (dispatch)
  uint32_t* ticket;             // local: CTAs done with this exchange
  const uint32_t* epoch;        // local: step number
};
void launch_ep_begin(uint32_t* epoch, cudaStream_t stream);
void launch_ep_send(const int32_t* idx, const Plan& p, int T, int K, int per_rank, int world, int capacity,
                    int32_t* pair_pos, const uint16_t* x, int H, const EpPeers& pe, int num_sms, cudaStream_t stream);
// The whole dispatch of a small call in one launch (step number, owners,
// slots, ids, rows, flags): P = T * K pairs within ep_dispatch_small_ok.
bool ep_dispatch_small_ok(int P, int world, int capacity);
void launch_ep_dispatch_small(const int32_t* idx, int T, int K, int per_rank, int world, int capacity,
                              int32_t* pair_pos, const uint16_t* x, int H, const EpPeers& pe, uint32_t* epoch,
                              uint32_t* status, int num_sms, cudaStream_t stream);
void launch_ep_return(const uint16_t* y, const int32_t* recv_e, int world, int capacity, int H, const EpPeers& pe,
                      int num_sms, cudaStream_t stream);
void launch_ep_wait(const uint32_t* flags, int world, const uint32_t* epoch, uint32_t* status, int code,
                    cudaStream_t stream);
// The owner's plan over its recv blocks: block r holds counts[r] real pairs
// (ids[r * capacity + j], j < counts[r], local expert ids); slots past a
// block's count are never read.  row_token[row] = slot, pair_pos[slot] = row.
void launch_plan_blocks(const int32_t* ids, const int32_t* counts, int world, int capacity, int E, int align,
                        const Plan& p, int max_rows, int max_mtiles, int max_chunks, uint32_t* status,
                        cudaStream_t stream, int* launches);
// Result rows straight from the owner's sorted rows (routed[pair_pos[slot]])
// into each sender's back block, then the return flags.
// After a down kernel that stored the rows itself: raise this rank's return
// flag on every peer (system-scope fence first).
void launch_ep_signal(const EpPeers& pe, int world, cudaStream_t stream);
void launch_ep_return_sorted(const uint16_t* routed, const int32_t* pair_pos, const int32_t* counts, int world,
                             int capacity, int H, const EpPeers& pe, int num_sms, cudaStream_t stream);
void launch_unpermute(const uint16_t* routed, const Plan& p, int TK, int H, uint16_t* out, int num_sms,
                      cudaStream_t stream);

// ---- decode GEMV (wm_gemv.cu)
struct GemvArgs {
  Plan plan;
  ExpertWeights wts;
  const uint16_t* x;  // [T, H] bf16 (rows gathered through plan.row_token)
  uint16_t* act;      // [rows, I] bf16, sorted rows
  uint16_t* routed;   // [rows, H] bf16, sorted rows
  int H, I;
  int gate_first;     // 1: gate rows [0, I), up rows [I, 2I); 0: the reverse
  float limit;        // SwiGLU clamp (<= 0: none)
};
void gemv_init_attributes(int max_smem);
size_t gemv_smem_bytes(int H, int I);
void launch_gemv(const GemvArgs& a, int fmt, int max_unique, cudaStream_t stream, Profiler* prof);

// ---- decode kernel arguments (register-direct warp MMAs, wm_decode_mma.cu)
struct DecodeArgs {
  Plan plan;            // 16-row tiles, no padding, rowmax set
  ExpertWeights wts;
  const float* bscale;  // [rows] power-of-two prescale of the f16 activation rows
  uint16_t* act;        // [rows, I] bf16 (gate/up output)
  uint16_t* routed;     // [rows, H] bf16 (down output)
  int H, I;
  int gate_first;
  float limit;
  uint32_t* status;
  int nbuf;             // decode_mma_kernel: token-tile buffers, 1 or 2 (decode_mma_buffers)
};
// f16 sorted activation rows with their per-row prescale (x rows for gate/up,
// act rows for down).
void launch_gather_f16(const uint16_t* x, const Plan& p, int E, int H, uint16_t* out, float* scale, int num_sms,
                       cudaStream_t stream);
void launch_act_f16(const uint16_t* act, const Plan& p, int E, int I, uint16_t* out, float* scale, int num_sms,
                    cudaStream_t stream);


// ---- decode, register-direct warp MMAs (wm_decode_mma.cu): plan tiles of 8
// rows; tmap_x points to a CUtensorMap of the f16 activation rows [max_rows, K]
// (boxes of 64 x 8, 128-byte swizzle), K = H for kind 0 (gate/up) and I for kind 1.
// fmt: kFmtMxfp4 (f16 token rows from gather_f16 / act_f16, bscale set) or an
// FP8 format (bf16 token rows from gather_rows / the bf16 act, bscale unused).
bool decode_mma_shape_ok(int H, int I, int fmt = kFmtMxfp4);
void decode_mma_init_attributes(int max_h, int max_i);
// ks: K split (1, 2, 4, 8; see decode_mma_split) -- items of 1 / ks of the
// rows, each warp over 1 / ks of K
void launch_decode_mma(const DecodeArgs& a, int kind, const void* tmap_x, int num_sms, cudaStream_t stream,
                       int ks = 1, int fmt = kFmtMxfp4);
// The K split for a call of about `tiles` 8-token tiles: the smallest that
// spreads the items over the SMs (within the segments of K).
int decode_mma_split(int kind, int H, int I, int tiles, int num_sms, int fmt = kFmtMxfp4);
// Token-tile buffers (1 or 2) for a launch with split ks over about `tiles` tiles.
int decode_mma_buffers(int kind, int H, int I, int ks, int tiles, int num_sms, int fmt = kFmtMxfp4);

// ---- decode on tcgen05 block-scaled MMA (wm_bs_sm100.cu): E2M1 weights by TMA,
// E8M0 scales as UE8M0 scale factors, token rows as hi / lo E4M3 parts.
struct BsArgs {
  Plan plan;             // 16-row tiles, groups padded to 16 rows
  ExpertWeights wts;
  int H, I;
  int gate_first;
  float limit;
  uint32_t* status;
  const uint8_t* img;    // token tile images [tiles][K / 128][4608]: hi rows 0..15, lo rows 16..31, scale atom
  uint8_t* act_img;      // gate/up: act tile images for the down kernel (K = I)
  uint16_t* routed;      // down: [rows, H] bf16
  EpReturn ret;          // down: with ret.rows[0] set, rows go to the senders instead of `routed`
  int stages;
  uint32_t* tile_done;   // fused launch: per-tile counts of act-image writers, then a finish count
  int max_tiles;         // ... at tile_done[max_tiles]
};
void bs_init_attributes();
// H and I multiples of 512 (four 128-K stages per raw scale load)
bool bs_shape_ok(int H, int I);
// x rows (through the plan, 16-row tiles) -> hi / lo E4M3 tile images and scale atoms
void launch_bs_quant_rows(const uint16_t* x, const Plan& p, int E, int K, uint8_t* img, int num_sms,
                          cudaStream_t stream);
// Calls of up to 64 tokens on the block-scaled decode path: the plan (groups
// padded to 16 rows) and the token images in one launch of T blocks, the same
// plan and images as launch_plan + launch_bs_quant_rows (T <= 64, T * K <=
// 1024, E <= 512).  Router calls of up to kSmallCallTokens tokens also select
// the top-k in that launch (launch_bs_route_plan_quant: the routes of
// launch_router_topk as well).
constexpr int kSmallCallTokens = 4;  // top-k inside too: batch 1 41.5 against 49.4 us; batch 8 slower (75.2 / 74.1)
constexpr int kSmallCallThreads = 512;
bool bs_plan_quant_ok(int T, int K, int E);
bool bs_route_plan_quant_ok(int T, int K, int E, int kind);
void launch_bs_plan_quant(const int32_t* routes, int T, int K, int E, bool has_shared, const Plan& p, int max_rows,
                          int max_mtiles, uint32_t* status, const uint16_t* x, int H, uint8_t* img,
                          cudaStream_t stream);
void launch_bs_route_plan_quant(const float* logits, int T, int E, const TopkArgs& tk, bool has_shared, const Plan& p,
                                int max_rows, int max_mtiles, uint32_t* status, const uint16_t* x, int H,
                                uint8_t* img, cudaStream_t stream);
// maps[0..3]: CUtensorMaps of the routed and the shared expert's packed weights
// (16U4_ALIGN16B, 128-byte swizzle; gate/up 4-D [E][2][I][H] with boxes
// 128 x 64 x 2, down 3-D [E][H][I] with boxes 128 x 128) and of their E8M0
// rows (uint8, gate/up [E][2][I][H/32] boxes 16 x 64 x 2, down [E][H][I/32] boxes 16 x 128).
void launch_bs_decode(const BsArgs& a, int kind, const void* const* maps, int num_sms, cudaStream_t stream);
// Both expert kernels in one persistent launch (down items wait, bounded, for
// their tile's gate/up items): maps[0..3] as launch_bs_decode's gate/up maps,
// maps[4..7] its down maps; a.tile_done zero on entry (left zero on exit).
void launch_bs_decode_fused(const BsArgs& a, const void* const* maps, int num_sms, cudaStream_t stream);

// ---- prefill grouped GEMM on tcgen05 block-scaled MMA (wm_bsgemm_sm100.cu):
// 128 token rows (hi / lo E4M3) x 256 weight rows per tile.  The same BsArgs
// (plan with 128-row tiles; act_img holds 33,792-byte images per 128-row
// tile and 128-K stage, bsg_image_bytes) and weight maps as launch_bs_decode;
// shapes as bs_shape_ok.
void bsg_init_attributes();
size_t bsg_image_bytes(int64_t mtiles, int K);
// x rows [0, rows) (with counts: expert-parallel slots, block r = row / capacity
// holding counts[r]) -> hi / lo E4M3 parts and UE8M0 scales at every sorted
// row that holds them (pair_pos[t * topk + k], and offsets[E] + t with
// has_shared): hi, lo [sorted rows][K], shi, slo [sorted rows][K / 32]
void launch_bsg_quant_scatter(const uint16_t* x, int rows, int K, const Plan& p, int topk, bool has_shared, int E,
                              const int32_t* counts, int capacity, uint8_t* hi, uint8_t* lo, uint8_t* shi,
                              uint8_t* slo, int num_sms, cudaStream_t stream);
// ---- prefill grouped GEMM for FP8 experts with fp32 128 x 128 block scales
// (wm_fp8gemm_sm100.cu): E4M3 weights by TMA into block-scaled tcgen05 MMAs
// (weight scale factors 2^0), each 128-K block's fp32 partial scaled by its
// weight block scale in registers; tokens as for launch_bsg.  maps: gate/up
// {w13, shared w13, hi, lo, hi scales, lo scales} (w13: uint8 4-D [E][2][I][H],
// boxes 128 x 64 x 2, 128-byte swizzle), down {w2, shared w2} (uint8 3-D
// [E][H][I], boxes 128 x 128).
void fp8g_init_attributes();
bool fp8g_shape_ok(int H, int I);
void launch_fp8g(const BsArgs& a, int kind, const void* const* maps, int num_sms, cudaStream_t stream);

// maps[0..3] as launch_bs_decode; gate/up (kind 0) also maps[4..7]: the
// sorted rows' hi and lo parts (uint8 [rows][H], boxes 128 x 128, 128-byte
// swizzle) and their scale rows (uint8 [rows][H / 32], boxes 16 x 128)
void launch_bsg(const BsArgs& a, int kind, const void* const* maps, int num_sms, cudaStream_t stream);

// ---- prefill grouped GEMM on tcgen05 (wm_gemm_sm100.cu)
struct GemmArgs {
  Plan plan;
  ExpertWeights wts;
  uint16_t* out;        // gate/up: act [rows, I]; down: routed [rows, H]
  int Kdim;             // H (gate/up) or I (down)
  int N;                // 2I (gate/up) or H (down)
  int I;
  int gate_first;
  float limit;
  int fmt;
  uint32_t* status;
  const float* ascale;  // MXFP4: [rows] 2^k prescale of the f16 A rows
  uint32_t* rowmax;     // MXFP4 gate/up: [rows] per-row |act| maxima (float bits), or null
  int w32;              // 1: every expert's weight rows start 32-byte aligned (256-bit loads)
  EpReturn ret;         // down: with ret.rows[0] set, rows go to the senders instead of `out`
};
// `kind`: 0 = gate/up + SwiGLU, 1 = down.  MXFP4 takes f16 A rows (gather_f16 /
// act_f16), FP8 bf16 rows (gather_rows / the bf16 act).  tmap_a points to a CUtensorMap
// passed by value to the kernel.
void gemm_init_attributes();
bool gemm_shape_ok(int H, int I);
void launch_gemm(const GemmArgs& a, int kind, const void* tmap_host, int num_sms, cudaStream_t stream);

}  // namespace wm
