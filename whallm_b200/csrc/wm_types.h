// Internal types shared by the host orchestrator (wm_capi.cu) and the kernels.
#pragma once

#include <cstdint>

namespace wm {

// Weight formats the expert kernels decode.
enum Fmt : int { kFmtMxfp4 = 0, kFmtFp8B128 = 1, kFmtFp8B32 = 2 };

// Sorted-row plan of one call.  The (token, k) pairs are grouped by expert in
// a stable order (ascending token, then k), each expert's group starting at
// offsets[e]; expert index E is the shared expert, whose rows are the tokens
// in order.  With alignment 128 every group starts on a 128-row boundary and
// the padding rows carry token -1.
struct Plan {
  int32_t* counts;     // [E + 1] rows of each expert
  int32_t* offsets;    // [E + 2] first sorted row of each expert; offsets[E + 1] = rows used
  int32_t* pair_pos;   // [T * K] sorted row of pair (t, k)
  int32_t* row_token;  // [max_rows] token of each sorted row (-1 = padding)
  int32_t* unique;     // [E + 1] experts with rows, ascending (shared last)
  int32_t* n_unique;   // [1]
  int32_t* mtiles;     // [2 * max_mtiles] (expert, first row) of each 128-row tile
  int32_t* n_mtiles;   // [1]
  int32_t* hist;       // [chunks * (E + 1)] per-chunk counts (large-T sort)
  uint32_t* rowmax;    // [max_rows] or null: zeroed by the plan (decode activation maxima)
  int32_t skip_negative;  // 1: routes < 0 are padding (no row, no error), else an error
  int32_t tile_rows;      // rows per tile of unpadded groups (0: 16)
};

// Where the weights of every expert live (expert E = the shared expert).
struct ExpertWeights {
  const uint8_t* w13;
  int64_t w13_stride;
  const uint8_t* s13;
  int64_t s13_stride;
  const uint8_t* w2;
  int64_t w2_stride;
  const uint8_t* s2;
  int64_t s2_stride;
  const uint8_t* sh_w13;
  const uint8_t* sh_s13;
  const uint8_t* sh_w2;
  const uint8_t* sh_s2;
  int32_t E;

  __host__ __device__ const uint8_t* w13_of(int e) const { return e < E ? w13 + e * w13_stride : sh_w13; }
  __host__ __device__ const uint8_t* s13_of(int e) const { return e < E ? s13 + e * s13_stride : sh_s13; }
  __host__ __device__ const uint8_t* w2_of(int e) const { return e < E ? w2 + e * w2_stride : sh_w2; }
  __host__ __device__ const uint8_t* s2_of(int e) const { return e < E ? s2 + e * s2_stride : sh_s2; }
};

constexpr int kTileM = 128;  // rows per GEMM tile (and plan alignment for the GEMM path)

}  // namespace wm
