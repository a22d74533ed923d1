// Internal interface of the tcgen05 GEMM (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>

#define EESD_EPI_ARGMAX_INTERNAL 3   // head: logits rounded to bf16 -> per-token argmax keys
#define EESD_EPI_ARGMAX2_INTERNAL 4  // the same, two 128-row tiles per CTA (two accumulators)

namespace eesd {

typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct TcPlan {
  int tok_tiles, out_tiles, bn, b_boxes, mma_n, kb_total, kb_per, splits, stages, acc_cols, tmem_cols;
  int pair;               // 1: CTA pairs (cta_group::2), grid (2, tok_tiles, out_tiles / 2)
  int argmax2;            // head: two row tiles per CTA, grid (tok_tiles, ceil(out_tiles / 2), 1)
  size_t smem;
  size_t partial_bytes;   // split-K scratch the launch needs (0 without split)
};

// Global scratch of a split-K launch: fp32 partial tiles (16-byte aligned).
struct TcScratch {
  void* partials = nullptr;
  size_t partial_bytes = 0;
};

PFN_encodeTiled_t tensor_map_encoder();
// 2-D K-major bf16 map [rows, k] with a (64 x box_rows) box and 128-byte swizzle
int encode_kmajor_map(CUtensorMap* map, const void* base, int rows, int k, int box_rows);
TcPlan tc_plan(int n_tok, int n_out, int k, int epi);
void tc_set_mma_n(int n);
void tc_set_splits(int n);
void tc_set_stages(int n);
void tc_set_pair(int n);
void tc_set_head_two_tiles(int n);
void tc_set_split_n(int n);
// a_packed = 1: map_w is a tile-packed weight map (encode_packed_map), else a row-major 2-D map
int tc_gemm_launch(int epi, const CUtensorMap& map_w, const void* x, int n_tok, int n_out, int k, int up_offset,
                   const void* residual, int ld_res, void* y, int ld_y, unsigned long long* keys, int* status,
                   cudaStream_t stream, int a_packed, const TcScratch& scratch);
// split-K scratch that covers every launch of this weight shape with 1..max_tok tokens
size_t tc_partial_bytes_max(int max_tok, int n_out, int k, int epi);
// Tile-packed weight layout: [ceil(rows/128) * (k/64) tiles][128 rows][64 cols], tile = row tile *
// (k/64) + k-block, so every 128 x 64 operand tile is one contiguous 16 KB block (rows past the
// end zero).  3-D map: {64, 128, tiles} with one tile per box and 128-byte swizzle.
size_t packed_weight_bytes(int rows, int k);
int pack_weight(const void* w, int rows, int k, void* out, cudaStream_t s);
int encode_packed_map(CUtensorMap* map, const void* base, int rows, int k);

}  // namespace eesd
