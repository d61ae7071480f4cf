// gemm_tc.h — the tensor-core int8 matmul (gemm_tc.cu) for prompt blocks and batched tokens.
#pragma once

#include <cuda.h>
#include <cstdint>
#include <cuda_runtime.h>

namespace b200 {

struct GemmArgs {
  float *out;        // token t's row r at out[t * out_stride + r] (rows of this matrix, from 0)
  int *error;        // device word: 0, or the code of a wait that gave up
  int n, rows, count;
  int w_row0;        // this matrix's first row in the weight view (a layer's offset)
  int64_t out_stride;
  int accumulate;    // out += result
};

// the four TMA maps of one matmul
struct GemmMaps {
  CUtensorMap w;   // int8 weights [rows_total][n]: boxes of 128 bytes x 128 rows (make_i8_map)
  CUtensorMap x;   // int8 activations less the bias [tokens][..]: boxes of 128 bytes x bn tokens
  CUtensorMap ws;  // float32 weight scales [rows_total][stride], stride a multiple of 4: boxes of 4 x 128
  CUtensorMap xs;  // float32 activation scales [groups][stride >= tokens], one row per group: boxes of bn x 4
};

// a 2-D TMA map: cols elements of esize bytes per row, rows rows row_bytes apart, boxes of box_cols x box_rows
int make_map(CUtensorMap *map, CUtensorMapDataType type, int esize, const void *base, int64_t cols, int64_t rows,
             int64_t row_bytes, int box_cols, int box_rows, CUtensorMapSwizzle swizzle);
// int8 rows: cols bytes of rows rows, row_bytes apart; boxes of 128 bytes x box_rows rows, 128-byte swizzle (the
// layout the tcgen05 descriptors of gemm_tc.cu read)
int make_i8_map(CUtensorMap *map, const void *base, int64_t cols, int64_t rows, int64_t row_bytes, int box_rows);
// float32 scale rows: groups of rows rows, row_floats apart (a multiple of 4); boxes of 4 groups x box_rows
int make_scale_map(CUtensorMap *map, const float *base, int64_t groups, int64_t rows, int64_t row_floats,
                   int box_rows);
// float32 activation scales one row per group: tokens of groups rows, row_floats apart (a multiple of 4); boxes of
// box_tokens tokens x 4 groups
int make_token_scale_map(CUtensorMap *map, const float *base, int64_t tokens, int64_t groups, int64_t row_floats,
                         int box_tokens);
// bn: tokens of a tile, 16, 32 or 64 (the token map's box); a persistent grid of at most one block per SM
int launch_gemm_tc(const GemmMaps &maps, const GemmArgs &args, int bn, cudaStream_t stream);
// the tile width (16, 32 or 64, at most `widest`) that spreads rows x count best over `sms` SMs
int choose_gemm_bn(int rows, int count, int sms, int widest);
// the estimated time of q8_gemm_tc with tiles of bn tokens, in hundredths of a microsecond (measured stage times)
int64_t gemm_tc_cost(int rows, int count, int n, int sms, int bn);
// the current device's SM count (after its opt-in)
int gemm_sms();
// the kernels' shared-memory opt-in on the current device (before any graph capture)
int prepare_gemm();
size_t gemm_smem_bytes();

// ---- the lane-split matmul (gemm_lanes.cu): a cluster of four CTAs per tile, one per chain lane; for n a multiple
// of 128 with at least 16 quads (four stages a tile). Its maps (GemmMaps, other geometry):
// weights [rows][n] int8 and their scales [rows][sstride] (sstride a multiple of 4)
int make_lane_weight_maps(CUtensorMap *wmap, CUtensorMap *smap, const void *w, const float *s, int64_t n,
                          int64_t rows, int64_t sstride);
// activations [tokens][row_bytes] (k bytes used) and their scales [k / 32][tp] (one row per group), for tiles of bn
int make_lane_token_maps(CUtensorMap *xmap, CUtensorMap *xsmap, const int8_t *xq, const float *xs, int64_t tokens,
                         int64_t row_bytes, int64_t k, int64_t tp, int bn);
bool gemm_lanes_fits(int n, int rows, int count);
// whether the lane split is estimated faster than q8_gemm_tc (at its best width up to `widest`) for rows x n by count
// tokens on `sms` SMs (few row tiles)
bool gemm_lanes_pays(int rows, int count, int n, int sms, int widest);
// the tile width for count tokens: one tile up to 64 tokens, else tiles of 64; at most `widest` (16, 32 or 64: the
// token maps' boxes must fit their tensors)
int choose_lanes_bn(int count, int widest);
// false when B200FWD_GEMM_LANES=0 (a measurement knob: the one-CTA kernel for every shape)
bool gemm_lanes_enabled();
int prepare_gemm_lanes();
int launch_gemm_lanes(const GemmMaps &maps, const GemmArgs &args, int bn, cudaStream_t stream);

}  // namespace b200
