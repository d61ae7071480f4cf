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
// the current device's SM count (after its opt-in)
int gemm_sms();
// the kernels' shared-memory opt-in on the current device (before any graph capture)
int prepare_gemm();
size_t gemm_smem_bytes();

}  // namespace b200
