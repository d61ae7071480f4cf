// gemm_tc.h — the tensor-core int8 matmul (gemm_tc.cu) for count >= 16 tokens.
#pragma once

#include <cuda.h>
#include <cstdint>
#include <cuda_runtime.h>

namespace b200 {

struct GemmArgs {
  const float *ws;   // weight scales of the whole 2-D weight view: [rows_total][n/32]
  const float *xs;   // activation scales: token t's at xs + t * s_stride
  float *out;        // token t's row r at out[t * out_stride + r] (rows of this matrix, from 0)
  int *error;        // device word: 0, or the code of a wait that gave up
  int n, rows, count;
  int w_row0;        // this matrix's first row in the weight view (a layer's offset)
  int64_t s_stride, out_stride;
  int accumulate;    // out += result
};

// a 2-D TMA map over int8 rows: cols bytes of rows rows, row_bytes apart; boxes of 128 bytes x box_rows rows,
// 128-byte swizzle (the layout the tcgen05 descriptors of gemm_tc.cu read)
int make_i8_map(CUtensorMap *map, const void *base, int64_t cols, int64_t rows, int64_t row_bytes, int box_rows);
// wmap: the weights (box rows 128); xmap: the activations, already less the bias of 64 (box rows bn: 16 or 32)
int launch_gemm_tc(const CUtensorMap &wmap, const CUtensorMap &xmap, const GemmArgs &args, int bn,
                   cudaStream_t stream);
// the kernels' shared-memory opt-in on the current device (before any graph capture)
int prepare_gemm();
size_t gemm_smem_bytes();

}  // namespace b200
