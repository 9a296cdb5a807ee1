// tensormap.h — TMA tensor maps for row-major weight matrices.
//
// A weight matrix W[rows, K] (row-major, FP32 or bf16) is described to the
// TMA engine as a 2-D tensor {K, rows} with boxes of {256 columns, box_rows
// rows}: one cp.async.bulk.tensor.2d moves 4-8 KB, large enough that the
// per-instruction cost of the copy engine does not limit HBM bandwidth
// (2 KB copies cap a single issuing thread near 2.8 TB/s on B200).  Rows
// past the end of the matrix read as zeros.
// The encoder is taken from the driver through cudaGetDriverEntryPoint, so
// the library does not link libcuda directly.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

namespace infernt {

constexpr int kBoxCols = 256;  // inner box extent (elements)

// Encodes the map for W (16-byte aligned, K * elem_bytes a multiple of 16,
// box_rows <= 256).  Returns cudaSuccess or the error of the entry-point
// lookup / encode call.
cudaError_t encode_weight_map(CUtensorMap* map, const void* W, int rows, int K, int elem_bytes, int box_rows);

}  // namespace infernt
