// Host-side TMA tensor-map encoding shared by the kernels (driver entry point resolved at runtime,
// so the library does not link libcuda), with a process-wide cache keyed by (address, shape, box).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace cob {

// Row-major 2-D 16-bit matrix [rows, cols] (row stride `row_bytes`), box = box_cols x box_rows,
// 128-byte swizzle (box_cols * 2 must be 128). Returns cudaSuccess or an error code.
cudaError_t tensor_map_2d(const void* ptr, uint64_t rows, uint64_t cols, uint64_t row_bytes, uint32_t box_rows,
                          uint32_t box_cols, bool bf16, CUtensorMap* out);

}  // namespace cob
