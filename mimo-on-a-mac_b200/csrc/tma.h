// Host-side TMA tensor-map construction (cuTensorMapEncodeTiled through the runtime's driver entry
// point, so the library does not link libcuda).  Maps are cached by their full description.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace mimo {

// Weight map of one MXFP4 projection [rows, K/2 bytes]: boxes of 16 rows x `panels` 128-byte K panels,
// 128B swizzle, landing in shared memory as [panel][row][128 B].  `per_panel` reports a 2-D map
// (one panel per copy) when the 3-D form could not be encoded.
struct WeightMap {
  alignas(64) CUtensorMap map;
  int per_panel;  // 0: one 3-D box covers all panels; 1: one 2-D box per panel
};

// Returns cudaSuccess or an error (cudaErrorInvalidValue when encoding fails).
cudaError_t weight_map(WeightMap* out, const void* base, uint64_t rows, uint64_t row_bytes, int panels);
// Scale map [rows, K/32 bytes]: boxes of 16 rows x box_bytes, no swizzle.
cudaError_t scale_map(CUtensorMap* out, const void* base, uint64_t rows, uint64_t row_bytes, int box_bytes);

}  // namespace mimo
