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

// MXFP4 weight map for the block-scaled tensor cores: [rows][K] e2m1 values (K / 2 bytes a row),
// 16U4_ALIGN16B (each 16 values land as 8 data bytes + 8 gap bytes), box [128 values, 128 rows],
// 128B swizzle.  K must be a multiple of 128 and the rows 32-byte aligned.
cudaError_t fp4_weight_map(CUtensorMap* out, const void* base, uint64_t rows, uint64_t K);
// 3-D view of the same weights: dims [128 values, rows, K / 128 chunks] (chunk stride 64 B), box
// [128, 128, chunks], 128B swizzle: lands as `chunks` consecutive 16 KiB tiles [row][128 B].
cudaError_t fp4_weight_map3(CUtensorMap* out, const void* base, uint64_t rows, uint64_t K, int chunks);
// 3-D view of a byte matrix [rows][row_bytes]: dims [128, rows, row_bytes / 128], box
// [128, box_rows, chunks], 128B swizzle: lands as `chunks` consecutive [box_rows][128 B] tiles.
cudaError_t rows_map3(CUtensorMap* out, const void* base, uint64_t rows, uint64_t row_bytes, int box_rows,
                      int chunks);
// Scale-matrix map [rows][row_bytes], box [16 bytes, box_rows], no swizzle.
cudaError_t sf_map(CUtensorMap* out, const void* base, uint64_t rows, uint64_t row_bytes, int box_rows);
// bf16 matrix map [rows][cols], box [64 values, box_rows], 128B swizzle; rows past the end read 0.
cudaError_t bf16_rows_map(CUtensorMap* out, const void* base, uint64_t rows, uint64_t cols, int box_rows);
// 3-D bf16 tensor [d2][d1][d0] (d0 contiguous), box [64 values, b1, b2], 128B swizzle: lands as b1 * b2
// consecutive 128-byte rows (d1 fastest); coordinates past an extent read 0.
cudaError_t bf16_map3(CUtensorMap* out, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, int b1, int b2);
// Byte-matrix map [rows][row_bytes], box [128 bytes, box_rows], 128B swizzle.
cudaError_t rows_map(CUtensorMap* out, const void* base, uint64_t rows, uint64_t row_bytes, int box_rows);
// Packed rows (e2m1, two values per byte: pool weights [rows][K/2] or activation terms) read 64 bytes
// (128 values) of box_rows rows per box, 64B swizzle (the layout kind::mxf4 reads).
cudaError_t packed64_map(CUtensorMap* out, const void* base, uint64_t rows, uint64_t row_bytes, int box_rows);

}  // namespace mimo
