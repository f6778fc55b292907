// Host-side TMA tensor maps for the expert pools (see tma.h).
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <unordered_map>

#include "tma.h"

namespace mimo {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

struct Key {
  uint64_t base, rows, row_bytes;
  int kind, arg;
  bool operator==(const Key& o) const {
    return base == o.base && rows == o.rows && row_bytes == o.row_bytes && kind == o.kind && arg == o.arg;
  }
};
struct KeyHash {
  size_t operator()(const Key& k) const {
    uint64_t h = k.base * 0x9E3779B97F4A7C15ull ^ (k.rows << 17) ^ (k.row_bytes << 3) ^ (uint64_t)k.kind ^
                 ((uint64_t)k.arg << 40);
    return (size_t)(h ^ (h >> 29));
  }
};

std::mutex g_mu;
std::unordered_map<Key, WeightMap, KeyHash>& cache() {
  static std::unordered_map<Key, WeightMap, KeyHash> c;
  return c;
}

}  // namespace

cudaError_t weight_map(WeightMap* out, const void* base, uint64_t rows, uint64_t row_bytes, int panels) {
  const Key key{(uint64_t)base, rows, row_bytes, 0, panels};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = cache().find(key);
    if (it != cache().end()) {
      *out = it->second;
      return cudaSuccess;
    }
  }
  auto fn = encode_fn();
  if (!fn || row_bytes % 128 != 0 || panels < 1 || panels > 256) return cudaErrorInvalidValue;
  WeightMap wm{};
  // 3-D view: d0 = 128 bytes of a panel, d1 = rows (stride row_bytes), d2 = panels (stride 128 B).
  // A box [128, 16, panels] lands as [panel][row][128 B], so the 128B swizzle permutes 16-byte chunks
  // by row: the consumers' per-row 4-byte reads of one column hit 8 different bank groups.
  const cuuint64_t dims3[3] = {128, rows, row_bytes / 128};
  const cuuint64_t strides3[2] = {row_bytes, 128};
  const cuuint32_t box3[3] = {128, 16, (cuuint32_t)panels};
  const cuuint32_t es3[3] = {1, 1, 1};
  CUresult r = fn(&wm.map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims3, strides3, box3,
                  es3, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  wm.per_panel = 0;
  if (r != CUDA_SUCCESS) {
    // 2-D view [rows][row_bytes]; one box [128 B, 16 rows] per panel.
    const cuuint64_t dims2[2] = {row_bytes, rows};
    const cuuint64_t strides2[1] = {row_bytes};
    const cuuint32_t box2[2] = {128, 16};
    const cuuint32_t es2[2] = {1, 1};
    r = fn(&wm.map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims2, strides2, box2, es2,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    wm.per_panel = 1;
  }
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (cache().size() > 4096) cache().clear();
    cache()[key] = wm;
  }
  *out = wm;
  return cudaSuccess;
}

cudaError_t scale_map(CUtensorMap* out, const void* base, uint64_t rows, uint64_t row_bytes, int box_bytes) {
  const Key key{(uint64_t)base, rows, row_bytes, 1, box_bytes};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = cache().find(key);
    if (it != cache().end()) {
      *out = it->second.map;
      return cudaSuccess;
    }
  }
  auto fn = encode_fn();
  if (!fn || row_bytes % 16 != 0 || box_bytes % 16 != 0 || box_bytes > 256) return cudaErrorInvalidValue;
  WeightMap wm{};
  const cuuint64_t dims[2] = {row_bytes, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)box_bytes, 16};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = fn(&wm.map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                        es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (cache().size() > 4096) cache().clear();
    cache()[key] = wm;
  }
  *out = wm.map;
  return cudaSuccess;
}

namespace {
bool cached(const Key& key, CUtensorMap* out) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = cache().find(key);
  if (it == cache().end()) return false;
  *out = it->second.map;
  return true;
}
void remember(const Key& key, const CUtensorMap& m) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (cache().size() > 4096) cache().clear();
  WeightMap wm{};
  wm.map = m;
  cache()[key] = wm;
}
}  // namespace

cudaError_t fp4_weight_map(CUtensorMap* out, const void* base, uint64_t rows, uint64_t K) {
  const Key key{(uint64_t)base, rows, K, 2, 0};
  if (cached(key, out)) return cudaSuccess;
  auto fn = encode_fn();
  if (!fn || K % 128 != 0 || ((uint64_t)base & 31) != 0 || (K / 2) % 32 != 0) return cudaErrorInvalidValue;
  CUtensorMap m;
  const cuuint64_t dims[2] = {K, rows};
  const cuuint64_t strides[1] = {K / 2};
  const cuuint32_t box[2] = {128, 128};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 2, const_cast<void*>(base), dims, strides,
                        box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  remember(key, m);
  *out = m;
  return cudaSuccess;
}

cudaError_t fp4_weight_map3(CUtensorMap* out, const void* base, uint64_t rows, uint64_t K, int chunks) {
  const Key key{(uint64_t)base, rows, K, 6, chunks};
  if (cached(key, out)) return cudaSuccess;
  auto fn = encode_fn();
  if (!fn || K % 128 != 0 || ((uint64_t)base & 31) != 0 || (K / 2) % 32 != 0 || chunks < 1 || chunks > 8)
    return cudaErrorInvalidValue;
  CUtensorMap m;
  const cuuint64_t dims[3] = {128, rows, K / 128};
  const cuuint64_t strides[2] = {K / 2, 64};
  const cuuint32_t box[3] = {128, 128, (cuuint32_t)chunks};
  const cuuint32_t es[3] = {1, 1, 1};
  const CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 3, const_cast<void*>(base), dims, strides, box,
                        es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  remember(key, m);
  *out = m;
  return cudaSuccess;
}

cudaError_t rows_map3(CUtensorMap* out, const void* base, uint64_t rows, uint64_t row_bytes, int box_rows,
                      int chunks) {
  const Key key{(uint64_t)base, rows, row_bytes, 7, box_rows * 16 + chunks};
  if (cached(key, out)) return cudaSuccess;
  auto fn = encode_fn();
  if (!fn || row_bytes % 128 != 0 || box_rows < 1 || box_rows > 256 || chunks < 1 || chunks > 8 ||
      ((uint64_t)base & 15) != 0)
    return cudaErrorInvalidValue;
  CUtensorMap m;
  const cuuint64_t dims[3] = {128, rows, row_bytes / 128};
  const cuuint64_t strides[2] = {row_bytes, 128};
  const cuuint32_t box[3] = {128, (cuuint32_t)box_rows, (cuuint32_t)chunks};
  const cuuint32_t es[3] = {1, 1, 1};
  const CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  remember(key, m);
  *out = m;
  return cudaSuccess;
}

cudaError_t sf_map(CUtensorMap* out, const void* base, uint64_t rows, uint64_t row_bytes, int box_rows) {
  const Key key{(uint64_t)base, rows, row_bytes, 4, box_rows};
  if (cached(key, out)) return cudaSuccess;
  auto fn = encode_fn();
  if (!fn || row_bytes % 16 != 0 || box_rows < 1 || box_rows > 256 || ((uint64_t)base & 15) != 0)
    return cudaErrorInvalidValue;
  CUtensorMap m;
  const cuuint64_t dims[2] = {row_bytes, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {16, (cuuint32_t)box_rows};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  remember(key, m);
  *out = m;
  return cudaSuccess;
}

cudaError_t bf16_rows_map(CUtensorMap* out, const void* base, uint64_t rows, uint64_t cols, int box_rows) {
  const Key key{(uint64_t)base, rows, cols, 5, box_rows};
  if (cached(key, out)) return cudaSuccess;
  auto fn = encode_fn();
  if (!fn || (cols * 2) % 16 != 0 || box_rows < 1 || box_rows > 256 || ((uint64_t)base & 15) != 0)
    return cudaErrorInvalidValue;
  CUtensorMap m;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  remember(key, m);
  *out = m;
  return cudaSuccess;
}

cudaError_t bf16_map3(CUtensorMap* out, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, int b1, int b2) {
  const Key key{(uint64_t)base, d1 | (d2 << 32), d0, 9, b1 * 1024 + b2};
  if (cached(key, out)) return cudaSuccess;
  auto fn = encode_fn();
  if (!fn || d0 % 64 != 0 || b1 < 1 || b1 > 256 || b2 < 1 || b2 > 256 || ((uint64_t)base & 15) != 0 ||
      d1 >= (1ull << 32) || d2 >= (1ull << 31))
    return cudaErrorInvalidValue;
  CUtensorMap m;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {d0 * 2, d0 * d1 * 2};
  const cuuint32_t box[3] = {64, (cuuint32_t)b1, (cuuint32_t)b2};
  const cuuint32_t es[3] = {1, 1, 1};
  const CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  remember(key, m);
  *out = m;
  return cudaSuccess;
}

cudaError_t rows_map(CUtensorMap* out, const void* base, uint64_t rows, uint64_t row_bytes, int box_rows) {
  const Key key{(uint64_t)base, rows, row_bytes, 3, box_rows};
  if (cached(key, out)) return cudaSuccess;
  auto fn = encode_fn();
  if (!fn || row_bytes % 128 != 0 || box_rows < 1 || box_rows > 256 || ((uint64_t)base & 15) != 0)
    return cudaErrorInvalidValue;
  CUtensorMap m;
  const cuuint64_t dims[2] = {row_bytes, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  remember(key, m);
  *out = m;
  return cudaSuccess;
}

cudaError_t packed64_map(CUtensorMap* out, const void* base, uint64_t rows, uint64_t row_bytes, int box_rows) {
  const Key key{(uint64_t)base, rows, row_bytes, 7, box_rows};
  if (cached(key, out)) return cudaSuccess;
  auto fn = encode_fn();
  if (!fn || row_bytes % 64 != 0 || box_rows < 1 || box_rows > 256 || ((uint64_t)base & 15) != 0)
    return cudaErrorInvalidValue;
  CUtensorMap m;
  const cuuint64_t dims[2] = {row_bytes, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  remember(key, m);
  *out = m;
  return cudaSuccess;
}

}  // namespace mimo
