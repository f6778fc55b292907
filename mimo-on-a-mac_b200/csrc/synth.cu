// Synthetic expert pools (benchmarks / tests): splitmix64 finaliser over a per-tensor key and a Weyl
// sequence (Steele, Lea & Flood 2014).  The numpy twin regenerates any single expert bit for bit.
#include "common.cuh"
#include "kernels.h"

namespace mimo {

__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

static uint64_t tensor_key(uint64_t seed, int layer, int tensor) {
  return mix64(seed) ^ ((uint64_t)(layer * 8 + tensor + 1) * kGolden);
}

// Weights: u64 j of the whole layer tensor -> two little-endian u32 words.
__global__ void fill_words_kernel(uint64_t* __restrict__ dst, uint64_t key, uint64_t first, uint64_t n) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    dst[i] = mix64(key + (first + i + 1) * kGolden);
}

// Scales: byte b of hash u64 j -> scale byte 8j+b = 120 if (hash byte < 176) else 119.
__global__ void fill_scales_kernel(uint64_t* __restrict__ dst, uint64_t key, uint64_t first, uint64_t n) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t h = mix64(key + (first + i + 1) * kGolden);
    uint64_t out = 0;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const uint64_t byte = (h >> (8 * b)) & 0xFFull;
      out |= (byte < 176ull ? 120ull : 119ull) << (8 * b);
    }
    dst[i] = out;
  }
}

cudaError_t launch_fill_synthetic(uint32_t* gw, uint8_t* gs, uint32_t* uw, uint8_t* us, uint32_t* dw,
                                  uint8_t* ds, int S, int H, int I, uint64_t seed, int layer,
                                  int first_expert, cudaStream_t st) {
  struct T {
    void* p;
    int tensor;
    bool scale;
    uint64_t per_expert;  // u64 units per expert
  };
  const uint64_t w_pe = (uint64_t)I * H / 16, s_pe = (uint64_t)I * H / 256;
  const T ts[6] = {{gw, 0, false, w_pe}, {gs, 1, true, s_pe}, {uw, 2, false, w_pe},
                   {us, 3, true, s_pe},  {dw, 4, false, w_pe}, {ds, 5, true, s_pe}};
  for (const T& x : ts) {
    const uint64_t key = tensor_key(seed, layer, x.tensor);
    const uint64_t first = (uint64_t)first_expert * x.per_expert;
    const uint64_t n = (uint64_t)S * x.per_expert;
    const unsigned blocks = (unsigned)std::min<uint64_t>((n + 255) / 256, 148ull * 64);
    if (x.scale)
      fill_scales_kernel<<<blocks, 256, 0, st>>>(static_cast<uint64_t*>(x.p), key, first, n);
    else
      fill_words_kernel<<<blocks, 256, 0, st>>>(static_cast<uint64_t*>(x.p), key, first, n);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace mimo
