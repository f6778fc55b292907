// RMSNorm between MoE layers: the decoder layer normalises the residual stream before its MoE block
// (engine/mimo_stream/model.py:75, `nn.RMSNorm(hidden, eps)`), which MLX evaluates as
// x * rsqrt(mean(x^2) + eps) * weight along the hidden axis.
//
// Here, per row t (fixed reduction order, so the result does not depend on the launch):
//   ss    = float32 sum of x^2: each thread sums its 8-element chunks in index order, then a
//           butterfly over the warp and the warps' partials in warp order
//   inv   = rsqrt(ss / H + eps), division and rsqrt correctly rounded (__fdiv_rn, __frsqrt_rn)
//   y     = bf16(x * inv)                          (no weight: unit weight)
//   y     = bf16(f32(weight) * bf16(x * inv))      (weight given: MLX casts the normalised row to the
//                                                   input type before the weight multiply)
// HBM-bound: one read of x and one write of y per row (16 KiB per 4096-wide bf16 row).
#include "common.cuh"
#include "kernels.h"

namespace mimo {

namespace {
constexpr int kNormThreads = 256;

__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const uint16_t* __restrict__ x,
                                                               const uint16_t* __restrict__ weight, int H,
                                                               float eps, uint16_t* __restrict__ y) {
  __shared__ float warp_ss[kNormThreads / 32];
  pdl_wait();  // inputs come from the preceding kernel (programmatic dependent launch)
  pdl_launch_dependents();
  const size_t row = (size_t)blockIdx.x * H;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row);
  const int chunks = H / 8;
  float ss = 0.f;
  for (int c = threadIdx.x; c < chunks; c += kNormThreads) {
    const uint4 v = __ldg(xr + c);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a = bf16_to_f32(w[i] & 0xFFFFu), b = bf16_to_f32(w[i] >> 16);
      ss = __fmaf_rn(a, a, ss);
      ss = __fmaf_rn(b, b, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xFFFFFFFFu, ss, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) warp_ss[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot = __fadd_rn(tot, warp_ss[i]);
  const float inv = __frsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)H), eps));
  uint4* yr = reinterpret_cast<uint4*>(y + row);
  const uint4* wr = reinterpret_cast<const uint4*>(weight);
  for (int c = threadIdx.x; c < chunks; c += kNormThreads) {
    const uint4 v = __ldg(xr + c);
    const uint32_t xw[4] = {v.x, v.y, v.z, v.w};
    uint32_t ww[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};  // bf16 1.0 pairs
    if (weight) {
      const uint4 g = __ldg(wr + c);
      ww[0] = g.x, ww[1] = g.y, ww[2] = g.z, ww[3] = g.w;
    }
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float a = bf16_round(__fmul_rn(bf16_to_f32(xw[i] & 0xFFFFu), inv));
      float b = bf16_round(__fmul_rn(bf16_to_f32(xw[i] >> 16), inv));
      if (weight) {
        a = __fmul_rn(bf16_to_f32(ww[i] & 0xFFFFu), a);
        b = __fmul_rn(bf16_to_f32(ww[i] >> 16), b);
      }
      o[i] = f32_to_bf16(a) | (f32_to_bf16(b) << 16);
    }
    yr[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}
}  // namespace

cudaError_t launch_rmsnorm(const uint16_t* x, const uint16_t* weight, int T, int H, float eps, uint16_t* y,
                           cudaStream_t st) {
  return launch_k(rmsnorm_kernel, dim3(T), dim3(kNormThreads), 0, st, x, weight, H, eps, y);
}

}  // namespace mimo
