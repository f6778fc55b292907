// Test and benchmark kit of the MiMo MoE library, built as its own shared library
// (libmimo_moe_testkit.so, C ABI in include/mimo_moe_testkit.h) so that the product library carries
// only the block's path: the seeded synthetic expert-pool fill (synth.cu) and the dense tensor-peak
// probe that gives the prefill roofline its denominators.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"
#include "mimo_moe.h"
#include "mimo_moe_testkit.h"

namespace mimo {
namespace tc {

// --------------------------------------------------------------------- dense tensor peak probe
// The block-scaled tensor-core peak of this GPU for the MMA forms the expert kernels use, measured
// rather than taken from a data sheet:
//   fp4 = 0  tcgen05.mma.kind::mxf8f6f4.block_scale, A e2m1 (padded layout), B e4m3, K = 32 a step;
//   fp4 = 1  tcgen05.mma.kind::mxf4.block_scale,      A and B e2m1 (packed),      K = 64 a step;
// both M = 128, N = 256 (the largest single-SM tile, long enough per instruction that one issuing
// thread keeps the pipe busy).  One CTA per SM; thread 0 issues `iters` x K = 128 worth of MMAs back
// to back on operands that stay in shared memory (no memory traffic in the loop) into one TMEM
// accumulator, then commits and waits (bounded).  FLOPs per launch = CTAs x iters x 2 x 128 x 256 x 128.
constexpr int kPeakM = 128;
constexpr int kPeakN = 256;
// 52 KB used; 120 KB requested so that no SM holds two CTAs (each allocates all 512 TMEM columns).
constexpr int kPeakSmem = 120 * 1024;
static_assert(1024 + 1024 + 16384 + 32768 + 1024 <= kPeakSmem, "probe shared memory");
__global__ void __launch_bounds__(128, 1) tc_peak_kernel(int iters, int fp4, int32_t* status) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* done = reinterpret_cast<uint64_t*>(smem);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + 8);
  uint8_t* base = reinterpret_cast<uint8_t*>(((uintptr_t)(smem + 1024) + 1023) & ~(uintptr_t)1023);
  uint8_t* A = base;                  // 128 x 128 e2m1: 16 KB padded / 8 KB packed
  uint8_t* B = base + 16384;          // 256 x 128 e4m3 (32 KB) or e2m1 packed (16 KB)
  uint8_t* SF = base + 16384 + 32768; // two 512-byte scale blocks
  const int warp = threadIdx.x >> 5;
  // Small finite operands: e2m1 1.0 in every nibble, e4m3 1.0, scales 2^0.
  for (int i = threadIdx.x; i < 16384 / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(A)[i] = 0x22222222u;
  for (int i = threadIdx.x; i < 32768 / 4; i += blockDim.x)
    reinterpret_cast<uint32_t*>(B)[i] = fp4 ? 0x22222222u : 0x38383838u;
  for (int i = threadIdx.x; i < 1024 / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(SF)[i] = 0x7F7F7F7Fu;
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    mbar_init(done, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  if (threadIdx.x == 0) {
    const uint32_t sfa = tbase + kPeakN, sfb = tbase + kPeakN + 4;
    tc_cp_sf(sfa, desc_sf(smem_u32(SF)));
    tc_cp_sf(sfb, desc_sf(smem_u32(SF + 512)));
    tc_cp_sf(sfb + 4, desc_sf(smem_u32(SF + 512)));  // scale rows 128..255 of B, if read from there
    const uint32_t a = smem_u32(A), b = smem_u32(B);
    for (int i = 0; i < iters; ++i) {
      if (fp4) {
#pragma unroll
        for (int kk = 0; kk < 2; ++kk)
          tc_mma_mxf4(tbase, desc_sw64(a + kk * 32), desc_sw64(b + kk * 32), idesc_mxf4(kPeakM, kPeakN, 2 * kk),
                      sfa | ((uint32_t)(2 * kk) << 30), sfb | ((uint32_t)(2 * kk) << 30), (i | kk) != 0);
      } else {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_mx(tbase, desc_sw128(a + kk * 32), desc_sw128(b + kk * 32), idesc_mx(kPeakN, kk),
                    sfa | ((uint32_t)kk << 30), sfb | ((uint32_t)kk << 30), (i | kk) != 0);
      }
    }
    tc_commit(done);
    if (!mbar_wait(done, 0)) set_status(status, MIMO_ETIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

}  // namespace tc
}  // namespace mimo

extern "C" {

int mimo_moe_fill_synthetic_pool(uint32_t* gate_w, uint8_t* gate_s, uint32_t* up_w, uint8_t* up_s,
                                 uint32_t* down_w, uint8_t* down_s, int32_t S, int32_t H, int32_t I,
                                 uint64_t seed, int32_t layer, int32_t first_expert, void* stream) {
  if (!gate_w || !gate_s || !up_w || !up_s || !down_w || !down_s || S < 1 || H < 256 || I < 256 ||
      H % 256 || I % 256 || layer < 0 || first_expert < 0)
    return MIMO_EINVAL;
  return mimo::launch_fill_synthetic(gate_w, gate_s, up_w, up_s, down_w, down_s, S, H, I, seed, layer,
                                     first_expert, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? MIMO_OK
             : MIMO_ECUDA;
}

int mimo_moe_tensor_peak(int32_t kind, int32_t iters, float* tflops, int32_t* status, void* stream) {
  if ((kind != 0 && kind != 1) || iters < 1 || iters > (1 << 24) || !tflops || !status) return MIMO_EINVAL;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(mimo::tc::tc_peak_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             mimo::tc::kPeakSmem);
  if (e != cudaSuccess) return MIMO_ECUDA;
  cudaEvent_t a = nullptr, b = nullptr;
  e = cudaEventCreate(&a);
  if (e == cudaSuccess) e = cudaEventCreate(&b);
  if (e == cudaSuccess) e = cudaEventRecord(a, st);
  if (e == cudaSuccess) {
    mimo::tc::tc_peak_kernel<<<sms, 128, mimo::tc::kPeakSmem, st>>>(iters, kind, status);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaEventRecord(b, st);
  if (e == cudaSuccess) e = cudaEventSynchronize(b);
  float ms = 0.f;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, a, b);
  if (a) cudaEventDestroy(a);
  if (b) cudaEventDestroy(b);
  if (e != cudaSuccess) return MIMO_ECUDA;
  *tflops = ms > 0.f ? (float)(2.0 * 128 * 256 * 128 * (double)iters * sms / (ms * 1e-3) / 1e12) : 0.f;
  return MIMO_OK;
}

}  // extern "C"
