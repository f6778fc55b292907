// Decode-size projections of the decoder layer (nn.Linear on T <= 8 token rows: the q|k|v and o projections
// of mimo_v2.py:117-149, the dense MLP's gate|up and down): y[T, N] = bf16(x[T, K] . W[N, K]^T), float32
// accumulation, on the tcgen05 tensor cores.  The weights are read once, so the kernel is an HBM stream:
//
//   work item = (128-row tile of W, K segment); items are dealt round-robin over a persistent grid of one
//   CTA per SM (the split count S is chosen on the host to balance the items over the SMs);
//   warp 0 (one thread)  TMA producer: per 64-value K chunk a [128 rows x 64] box of W (16 KB) and the
//                        [16 rows x 64] box of x (T rows, the rest read as zeros) into a 12-stage ring;
//   warp 1 (one thread)  MMA issuer: D[128 x 16] += W_chunk . x_chunk^T (tcgen05 kind::f16, M 128, N 16,
//                        K 16 per instruction) into one of two TMEM accumulators (the next item's MMAs run
//                        while the epilogue reads the previous one);
//   warps 4-7            epilogue, one thread per W row (TMEM lane): the T values of its row to y (bf16,
//                        S = 1) or to the float32 partial of its segment (S > 1), which a second kernel adds
//                        in segment order (so the result does not depend on the launch).
// Every wait is bounded and sets MIMO_ETIMEOUT in the status word.
#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace mimo {

namespace {

constexpr int kLinStages = 12;  // 216 KB of weights and activations in flight per SM
constexpr int kLinRows = 128, kLinTok = 16, kLinKC = 64;
constexpr uint32_t kLinWBytes = kLinRows * kLinKC * 2;  // 16 KB
constexpr uint32_t kLinXBytes = kLinTok * kLinKC * 2;   // 2 KB
constexpr uint32_t kLinStage = kLinWBytes + kLinXBytes;
constexpr uint32_t kLinSmem = 2048 + kLinStages * kLinStage;  // barriers + alignment slack + ring
constexpr int kLinThreads = 256;

__global__ void __launch_bounds__(kLinThreads, 1) linear_decode_kernel(const __grid_constant__ LinearParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kLinStages;
  uint64_t* acc_full = empty + kLinStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + 512);
  uint8_t* ring = reinterpret_cast<uint8_t*>(((uintptr_t)(smem + 1024) + 1023) & ~(uintptr_t)1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kseg = p.K / p.S, nch = kseg / kLinKC;
  const int items = p.tiles * p.S;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kLinStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
    }
    mbar_init(drain, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tslot, 32);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tacc = *tslot;
  pdl_wait();  // x comes from the preceding kernel (programmatic dependent launch)
  pdl_launch_dependents();
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {  // ------------------------------------------------------------------- TMA producer
      tma_prefetch_map(&p.wmap);
      tma_prefetch_map(&p.xmap);
      const uint64_t pol_w = l2_evict_first_policy();    // weights: read once
      const uint64_t pol_x = tc::l2_evict_normal_policy();
      int it = 0;
      for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
        const int n0 = (item % p.tiles) * kLinRows, k0 = (item / p.tiles) * kseg;
        for (int c = 0; c < nch; ++c, ++it) {
          const int s = it % kLinStages;
          if (!mbar_wait(&empty[s], (uint32_t)(((it / kLinStages) & 1) ^ 1))) {
            ok = false;
            break;
          }
          uint8_t* st = ring + s * kLinStage;
          mbar_arrive_expect_tx(&full[s], kLinStage);
          tma_load_2d(st, &p.wmap, k0 + c * kLinKC, n0, &full[s], pol_w);
          tma_load_2d(st + kLinWBytes, &p.xmap, k0 + c * kLinKC, 0, &full[s], pol_x);
        }
      }
      for (int j = it - 1; j >= 0 && j >= it - kLinStages; --j)  // no copy still landing at exit
        if (!mbar_wait(&full[j % kLinStages], (uint32_t)((j / kLinStages) & 1))) ok = false;
    }
  } else if (warp == 1) {
    if (lane == 0) {  // -------------------------------------------------------------------- MMA issuer
      const uint32_t idesc = tc::idesc_bf16(kLinRows, kLinTok);
      int it = 0, local = 0;
      for (int item = blockIdx.x; item < items && ok; item += gridDim.x, ++local) {
        const int buf = local & 1;
        if (local >= 2 && !mbar_wait(&acc_empty[buf], (uint32_t)(((local >> 1) - 1) & 1))) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        for (int c = 0; c < nch; ++c, ++it) {
          const int s = it % kLinStages;
          if (!mbar_wait(&full[s], (uint32_t)((it / kLinStages) & 1))) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t aw = smem_u32(ring + s * kLinStage), ax = aw + kLinWBytes;
#pragma unroll
          for (int kk = 0; kk < kLinKC / 16; ++kk)
            tc::tc_mma_f16(tacc + buf * kLinTok, tc::desc_sw128(aw + kk * 32), tc::desc_sw128(ax + kk * 32), idesc,
                           (c | kk) != 0 ? 1u : 0u);
          tc::tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc::tc_commit(&acc_full[buf]);
      }
      tc::tc_commit(drain);  // every MMA issued above has completed once this arrives
      if (!mbar_wait(drain, 0)) ok = false;
    }
  } else if (warp >= 4) {  // --------------------------------------------------------------------- epilogue
    const int r = threadIdx.x - 128;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    int local = 0;
    for (int item = blockIdx.x; item < items; item += gridDim.x, ++local) {
      const int buf = local & 1;
      ok = ok && mbar_wait(&acc_full[buf], (uint32_t)((local >> 1) & 1));
      if (!__all_sync(0xFFFFFFFFu, ok)) {
        ok = false;
        break;
      }
      tc::tc_fence_after();
      float v[16];
      tc::tmem_ld<16>(tacc + lane_off + buf * kLinTok, v);
      tc::tmem_wait_ld();
      tc::tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
      const int n = (item % p.tiles) * kLinRows + r, seg = item / p.tiles;
      if (n < p.N) {
        if (p.S == 1) {
#pragma unroll
          for (int t = 0; t < kLinTok; ++t)
            if (t < p.T) p.y[(size_t)t * p.N + n] = (uint16_t)f32_to_bf16(v[t]);
        } else {
#pragma unroll
          for (int t = 0; t < kLinTok; ++t)
            if (t < p.T) p.part[((size_t)seg * p.T + t) * p.N + n] = v[t];
        }
      }
    }
  }
  if (!ok && p.status) set_status(p.status, MIMO_ETIMEOUT);
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tacc, 32);
  }
}

// y = bf16(sum over segments, in order, of the float32 partials); four values per thread.
__global__ void __launch_bounds__(256) linear_reduce_kernel(const float* __restrict__ part, int S, size_t n4,
                                                            uint16_t* __restrict__ y) {
  pdl_wait();  // inputs come from the preceding kernel (programmatic dependent launch)
  pdl_launch_dependents();
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    float4 a = reinterpret_cast<const float4*>(part)[i];
    for (int s = 1; s < S; ++s) {
      const float4 b = reinterpret_cast<const float4*>(part)[(size_t)s * n4 + i];
      a.x += b.x, a.y += b.y, a.z += b.z, a.w += b.w;
    }
    reinterpret_cast<uint2*>(y)[i] =
        make_uint2(f32_to_bf16(a.x) | (f32_to_bf16(a.y) << 16), f32_to_bf16(a.z) | (f32_to_bf16(a.w) << 16));
  }
}

}  // namespace

int linear_decode_splits(int N, int K, int num_sms) {
  // the item count per SM round times the chunks per item (plus ~2 chunks of per-item turnaround): the
  // smallest wins, fewer segments on ties
  const int tiles = (N + kLinRows - 1) / kLinRows;
  int best = 1;
  long best_cost = -1;
  for (int S = 1; S <= 32; S *= 2) {
    if (K % (S * kLinKC) != 0 || K / S < 4 * kLinKC) break;
    const long rounds = ((long)tiles * S + num_sms - 1) / num_sms;
    const long cost = rounds * (K / S / kLinKC + 2);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = S;
    }
  }
  return best;
}

cudaError_t launch_linear_decode(const uint16_t* x, const uint16_t* w, int T, int N, int K, int S, uint16_t* y,
                                 float* part, int32_t* status, int num_sms, cudaStream_t st) {
  LinearParams p;
  std::memset(&p, 0, sizeof(p));
  cudaError_t e = bf16_rows_map(&p.wmap, w, (uint64_t)N, (uint64_t)K, kLinRows);
  if (e == cudaSuccess) e = bf16_rows_map(&p.xmap, x, (uint64_t)T, (uint64_t)K, kLinTok);
  if (e != cudaSuccess) return e;
  p.y = y, p.part = part, p.status = status;
  p.T = T, p.N = N, p.K = K, p.S = S, p.tiles = (N + kLinRows - 1) / kLinRows;
  static bool attr_set[128] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 128 && !attr_set[dev]) {
    e = cudaFuncSetAttribute(linear_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kLinSmem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const int items = p.tiles * S;
  e = launch_k(linear_decode_kernel, dim3(std::min(items, num_sms)), dim3(kLinThreads), kLinSmem, st, p);
  if (e != cudaSuccess || S == 1) return e;
  const size_t n4 = (size_t)T * N / 4;
  return launch_k(linear_reduce_kernel, dim3((unsigned)std::min<size_t>((n4 + 255) / 256, (size_t)num_sms * 8)),
                  dim3(256), 0, st, (const float*)part, S, n4, y);
}

}  // namespace mimo
