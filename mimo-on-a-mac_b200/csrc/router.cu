// Router: FP32 logits GEMV/GEMM, sigmoid + noaux bias, warp top-k with a total order, normalised
// weights.  Follows Router.__call__ of the reference (engine/mimo_stream/model.py:58-65).
#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "route_dev.cuh"
#include "tcgen05.cuh"

namespace mimo {

// One warp: logits of expert row e for tokens [t0, t0+nt) (nt <= 8).  Lane l takes the 8-element
// chunks c = l + 32 i in ascending i; each chunk is 8 float32 FMAs in element order; lanes are then
// combined by a fixed xor tree.  The whole row (up to 4096 elements per pass) is loaded before use.
__device__ __forceinline__ void logits_warp(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                                            float* __restrict__ logits, int t0, int nt, int H, int E, int e) {
  const int lane = threadIdx.x & 31;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  const uint4* wr = reinterpret_cast<const uint4*>(w + (size_t)e * H);
  const int nchunk = H >> 3;
  for (int base = 0; base < nchunk; base += 32 * 16) {
    uint4 wv[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int c = base + lane + 32 * i;
      wv[i] = (c < nchunk) ? __ldg(wr + c) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int tt = 0; tt < 8; ++tt) {
      if (tt < nt) {
        const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)(t0 + tt) * H);
        float a = acc[tt];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int c = base + lane + 32 * i;
          if (c < nchunk) {
            const uint4 xv = __ldg(xr + c);
            a = fmaf(__uint_as_float(xv.x << 16), __uint_as_float(wv[i].x << 16), a);
            a = fmaf(__uint_as_float(xv.x & 0xFFFF0000u), __uint_as_float(wv[i].x & 0xFFFF0000u), a);
            a = fmaf(__uint_as_float(xv.y << 16), __uint_as_float(wv[i].y << 16), a);
            a = fmaf(__uint_as_float(xv.y & 0xFFFF0000u), __uint_as_float(wv[i].y & 0xFFFF0000u), a);
            a = fmaf(__uint_as_float(xv.z << 16), __uint_as_float(wv[i].z << 16), a);
            a = fmaf(__uint_as_float(xv.z & 0xFFFF0000u), __uint_as_float(wv[i].z & 0xFFFF0000u), a);
            a = fmaf(__uint_as_float(xv.w << 16), __uint_as_float(wv[i].w << 16), a);
            a = fmaf(__uint_as_float(xv.w & 0xFFFF0000u), __uint_as_float(wv[i].w & 0xFFFF0000u), a);
          }
        }
        acc[tt] = a;
      }
    }
  }
#pragma unroll
  for (int tt = 0; tt < 8; ++tt) {
    float v = acc[tt];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    acc[tt] = v;
  }
#pragma unroll
  for (int tt = 0; tt < 8; ++tt)
    if (lane == tt && tt < nt) logits[(size_t)(t0 + tt) * E + e] = acc[tt];
}

// logits[t, e] = sum_k f32(x[t,k]) * f32(w[e,k]): one warp per expert row, 8 tokens per block row.
__global__ void __launch_bounds__(256) router_logits_kernel(const uint16_t* __restrict__ x,
                                                            const uint16_t* __restrict__ w,
                                                            float* __restrict__ logits, int T, int H,
                                                            int E) {
  const int warp = threadIdx.x >> 5;
  const int e = blockIdx.y * 8 + warp;
  const int t0 = blockIdx.x * 8;  // token blocks on x: gridDim.y stops at 65535
  if (e >= E) return;
  logits_warp(x, w, logits, t0, min(8, T - t0), H, E, e);
}

// One warp per token (see topk_warp).
__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ logits,
                                                          const float* __restrict__ bias, int T,
                                                          int E, int topk, int32_t* __restrict__ idx,
                                                          float* __restrict__ weight) {
  const int warp = threadIdx.x >> 5;
  const int t = blockIdx.x * 8 + warp;
  if (t >= T) return;
  topk_warp(logits + (size_t)t * E, bias, E, topk, idx + (size_t)t * topk, weight + (size_t)t * topk);
}

// Decode (T <= 8) routing in two launches.  route_logits_kernel: CTA c owns router rows [4c, 4c+4) (E / 4
// CTAs, so the 2 MiB router weight streams through 64 SMs): float32 FMAs of exact bf16 products in a
// fixed order (route_logits4_cta); each CTA turns its logits into scores (the exact sigmoid) at once
// and, with xq non-null, first splits its share of x into the terms the tensor-core expert kernels
// read.  route_select_kernel (one CTA, launched as its programmatic dependent): top-k of every token
// and grouping of the routes by distinct expert.
constexpr int kRouteWarps = 16;
// Logits of router rows [4c, 4c+4) (c = blockIdx.x) for T <= 8 tokens, on 16 warps: warp w takes the
// K slice [w H / 16, (w + 1) H / 16) of all 4 rows and all T tokens (so the CTA reads its 4 rows and x
// once); lane l reads the 8-value chunks l, l + 32, ... of the slice (16-byte loads) and accumulates
// float32 FMAs of the exact bf16 products in chunk order.  The 32 sums (row, token) of a warp are
// reduce-scattered over its lanes in a fixed butterfly (lane j ends with sum j = row * 8 + token), and
// the 16 warps' sums are added in warp order (shared memory), so the sum order is fixed.  score
// (optional) receives sigmoid_score of each logit.  Needs H % 128 == 0 and 16 warps; ends after the
// stores (one __syncthreads inside).
__device__ __forceinline__ void route_logits4_cta(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                                                  int T, int H, int E, float* __restrict__ logits,
                                                  float* __restrict__ score, float (*red)[128]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = H / 128;  // 8-value chunks per slice
  const int c0 = warp * nch;
  float a[32];  // a[r * 8 + t]
#pragma unroll
  for (int j = 0; j < 32; ++j) a[j] = 0.f;
  for (int c = lane; c < nch; c += 32) {
    uint4 wv[4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
      wv[r] = __ldg(reinterpret_cast<const uint4*>(w + (size_t)(blockIdx.x * 4 + r) * H) + c0 + c);
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      if (t < T) {
        const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + (size_t)t * H) + c0 + c);
        const float x0 = __uint_as_float(xv.x << 16), x1 = __uint_as_float(xv.x & 0xFFFF0000u);
        const float x2 = __uint_as_float(xv.y << 16), x3 = __uint_as_float(xv.y & 0xFFFF0000u);
        const float x4 = __uint_as_float(xv.z << 16), x5 = __uint_as_float(xv.z & 0xFFFF0000u);
        const float x6 = __uint_as_float(xv.w << 16), x7 = __uint_as_float(xv.w & 0xFFFF0000u);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          float v = a[r * 8 + t];
          v = fmaf(x0, __uint_as_float(wv[r].x << 16), v);
          v = fmaf(x1, __uint_as_float(wv[r].x & 0xFFFF0000u), v);
          v = fmaf(x2, __uint_as_float(wv[r].y << 16), v);
          v = fmaf(x3, __uint_as_float(wv[r].y & 0xFFFF0000u), v);
          v = fmaf(x4, __uint_as_float(wv[r].z << 16), v);
          v = fmaf(x5, __uint_as_float(wv[r].z & 0xFFFF0000u), v);
          v = fmaf(x6, __uint_as_float(wv[r].w << 16), v);
          v = fmaf(x7, __uint_as_float(wv[r].w & 0xFFFF0000u), v);
          a[r * 8 + t] = v;
        }
      }
    }
  }
  // reduce-scatter: at offset o a lane keeps the upper half of its values if lane & o, else the lower
  // half, and adds its partner's copy of the half it keeps; lane j ends with the warp's sum j
#pragma unroll
  for (int o = 16, n = 32; o > 0; o >>= 1, n >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int j = 0; j < n / 2; ++j) {
      const float send = up ? a[j] : a[j + n / 2];
      const float keep = up ? a[j + n / 2] : a[j];
      a[j] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, o);
    }
  }
  red[warp][lane] = a[0];
  __syncthreads();
  if (threadIdx.x < 32) {
    const int r = threadIdx.x >> 3, t = threadIdx.x & 7;
    if (t < T) {
      float sum = 0.f;
#pragma unroll
      for (int ww = 0; ww < kRouteWarps; ++ww) sum += red[ww][threadIdx.x];
      const int e = blockIdx.x * 4 + r;
      logits[(size_t)t * E + e] = sum;
      if (score) score[(size_t)t * E + e] = sigmoid_score(sum);
    }
  }
}

// Stand-alone logits for T <= 8 (the router entry point and the expert-parallel route scatter): E / 4
// CTAs of the decode route kernel's arithmetic, so every path routes from the same logits bit for bit.
__global__ void __launch_bounds__(kRouteWarps * 32) router_logits_small_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ w, int T, int H, int E,
    float* __restrict__ logits) {
  __shared__ float red[kRouteWarps][128];
  route_logits4_cta(x, w, T, H, E, logits, nullptr, red);
}

__global__ void __launch_bounds__(kRouteWarps * 32) route_logits_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ w, int T, int H, int E,
    float* __restrict__ logits, float* __restrict__ score, uint8_t* __restrict__ xq, uint8_t* __restrict__ xs,
    int32_t* status, int fp4, int32_t* ready, int ready_n) {
  __shared__ float red[kRouteWarps][128];
  // The expert kernels' copy of x, split by every CTA before its logits: e4m3 terms (token t -> rows
  // t (hi) and 8 + t (lo)) one 32-value block per warp (lane = value), or e2m1 terms (token t's term j
  // at row j * 8 + t) one block per thread.
  auto split_share = [&]() {
    const int nb = H / 32;
    if (!fp4) {
      const int nw = blockDim.x >> 5;
      for (int b = (threadIdx.x >> 5) * gridDim.x + blockIdx.x; b < T * nb; b += gridDim.x * nw) {
        const int t = b / nb, blk = b - t * nb;
        tc::split_block32_warp(x + (size_t)t * H + blk * 32, xq + (size_t)t * H + blk * 32,
                               xq + (size_t)(8 + t) * H + blk * 32, xs + (size_t)t * nb + blk,
                               xs + (size_t)(8 + t) * nb + blk, status);
      }
      return;
    }
    for (int b = threadIdx.x * gridDim.x + blockIdx.x; b < T * nb; b += gridDim.x * blockDim.x) {
      const int t = b / nb, blk = b - t * nb;
      tc::split_block32_fp4(x + (size_t)t * H + blk * 32, xq + (size_t)t * (H / 2) + blk * 16,
                            (size_t)8 * (H / 2), xs + (size_t)t * nb + blk, (size_t)8 * nb, status);
    }
  };
  pdl_wait();  // x may come from the preceding kernel
  pdl_launch_dependents();
  // the expert kernel's per-call counters and flags: every CTA zeroes a share (that kernel starts
  // reading them only after both route launches have completed)
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; ready && i < ready_n; i += gridDim.x * blockDim.x) ready[i] = 0;
  if (xq) split_share();
  route_logits4_cta(x, w, T, H, E, logits, score, red);
}

// Decode routing, second launch (one CTA, programmatically dependent on route_logits_kernel): warp t
// selects token t's top-k from the scores (the router's order); the CTA then groups the routes by
// distinct expert (group_routes, engine/mimo_stream/kernels.py:149-173) and, with x16 non-null, writes
// the f16 copy of x that the mma.sync expert kernels read.
__global__ void __launch_bounds__(kRouteWarps * 32) route_select_kernel(
    const uint16_t* __restrict__ x, const float* __restrict__ bias, int T, int H, int E, int topk, int R,
    int32_t* __restrict__ idx, float* __restrict__ wts, int32_t* uids, int32_t* urows, int32_t* ucnt, float* uw,
    int32_t* gidx, int32_t* num_unique, __half* __restrict__ x16, const float* __restrict__ score, int32_t* status) {
  __shared__ int32_t sid[64], s_idx[64];
  __shared__ float s_w[64];
  __shared__ uint32_t bitmap[32];
  const int warp = threadIdx.x >> 5;
  pdl_wait();  // the scores come from route_logits_kernel
  pdl_launch_dependents();
  if (warp < T)
    topk_warp_impl<true>(score + (size_t)warp * E, bias, E, topk, idx + warp * topk, wts + warp * topk,
                         s_idx + warp * topk, s_w + warp * topk);
  __syncthreads();
  const int P = T * topk;
  group_routes_cta(s_idx, s_w, P, topk, R, E, min(E, P), uids, urows, ucnt, uw, gidx, num_unique, status,
                   sid, bitmap);
  for (int i = threadIdx.x * 2; x16 && i < T * H; i += blockDim.x * 2) {
    const uint32_t v = *reinterpret_cast<const uint32_t*>(x + i);
    float lo = __uint_as_float(v << 16), hi = __uint_as_float(v & 0xFFFF0000u);
    if ((fabsf(lo) > 65504.f && !isnan(lo)) || (fabsf(hi) > 65504.f && !isnan(hi))) {
      set_status(status, MIMO_ERANGE);
      lo = fminf(fmaxf(lo, -65504.f), 65504.f);
      hi = fminf(fmaxf(hi, -65504.f), 65504.f);
    }
    *reinterpret_cast<__half2*>(x16 + i) = __halves2half2(__float2half_rn(lo), __float2half_rn(hi));
  }
}

// Prefill router logits on the tensor cores: one CTA per 128-token x 64-expert tile, K = H in
// 64-value chunks through a TMA ring; tcgen05.mma.kind::f16 multiplies bf16 x by bf16 W exactly and
// accumulates in float32 in TMEM.  Warp 0 lane 0 issues the copies, warp 1 lane 0 the MMAs; all four
// warps then read their 32 token rows back (tcgen05.ld) and store 64 logits per row.
constexpr int kRtM = 128, kRtN = 64, kRtKC = 64, kRtStages = 6;
constexpr int kRtStageBytes = (kRtM + kRtN) * kRtKC * 2;  // 24 KiB
constexpr int kRtSmem = 1024 + 1024 + kRtStages * kRtStageBytes;

struct RouterTcParams {
  CUtensorMap xmap;  // x bf16 [T][H], box [64, 128], 128B swizzle (rows past T read as zero)
  CUtensorMap wmap;  // W bf16 [E][H], box [64, 64], 128B swizzle
  float* logits;
  int T, H, E;
  int32_t* status;  // may be null (the stand-alone router entry has no status word)
};

__global__ void __launch_bounds__(128, 1) router_tc_kernel(const __grid_constant__ RouterTcParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kRtStages;
  uint64_t* acc = empty + kRtStages;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(acc + 1);
  uint8_t* stages = reinterpret_cast<uint8_t*>(((uintptr_t)(smem + 1024) + 1023) & ~(uintptr_t)1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kRtM, e0 = blockIdx.y * kRtN;
  const int nk = p.H / kRtKC;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kRtStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc, 1);
    mbar_fence_init();
  }
  if (warp == 2) {
    tc::tmem_alloc(tslot, kRtN);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tslot;
  bool ok = true;
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&p.xmap);
    tma_prefetch_map(&p.wmap);
    const uint64_t pol = tc::l2_evict_normal_policy();
    int issued = 0;
    for (int k = 0; k < nk; ++k) {
      const int s = k % kRtStages;
      if (!mbar_wait(&empty[s], (uint32_t)(((k / kRtStages) & 1) ^ 1))) {
        ok = false;
        break;
      }
      uint8_t* sb = stages + s * kRtStageBytes;
      mbar_arrive_expect_tx(&full[s], kRtStageBytes);
      tma_load_2d(sb, &p.xmap, k * kRtKC, m0, &full[s], pol);
      tma_load_2d(sb + kRtM * kRtKC * 2, &p.wmap, k * kRtKC, e0, &full[s], pol);
      ++issued;
    }
    for (int k = issued - 1; k >= 0 && k >= issued - kRtStages; --k)  // copies landed before exit
      if (!mbar_wait(&full[k % kRtStages], (uint32_t)((k / kRtStages) & 1))) ok = false;
  } else if (warp == 1 && lane == 0) {
    const uint32_t idesc = tc::idesc_bf16(kRtM, kRtN);
    for (int k = 0; k < nk; ++k) {
      const int s = k % kRtStages;
      if (!mbar_wait(&full[s], (uint32_t)((k / kRtStages) & 1))) {
        ok = false;
        break;
      }
      tc::tc_fence_after();
      const uint32_t sa = smem_u32(stages + s * kRtStageBytes), sb = sa + kRtM * kRtKC * 2;
#pragma unroll
      for (int kk = 0; kk < kRtKC / 16; ++kk)
        tc::tc_mma_f16(tbase, tc::desc_sw128(sa + kk * 32), tc::desc_sw128(sb + kk * 32), idesc, (k | kk) != 0);
      tc::tc_commit(&empty[s]);
    }
    tc::tc_commit(acc);  // also drains every MMA issued before
  }
  if (!ok && p.status) set_status(p.status, MIMO_ETIMEOUT);
  __syncwarp();
  if (!mbar_wait(acc, 0)) {
    if (lane == 0 && p.status) set_status(p.status, MIMO_ETIMEOUT);
  } else {
    tc::tc_fence_after();
    const int row = m0 + warp * 32 + lane;
#pragma unroll
    for (int c = 0; c < kRtN; c += 16) {
      float v[16];
      tc::tmem_ld<16>(tbase + ((uint32_t)(warp * 32) << 16) + c, v);
      tc::tmem_wait_ld();
      if (row < p.T) {
        float4* dst = reinterpret_cast<float4*>(p.logits + (size_t)row * p.E + e0 + c);
#pragma unroll
        for (int j = 0; j < 4; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, kRtN);
  }
}

cudaError_t launch_router_logits(const uint16_t* x, const uint16_t* w, float* logits, int T, int H,
                                 int E, cudaStream_t st, int32_t* status) {
  if (T > 8 && E % kRtN == 0 && H % kRtKC == 0 && ((uintptr_t)x & 15) == 0 &&
      ((uintptr_t)w & 15) == 0 && ((uintptr_t)logits & 15) == 0) {
    RouterTcParams p;
    std::memset(&p, 0, sizeof(p));
    cudaError_t e = bf16_rows_map(&p.xmap, x, (uint64_t)T, (uint64_t)H, kRtM);
    if (e == cudaSuccess) e = bf16_rows_map(&p.wmap, w, (uint64_t)E, (uint64_t)H, kRtN);
    if (e == cudaSuccess) {
      p.logits = logits;
      p.T = T;
      p.H = H;
      p.E = E;
      p.status = status;
      e = cudaFuncSetAttribute(router_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kRtSmem);
      if (e != cudaSuccess) return e;
      router_tc_kernel<<<dim3((T + kRtM - 1) / kRtM, E / kRtN), 128, kRtSmem, st>>>(p);
      return cudaGetLastError();
    }
  }
  if (T <= 8 && E % 16 == 0 && H % 256 == 0) {  // decode sizes: 16-row tiles on bf16 mma.sync
    router_logits_small_kernel<<<E / 4, kRouteWarps * 32, 0, st>>>(x, w, T, H, E, logits);
    return cudaGetLastError();
  }
  dim3 grid((T + 7) / 8, (E + 7) / 8);
  router_logits_kernel<<<grid, 256, 0, st>>>(x, w, logits, T, H, E);
  return cudaGetLastError();
}

cudaError_t launch_router_topk(const float* logits, const float* bias, int T, int E, int topk,
                               int32_t* idx, float* weight, cudaStream_t st) {
  router_topk_kernel<<<(T + 7) / 8, 256, 0, st>>>(logits, bias, T, E, topk, idx, weight);
  return cudaGetLastError();
}

cudaError_t launch_route_decode(const uint16_t* x, const uint16_t* w, const float* bias, int T, int H,
                                int E, int topk, int R, float* logits, int32_t* idx, float* wts,
                                int32_t* uids, int32_t* urows, int32_t* ucnt, float* uw,
                                int32_t* gidx, int32_t* num_unique, __half* x16, uint8_t* xq, uint8_t* xs,
                                float* score, int32_t* status, cudaStream_t st, int fp4, int32_t* ready,
                                int ready_n) {
  if (T < 1 || T > 8 || T * topk > 64 || E % 16 || H % 256) return cudaErrorInvalidValue;
  const cudaError_t e = launch_k(route_logits_kernel, dim3(E / 4), dim3(kRouteWarps * 32), 0, st, x, w, T, H, E,
                                 logits, score, xq, xs, status, fp4, ready, ready_n);
  if (e != cudaSuccess) return e;
  return launch_k(route_select_kernel, dim3(1), dim3(kRouteWarps * 32), 0, st, x, bias, T, H, E, topk, R, idx, wts,
                  uids, urows, ucnt, uw, gidx, num_unique, x16, score, status);
}

}  // namespace mimo
