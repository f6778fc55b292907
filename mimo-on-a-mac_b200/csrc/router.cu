// Router: FP32 logits GEMV/GEMM, sigmoid + noaux bias, warp top-k with a total order, normalised
// weights.  Follows Router.__call__ of the reference (engine/mimo_stream/model.py:58-65).
#include "common.cuh"
#include "kernels.h"

namespace mimo {

// logits[t, e] = sum_k f32(x[t,k]) * f32(w[e,k]).  One warp per expert row, 8 tokens per block row.
// Each lane accumulates its 8-element chunks in order (float32 FMA), then a fixed xor-tree reduces the
// lanes, so the result is deterministic for a given (T, H).
__global__ void __launch_bounds__(256) router_logits_kernel(const uint16_t* __restrict__ x,
                                                            const uint16_t* __restrict__ w,
                                                            float* __restrict__ logits, int T, int H,
                                                            int E) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * 8 + warp;
  const int t0 = blockIdx.y * 8;
  if (e >= E) return;
  const int nt = min(8, T - t0);
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  const uint4* wr = reinterpret_cast<const uint4*>(w + (size_t)e * H);
  const int nchunk = H >> 3;
  for (int c = lane; c < nchunk; c += 32) {
    const uint4 wv = __ldg(wr + c);
    float wf[8];
    wf[0] = __uint_as_float(wv.x << 16); wf[1] = __uint_as_float(wv.x & 0xFFFF0000u);
    wf[2] = __uint_as_float(wv.y << 16); wf[3] = __uint_as_float(wv.y & 0xFFFF0000u);
    wf[4] = __uint_as_float(wv.z << 16); wf[5] = __uint_as_float(wv.z & 0xFFFF0000u);
    wf[6] = __uint_as_float(wv.w << 16); wf[7] = __uint_as_float(wv.w & 0xFFFF0000u);
#pragma unroll
    for (int tt = 0; tt < 8; ++tt) {
      if (tt < nt) {
        const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + (size_t)(t0 + tt) * H) + c);
        float a = acc[tt];
        a = fmaf(__uint_as_float(xv.x << 16), wf[0], a);
        a = fmaf(__uint_as_float(xv.x & 0xFFFF0000u), wf[1], a);
        a = fmaf(__uint_as_float(xv.y << 16), wf[2], a);
        a = fmaf(__uint_as_float(xv.y & 0xFFFF0000u), wf[3], a);
        a = fmaf(__uint_as_float(xv.z << 16), wf[4], a);
        a = fmaf(__uint_as_float(xv.z & 0xFFFF0000u), wf[5], a);
        a = fmaf(__uint_as_float(xv.w << 16), wf[6], a);
        a = fmaf(__uint_as_float(xv.w & 0xFFFF0000u), wf[7], a);
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

// Selection key order: larger sel first, ties -> smaller expert id first (NaN was mapped to -inf).
__device__ __forceinline__ bool key_better(float a, int ia, float b, int ib) {
  if (a != b) return a > b;
  return ia < ib;
}

// One warp per token.  s = sigmoid(logit) evaluated in double and rounded once to float32;
// sel = s + bias (float32); top-k by the total order; w_j = s_j / (sum_j s_j + 1e-20) with the sum
// taken in float32 in output order.
__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ logits,
                                                          const float* __restrict__ bias, int T,
                                                          int E, int topk, int32_t* __restrict__ idx,
                                                          float* __restrict__ weight) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= T) return;
  constexpr int kMaxPer = 8;  // E <= 256
  const int per = E >> 5;
  float sv[kMaxPer], key[kMaxPer];
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) {
    sv[j] = 0.f;
    key[j] = -INFINITY;
    if (j < per) {
      const int e = lane + 32 * j;
      const double l = (double)logits[(size_t)t * E + e];
      const float s = (float)(1.0 / (1.0 + exp(-l)));
      const float sel = s + (bias ? bias[e] : 0.f);
      sv[j] = s;
      key[j] = isnan(sel) ? -INFINITY : sel;
    }
  }
  unsigned taken = 0u;
  float chosen_s[8];
  int chosen_id[8];
  for (int r = 0; r < topk; ++r) {
    float bk = -INFINITY;
    int bid = 0x7FFFFFFF;
    float bs = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxPer; ++j) {
      if (j < per && !(taken & (1u << j))) {
        const int e = lane + 32 * j;
        if (bid == 0x7FFFFFFF || key_better(key[j], e, bk, bid)) {
          bk = key[j];
          bid = e;
          bs = sv[j];
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ok = __shfl_xor_sync(0xFFFFFFFFu, bk, o);
      const int oid = __shfl_xor_sync(0xFFFFFFFFu, bid, o);
      const float os = __shfl_xor_sync(0xFFFFFFFFu, bs, o);
      if (oid != 0x7FFFFFFF && (bid == 0x7FFFFFFF || key_better(ok, oid, bk, bid))) {
        bk = ok;
        bid = oid;
        bs = os;
      }
    }
    if ((bid & 31) == lane) taken |= 1u << (bid >> 5);
    chosen_s[r] = bs;
    chosen_id[r] = bid;
  }
  float tot = 0.f;
  for (int r = 0; r < topk; ++r) tot = __fadd_rn(tot, chosen_s[r]);
  tot = __fadd_rn(tot, 1e-20f);
  for (int r = 0; r < topk; ++r) {
    if (lane == r) {
      idx[(size_t)t * topk + r] = chosen_id[r];
      weight[(size_t)t * topk + r] = __fdiv_rn(chosen_s[r], tot);
    }
  }
}

cudaError_t launch_router_logits(const uint16_t* x, const uint16_t* w, float* logits, int T, int H,
                                 int E, cudaStream_t st) {
  dim3 grid((E + 7) / 8, (T + 7) / 8);
  router_logits_kernel<<<grid, 256, 0, st>>>(x, w, logits, T, H, E);
  return cudaGetLastError();
}

cudaError_t launch_router_topk(const float* logits, const float* bias, int T, int E, int topk,
                               int32_t* idx, float* weight, cudaStream_t st) {
  router_topk_kernel<<<(T + 7) / 8, 256, 0, st>>>(logits, bias, T, E, topk, idx, weight);
  return cudaGetLastError();
}

}  // namespace mimo
