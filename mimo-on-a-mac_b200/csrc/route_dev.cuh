// Device-side routing pieces shared by the stand-alone kernels and the fused decode route kernel:
// warp top-k with the total order of the router (engine/mimo_stream/model.py:60-64) and CTA-wide
// grouping of routes by distinct expert (engine/mimo_stream/kernels.py:149-173).
#pragma once
#include "common.cuh"

namespace mimo {

// Selection key order: larger sel first, ties -> smaller expert id first (NaN mapped to -inf).
__device__ __forceinline__ bool key_better(float a, int ia, float b, int ib) {
  if (a != b) return a > b;
  return ia < ib;
}

// One warp selects the top-k of one token's E <= 256 logits.  s = sigmoid(logit) in double, rounded
// once to float32; sel = s + bias in float32; weights s / (sum + 1e-20) with the float32 sum taken in
// output order.  Logits are read through L2 (they may come from other CTAs of the same kernel).
__device__ __forceinline__ void topk_warp(const float* logits_row, const float* bias, int E, int topk,
                                          int32_t* idx_row, float* w_row) {
  const int lane = threadIdx.x & 31;
  constexpr int kMaxPer = 8;
  const int per = E >> 5;
  float sv[kMaxPer], key[kMaxPer];
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) {
    sv[j] = 0.f;
    key[j] = -INFINITY;
    if (j < per) {
      const int e = lane + 32 * j;
      const double l = (double)__ldcg(logits_row + e);
      const float s = (float)(1.0 / (1.0 + exp(-l)));
      const float sel = s + (bias ? bias[e] : 0.f);
      sv[j] = s;
      key[j] = isnan(sel) ? -INFINITY : sel;
    }
  }
  unsigned taken = 0u;
  float tot = 0.f, my_s = 0.f;
  int my_id = 0;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    if (r < topk) {
      float bk = -INFINITY, bs = 0.f;
      int bid = 0x7FFFFFFF;
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
      tot = __fadd_rn(tot, bs);
      if (lane == r) {
        my_s = bs;
        my_id = bid;
      }
    }
  }
  tot = __fadd_rn(tot, 1e-20f);
  if (lane < topk) {
    idx_row[lane] = my_id;
    w_row[lane] = __fdiv_rn(my_s, tot);
  }
}

// CTA-wide grouping of P <= blockDim.x routes.  sid/bitmap are shared scratch (sid[P], bitmap[32]).
// Distinct ids ascending (bitmap popcount rank); routes of one id in flat (row, k) order.  Pads
// urows/uw of the first ucap ids with zeros like the reference.  Ends with a __syncthreads().
__device__ __forceinline__ void group_routes_cta(const int32_t* idx, const float* weight, int P, int topk,
                                                 int R, int E, int ucap, int32_t* uids, int32_t* urows,
                                                 int32_t* ucnt, float* uw, int32_t* gidx,
                                                 int32_t* num_unique, int32_t* status, int32_t* sid,
                                                 uint32_t* bitmap) {
  const int t = threadIdx.x;
  const int nwords = (E + 31) >> 5;
  if (t < 32) bitmap[t] = 0u;
  for (int i = t; i < ucap * R; i += blockDim.x) {
    urows[i] = 0;
    uw[i] = 0.f;
  }
  for (int i = t; i < ucap; i += blockDim.x) {
    ucnt[i] = 0;
    uids[i] = 0;
  }
  __syncthreads();
  int id = -1;
  if (t < P) {
    id = __ldcg(idx + t);
    if (id < 0 || id >= E) {
      set_status(status, MIMO_ERANGE);
      id = -1;
    } else {
      atomicOr(&bitmap[id >> 5], 1u << (id & 31));
    }
    sid[t] = id;
  }
  __syncthreads();
  if (t < P) {
    if (id >= 0) {
      int u = 0;
      for (int wv = 0; wv < (id >> 5); ++wv) u += __popc(bitmap[wv]);
      u += __popc(bitmap[id >> 5] & ((1u << (id & 31)) - 1u));
      int c = 0, n = 0;
      for (int q = 0; q < P; ++q) {
        const int same = (sid[q] == id);
        c += (q < t) & same;
        n += same;
      }
      if (c == 0) {
        uids[u] = id;
        ucnt[u] = min(n, R);
      }
      if (c >= R) {
        set_status(status, MIMO_ERANGE);
        gidx[t] = -1;
      } else {
        urows[u * R + c] = t / topk;
        uw[u * R + c] = __ldcg(weight + t);
        gidx[t] = u * R + c;
      }
    } else {
      gidx[t] = -1;
    }
  }
  if (t == 0) {
    int U = 0;
    for (int wv = 0; wv < nwords; ++wv) U += __popc(bitmap[wv]);
    num_unique[0] = U;
  }
  __syncthreads();
}

}  // namespace mimo
