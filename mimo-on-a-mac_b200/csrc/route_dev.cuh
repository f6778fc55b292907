// Device-side routing pieces shared by the stand-alone kernels and the fused decode route kernel:
// warp top-k with the total order of the router (engine/mimo_stream/model.py:60-64) and CTA-wide
// grouping of routes by distinct expert (engine/mimo_stream/kernels.py:149-173).
#pragma once
#include "common.cuh"

namespace mimo {

// Selection key order: larger sel first, ties -> smaller expert id first (NaN mapped to -inf).

// s = sigmoid(logit) evaluated in double and rounded once to float32 (the router's score).
__device__ __forceinline__ float sigmoid_score(float logit) {
  return (float)(1.0 / (1.0 + exp(-(double)logit)));
}

// One warp selects the top-k of one token's E <= 256 experts.  s = sigmoid_score(logit);
// sel = s + bias in float32; weights s / (sum + 1e-20) with the float32 sum taken in output order.
// PRE: `row` already holds the scores s (computed by the CTAs that produced the logits); otherwise it
// holds logits.  Rows are read through L2 (they may come from other CTAs of the same kernel).
// idx_s / w_s (optional, e.g. shared memory) receive a copy of the selection.
template <bool PRE>
__device__ __forceinline__ void topk_warp_impl(const float* row, const float* bias, int E, int topk,
                                               int32_t* idx_row, float* w_row, int32_t* idx_s, float* w_s) {
  const int lane = threadIdx.x & 31;
  constexpr int kMaxPer = 8;
  const int per = E >> 5;
  float sv[kMaxPer], key[kMaxPer], bz[kMaxPer];
  // All loads first (independent, so their L2 latencies overlap), then the arithmetic.
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) {
    const int e = lane + 32 * j;
    sv[j] = j < per ? __ldcg(row + e) : 0.f;
    bz[j] = (bias && j < per) ? __ldg(bias + e) : 0.f;
  }
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) {
    key[j] = -INFINITY;
    if (j < per) {
      const float s = PRE ? sv[j] : sigmoid_score(sv[j]);
      const float sel = s + bz[j];
      sv[j] = s;
      key[j] = isnan(sel) ? -INFINITY : sel;
    } else {
      sv[j] = 0.f;
    }
  }
  // Candidate keys as (order-preserving bits of sel, ~id) pairs, so "larger sel, then smaller id" is a
  // lexicographic maximum.  Each lane sorts its 8 candidates once (Batcher's 19-comparator network,
  // descending); a round then takes the warp maximum of the lanes' heads — one redux.sync on the
  // high words and a ballot, a second redux only when heads tie on sel — and the winning lane drops
  // its head.  Same selection order as scanning all candidates every round.
  uint32_t kh[kMaxPer], kl[kMaxPer];
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) {
    const uint32_t u = __float_as_uint(key[j] + 0.0f);  // -0 -> +0: equal keys compare equal
    kh[j] = j < per ? ((u >> 31) ? ~u : (u | 0x80000000u)) : 0u;  // valid keys are > 0 (-inf -> 0x007FFFFF)
    kl[j] = j < per ? ~(uint32_t)(lane + 32 * j) : 0u;
  }
  auto cx = [&](int a, int b) {  // keep the larger key at a
    const bool sw = kh[b] > kh[a] || (kh[b] == kh[a] && kl[b] > kl[a]);
    const uint32_t h = sw ? kh[b] : kh[a], l = sw ? kl[b] : kl[a];
    const float v = sw ? sv[b] : sv[a];
    kh[b] = sw ? kh[a] : kh[b];
    kl[b] = sw ? kl[a] : kl[b];
    sv[b] = sw ? sv[a] : sv[b];
    kh[a] = h;
    kl[a] = l;
    sv[a] = v;
  };
  cx(0, 1); cx(2, 3); cx(4, 5); cx(6, 7);
  cx(0, 2); cx(1, 3); cx(4, 6); cx(5, 7);
  cx(1, 2); cx(5, 6);
  cx(0, 4); cx(1, 5); cx(2, 6); cx(3, 7);
  cx(2, 4); cx(3, 5);
  cx(1, 2); cx(3, 4); cx(5, 6);
  float tot = 0.f, my_s = 0.f;
  int my_id = 0;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    if (r < topk) {
      const uint32_t wh = __reduce_max_sync(0xFFFFFFFFu, kh[0]);
      uint32_t m = __ballot_sync(0xFFFFFFFFu, kh[0] == wh);
      if (__popc(m) > 1) {  // warp-uniform: heads tie on sel, the larger ~id (smaller id) wins
        const uint32_t wl = __reduce_max_sync(0xFFFFFFFFu, kh[0] == wh ? kl[0] : 0u);
        m = __ballot_sync(0xFFFFFFFFu, kh[0] == wh && kl[0] == wl);
      }
      const int owner = __ffs(m) - 1;
      const int bid = (int)~__shfl_sync(0xFFFFFFFFu, kl[0], owner);
      const float bs = __shfl_sync(0xFFFFFFFFu, sv[0], owner);
      if (lane == owner) {
#pragma unroll
        for (int j = 0; j < kMaxPer - 1; ++j) {
          kh[j] = kh[j + 1];
          kl[j] = kl[j + 1];
          sv[j] = sv[j + 1];
        }
        kh[kMaxPer - 1] = 0u;
        kl[kMaxPer - 1] = 0u;
      }
      tot = __fadd_rn(tot, bs);
      if (lane == r) {
        my_s = bs;
        my_id = bid;
      }
    }
  }
  tot = __fadd_rn(tot, 1e-20f);
  if (lane < topk) {
    const float wv = __fdiv_rn(my_s, tot);
    idx_row[lane] = my_id;
    w_row[lane] = wv;
    if (idx_s) {
      idx_s[lane] = my_id;
      w_s[lane] = wv;
    }
  }
}
__device__ __forceinline__ void topk_warp(const float* logits_row, const float* bias, int E, int topk,
                                          int32_t* idx_row, float* w_row) {
  topk_warp_impl<false>(logits_row, bias, E, topk, idx_row, w_row, nullptr, nullptr);
}

// CTA-wide grouping of P <= blockDim.x routes (idx / weight: global or shared memory, written before
// the call's first barrier by this CTA or by an earlier kernel).  sid/bitmap are shared scratch
// (sid[P], bitmap[32]).
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
    id = idx[t];
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
        uw[u * R + c] = weight[t];
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
