// Dispatch: decode route grouping (group_routes, engine/mimo_stream/kernels.py:149-173) and the
// prefill stable token->expert permutation (engine/mimo_stream/model.py:235-244, 266-268).
#include "common.cuh"
#include "kernels.h"
#include "route_dev.cuh"

namespace mimo {

// ------------------------------------------------------------------------------ decode grouping
// One CTA, one thread per route t (P = M*topk <= 1024); see group_routes_cta.
__global__ void __launch_bounds__(1024) group_routes_kernel(
    const int32_t* __restrict__ idx, const float* __restrict__ weight, int P, int topk, int R, int E,
    int ucap, int32_t* __restrict__ uids, int32_t* __restrict__ urows, int32_t* __restrict__ ucnt,
    float* __restrict__ uw, int32_t* __restrict__ gidx, int32_t* __restrict__ num_unique,
    int32_t* status) {
  __shared__ uint32_t bitmap[32];  // E <= 1024
  __shared__ int32_t sid[1024];
  group_routes_cta(idx, weight, P, topk, R, E, ucap, uids, urows, ucnt, uw, gidx, num_unique, status, sid,
                   bitmap);
}

cudaError_t launch_group_routes(const int32_t* idx, const float* weight, int M, int topk, int R,
                                int E, int32_t* uids, int32_t* urows, int32_t* ucnt, float* uw,
                                int32_t* gidx, int32_t* num_unique, int32_t* status,
                                cudaStream_t st) {
  const int P = M * topk;
  const int ucap = min(E, P);
  const int threads = max(32, ((P + 31) / 32) * 32);
  group_routes_kernel<<<1, threads, 0, st>>>(idx, weight, P, topk, R, E, ucap, uids, urows, ucnt, uw,
                                             gidx, num_unique, status);
  return cudaGetLastError();
}

// ----------------------------------------------------------------------------- prefill dispatch
constexpr int kChunk = 2048;  // routes per CTA
constexpr int kDispThreads = 256;

__global__ void __launch_bounds__(kDispThreads) dispatch_count_kernel(const int32_t* __restrict__ idx,
                                                                      int P, int E,
                                                                      int32_t* __restrict__ chunk_counts,
                                                                      int id_base, int skip_outside,
                                                                      int32_t* status) {
  extern __shared__ int32_t hist[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int base = blockIdx.x * kChunk;
  for (int i = threadIdx.x; i < kChunk; i += blockDim.x) {
    const int p = base + i;
    if (p < P) {
      const int id = idx[p] - id_base;
      if (id >= 0 && id < E)
        atomicAdd(&hist[id], 1);
      else if (!skip_outside)
        set_status(status, MIMO_ERANGE);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) chunk_counts[(size_t)blockIdx.x * E + e] = hist[e];
}

// One CTA: per expert e (thread), running prefix over chunks; then an exclusive scan over experts.
__global__ void __launch_bounds__(1024) dispatch_scan_kernel(int32_t* __restrict__ chunk_counts,
                                                             int nchunks, int E,
                                                             int32_t* __restrict__ offsets) {
  __shared__ int32_t tot[1024];
  const int e = threadIdx.x;
  int run = 0;
  if (e < E) {
    for (int c = 0; c < nchunks; ++c) {
      const int v = chunk_counts[(size_t)c * E + e];
      chunk_counts[(size_t)c * E + e] = run;
      run += v;
    }
  }
  tot[e] = (e < E) ? run : 0;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {  // Hillis-Steele inclusive scan
    const int v = (e >= o) ? tot[e - o] : 0;
    __syncthreads();
    tot[e] += v;
    __syncthreads();
  }
  const int excl = tot[e] - ((e < E) ? run : 0);
  if (e < E) {
    offsets[e] = excl;
    for (int c = 0; c < nchunks; ++c) chunk_counts[(size_t)c * E + e] += excl;
  }
  if (e == E - 1) offsets[E] = tot[e];
}

// Stable scatter: warp w of chunk c owns routes [c*kChunk + w*256, +256) and walks them in order in
// batches of 32; ranks within a batch come from __match_any_sync, ranks across warps from a per-warp
// count table.
__global__ void __launch_bounds__(kDispThreads) dispatch_scatter_kernel(
    const int32_t* __restrict__ idx, int P, int E, const int32_t* __restrict__ chunk_base,
    int32_t* __restrict__ order, int32_t* __restrict__ inv, int id_base) {
  extern __shared__ int32_t sm[];
  constexpr int kWarps = kDispThreads / 32;
  constexpr int kPerWarp = kChunk / kWarps;  // 256
  int32_t* wcnt = sm;                        // [kWarps][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kWarps * E; i += blockDim.x) wcnt[i] = 0;
  __syncthreads();
  const int wbase = blockIdx.x * kChunk + warp * kPerWarp;
  const unsigned lt = (1u << lane) - 1u;
  for (int b = 0; b < kPerWarp; b += 32) {
    const int p = wbase + b + lane;
    int id = (p < P) ? idx[p] - id_base : -1;
    if (id >= E || id < 0) id = -1;
    const unsigned peers = __match_any_sync(0xFFFFFFFFu, id);
    if (id >= 0 && (peers & lt) == 0u) wcnt[warp * E + id] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = chunk_base[(size_t)blockIdx.x * E + e];
    for (int w = 0; w < kWarps; ++w) {
      const int v = wcnt[w * E + e];
      wcnt[w * E + e] = run;
      run += v;
    }
  }
  __syncthreads();
  for (int b = 0; b < kPerWarp; b += 32) {
    const int p = wbase + b + lane;
    int id = (p < P) ? idx[p] - id_base : -1;
    if (id >= E || id < 0) id = -1;
    const unsigned peers = __match_any_sync(0xFFFFFFFFu, id);
    int pos = -1;
    if (id >= 0) pos = wcnt[warp * E + id] + __popc(peers & lt);
    __syncwarp();
    if (id >= 0 && (peers & lt) == 0u) wcnt[warp * E + id] += __popc(peers);
    __syncwarp();
    if (p < P) {
      inv[p] = pos;
      if (pos >= 0) order[pos] = p;
    }
  }
}

size_t dispatch_workspace_bytes(int P, int E) {
  const int nchunks = (P + kChunk - 1) / kChunk;
  return (size_t)std::max(nchunks, 1) * E * sizeof(int32_t);
}

cudaError_t launch_dispatch(const int32_t* idx, int P, int E, int32_t* offsets, int32_t* order,
                            int32_t* inv, void* ws, int32_t* status, cudaStream_t st, int id_base,
                            int skip_outside) {
  const int nchunks = std::max(1, (P + kChunk - 1) / kChunk);
  int32_t* cc = static_cast<int32_t*>(ws);
  dispatch_count_kernel<<<nchunks, kDispThreads, E * sizeof(int32_t), st>>>(idx, P, E, cc, id_base,
                                                                             skip_outside, status);
  dispatch_scan_kernel<<<1, 1024, 0, st>>>(cc, nchunks, E, offsets);
  dispatch_scatter_kernel<<<nchunks, kDispThreads, (kDispThreads / 32) * E * sizeof(int32_t), st>>>(
      idx, P, E, cc, order, inv, id_base);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------- prefill work units
// Unit = (pool slot, first sorted route, count <= unit_max): an expert's bucket split into blocks of
// at most unit_max routes.
__global__ void __launch_bounds__(1024) build_units_kernel(
    const int32_t* __restrict__ offsets, const int32_t* __restrict__ slot_of, int E, int S,
    int unit_max, int ucap, int32_t* __restrict__ unit_slot, int32_t* __restrict__ unit_p0,
    int32_t* __restrict__ unit_cnt, int32_t* __restrict__ unit_first, int32_t* __restrict__ unit_nsub,
    int32_t* __restrict__ num_units, int32_t* status) {
  __shared__ int32_t nu[1024];
  const int e = threadIdx.x;
  int n = 0, c = 0, o0 = 0;
  if (e < E) {
    o0 = offsets[e];
    c = offsets[e + 1] - o0;
    n = (c + unit_max - 1) / unit_max;
  }
  nu[e] = n;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    const int v = (e >= o) ? nu[e - o] : 0;
    __syncthreads();
    nu[e] += v;
    __syncthreads();
  }
  const int first = nu[e] - n;
  if (e < E && n > 0) {
    int slot = slot_of ? slot_of[e] : e;
    if (slot < 0 || slot >= S) {
      set_status(status, MIMO_ERANGE);
      slot = -1;
    }
    for (int g = 0; g < n && first + g < ucap; ++g) {
      unit_slot[first + g] = slot;
      unit_p0[first + g] = o0 + g * unit_max;
      unit_cnt[first + g] = min(unit_max, c - g * unit_max);
      if (unit_first) {  // groups cut by ucap keep only their stored units
        unit_first[first + g] = first;
        unit_nsub[first + g] = min(n, ucap - first);
      }
    }
  }
  if (e == 1023) num_units[0] = min(nu[1023], ucap);
}

// Per sorted route position i: token row and router weight of the pair order[i] (route_row given:
// the row is route_row[pair]; weight null: 1).
__global__ void route_rows_kernel(const int32_t* __restrict__ order, const float* __restrict__ weight,
                                  const int32_t* __restrict__ offsets, int E, int P, int topk,
                                  const int32_t* __restrict__ route_row, int32_t* __restrict__ rtok,
                                  float* __restrict__ rw) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < P && i < offsets[E]) {  // positions past offsets[E] belong to dropped (invalid) routes
    const int p = order[i];
    rtok[i] = route_row ? route_row[p] : p / topk;
    rw[i] = weight ? weight[p] : 1.f;
  }
}

cudaError_t launch_build_units(const int32_t* offsets, const int32_t* slot_of, int E, int S,
                               int unit_max, int ucap, int32_t* unit_slot, int32_t* unit_p0,
                               int32_t* unit_cnt, int32_t* unit_first, int32_t* unit_nsub,
                               int32_t* num_units, const int32_t* order,
                               const float* weight, int P, int topk, int32_t* rtok, float* rw,
                               int32_t* status, cudaStream_t st, const int32_t* route_row) {
  build_units_kernel<<<1, 1024, 0, st>>>(offsets, slot_of, E, S, unit_max, ucap, unit_slot, unit_p0,
                                         unit_cnt, unit_first, unit_nsub, num_units, status);
  route_rows_kernel<<<(P + 255) / 256, 256, 0, st>>>(order, weight, offsets, E, P, topk, route_row, rtok, rw);
  return cudaGetLastError();
}

}  // namespace mimo
