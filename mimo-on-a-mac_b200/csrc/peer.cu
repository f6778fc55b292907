// Expert-parallel exchange over NVLink peer memory (one process per GPU, one node).
//
// Buffers shared between the ranks are plain cudaMalloc allocations exported with CUDA IPC (no
// multicast objects): every rank maps every other rank's buffers and stores into them directly.
//   * dispatch: the routing kernel writes each token's packed row [x | top-k ids | weights] into every
//     rank's gather buffer (rows rank * T + t);
//   * return: the down kernel's epilogue writes each route's float32 partial into the owner rank's
//     receive buffer (row t * topk + k), exactly once per route;
//   * a flag barrier between the phases: each rank stores an increasing epoch into slot `rank` of
//     every rank's signal array (release, system scope) and waits, with a time limit, until its own
//     array holds that epoch for every rank (acquire).  Stream order puts the data stores of the
//     preceding kernel before the release.
#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "route_dev.cuh"

namespace mimo {

__device__ __forceinline__ void st_release_sys(int32_t* p, int32_t v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One warp: lane r < world signals rank r and then waits for rank r's signal here.  `epoch` is this
// rank's device counter (the same count of barriers runs on every rank).  Waits give up after
// limit_ns with MIMO_ETIMEOUT; the kernel then returns, so a rank that never arrives costs its peers
// one expired wait, not a hung GPU.
__global__ void peer_barrier_kernel(int32_t* const* signals, int32_t* my_signals, int rank, int world,
                                    int32_t* epoch, uint64_t limit_ns, int32_t* status) {
  const int lane = threadIdx.x;
  const int32_t e = *epoch + 1;
  __syncwarp();
  __threadfence_system();
  if (lane < world) st_release_sys(signals[lane] + rank, e);
  if (lane < world) {
    const uint64_t t0 = global_timer_ns();
    while (ld_acquire_sys(my_signals + lane) < e) {
      if (global_timer_ns() - t0 > limit_ns) {
        set_status(status, MIMO_ETIMEOUT);
        break;
      }
    }
  }
  __syncwarp();
  if (lane == 0) *epoch = e;
}

// Routing + dispatch for T <= 8 tokens: warp t of every CTA selects token t's top-k from its logits
// (exact sigmoid scores, the router's order); the CTAs then write, between them, the packed row of
// every token into every rank's gather buffer at row rank * T + t: ld 32-bit words per row, x (H bf16)
// first, then topk ids and topk weights.
__global__ void __launch_bounds__(256) route_scatter_kernel(const uint16_t* __restrict__ x,
                                                            const float* __restrict__ logits,
                                                            const float* __restrict__ bias, int T, int H,
                                                            int E, int topk, int32_t* const* rows, int ld,
                                                            int rank, int world) {
  __shared__ int32_t s_idx[64];
  __shared__ float s_w[64];
  __shared__ int32_t* s_rows[16];
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x < world) s_rows[threadIdx.x] = rows[threadIdx.x];
  // Every CTA selects all T tokens' routes (8 warps, cheap) and copies its share of the rows.
  if (warp < T) {
    int32_t* di = s_idx + warp * topk;
    float* dw = s_w + warp * topk;
    topk_warp_impl<false>(logits + (size_t)warp * E, bias, E, topk, di, dw, nullptr, nullptr);
  }
  __syncthreads();
  const int hw = H / 2;  // 32-bit words of one bf16 row
  const int words = T * ld;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < words; i += gridDim.x * blockDim.x) {
    const int t = i / ld, c = i - t * ld;
    int32_t v;
    if (c < hw) v = reinterpret_cast<const int32_t*>(x + (size_t)t * H)[c];
    else if (c < hw + topk) v = s_idx[t * topk + (c - hw)];
    else v = __float_as_int(s_w[t * topk + (c - hw - topk)]);
    const size_t off = (size_t)(rank * T + t) * ld + c;
    for (int r = 0; r < world; ++r) s_rows[r][off] = v;
  }
}

// Work units of the routes whose expert is local, for P = rows * topk <= 1024 routes and S <= 256 local
// experts, in one CTA (replaces the general count / scan / scatter / unit passes at decode sizes).
// Route p = r * topk + k reads id idx[r * route_ld + k] and weight w[r * route_ld + k]; local
// expert e = id - base.  Routes of one expert keep their order (warp match + per-warp counts).
__global__ void __launch_bounds__(1024) routes_prep_kernel(const int32_t* __restrict__ idx,
                                                           const float* __restrict__ w, int route_ld,
                                                           int rows, int topk, int base, int S, int unit_max,
                                                           int ucap, int32_t* __restrict__ order,
                                                           int32_t* __restrict__ rtok, float* __restrict__ rw,
                                                           int32_t* __restrict__ unit_slot,
                                                           int32_t* __restrict__ unit_p0,
                                                           int32_t* __restrict__ unit_cnt,
                                                           int32_t* __restrict__ num_units) {
  __shared__ int32_t wcnt[32][256];
  __shared__ int32_t off[256], uoff[256];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int P = rows * topk;
  int e = -1, r = 0, k = 0;
  if (tid < P) {
    r = tid / topk;
    k = tid - r * topk;
    e = idx[(size_t)r * route_ld + k] - base;
    if (e < 0 || e >= S) e = -1;
  }
  for (int i = tid; i < 32 * 256; i += blockDim.x) (&wcnt[0][0])[i] = 0;
  __syncthreads();
  const unsigned peers = __match_any_sync(0xFFFFFFFFu, e);
  const int rank_w = __popc(peers & ((1u << lane) - 1u));
  if (e >= 0 && rank_w == 0) wcnt[warp][e] = __popc(peers);
  __syncthreads();
  int cnt = 0;
  if (tid < S) {  // per expert: exclusive prefix over warps, total count
    for (int ww = 0; ww < 32; ++ww) {
      const int v = wcnt[ww][tid];
      wcnt[ww][tid] = cnt;
      cnt += v;
    }
    off[tid] = cnt;
    uoff[tid] = (cnt + unit_max - 1) / unit_max;
  }
  __syncthreads();
  for (int o = 1; o < 256; o <<= 1) {  // inclusive scans of counts and unit counts (S <= 256)
    int a = 0, b = 0;
    if (tid < S && tid >= o) {
      a = off[tid - o];
      b = uoff[tid - o];
    }
    __syncthreads();
    if (tid < S) {
      off[tid] += a;
      uoff[tid] += b;
    }
    __syncthreads();
  }
  const int nu_e = tid < S ? (cnt + unit_max - 1) / unit_max : 0;
  const int off_e = tid < S ? off[tid] - cnt : 0;   // exclusive start of expert tid
  const int uo_e = tid < S ? uoff[tid] - nu_e : 0;
  __syncthreads();
  if (tid < S) {  // exclusive starts for the scatter below
    off[tid] = off_e;
    uoff[tid] = uo_e;
  }
  __syncthreads();
  if (e >= 0) {
    const int pos = off[e] + wcnt[warp][e] + rank_w;
    order[pos] = tid;
    rtok[pos] = r;
    rw[pos] = w[(size_t)r * route_ld + k];
  }
  if (tid < S) {
    for (int g = 0; g < nu_e && uo_e + g < ucap; ++g) {
      unit_slot[uo_e + g] = tid;
      unit_p0[uo_e + g] = off_e + g * unit_max;
      unit_cnt[uo_e + g] = min(unit_max, cnt - g * unit_max);
    }
  }
  if (tid == S - 1) num_units[0] = min(uo_e + nu_e, ucap);
}

cudaError_t launch_routes_prep(const int32_t* idx, const float* w, int route_ld, int rows, int topk, int base, int S,
                               int unit_max, int ucap, int32_t* order, int32_t* rtok, float* rw, int32_t* unit_slot,
                               int32_t* unit_p0, int32_t* unit_cnt, int32_t* num_units, cudaStream_t st) {
  if (rows * topk > 1024 || S < 1 || S > 256) return cudaErrorInvalidValue;
  routes_prep_kernel<<<1, 1024, 0, st>>>(idx, w, route_ld, rows, topk, base, S, unit_max, ucap, order, rtok, rw,
                                         unit_slot, unit_p0, unit_cnt, num_units);
  return cudaGetLastError();
}

cudaError_t launch_peer_barrier(int32_t* const* signals, int32_t* my_signals, int rank, int world, int32_t* epoch,
                                uint64_t limit_ns, int32_t* status, cudaStream_t st) {
  if (world < 1 || world > 32) return cudaErrorInvalidValue;
  peer_barrier_kernel<<<1, 32, 0, st>>>(signals, my_signals, rank, world, epoch, limit_ns, status);
  return cudaGetLastError();
}

cudaError_t launch_route_scatter(const uint16_t* x, const float* logits, const float* bias, int T, int H, int E,
                                 int topk, int32_t* const* rows, int ld, int rank, int world, cudaStream_t st) {
  if (T < 1 || T > 8 || topk > 8 || world < 1 || world > 16 || ld < H / 2 + 2 * topk) return cudaErrorInvalidValue;
  route_scatter_kernel<<<16, 256, 0, st>>>(x, logits, bias, T, H, E, topk, rows, ld, rank, world);
  return cudaGetLastError();
}

}  // namespace mimo
