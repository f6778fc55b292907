// Expert-parallel prefill exchange plan: routes to their expert's rank.
//
// The reference runs every expert on one device (engine/mimo_stream/model.py:230-271: the stable
// token -> expert permutation, per-pair products, weighted combine); expert parallelism adds the move
// of each route to the rank that owns its expert.  Rank d owns experts [d * per_rank, (d + 1) *
// per_rank).  A rank's P = T * topk routes are ordered stably by destination rank (route order kept
// within a destination); a destination's routes of one token are then adjacent, so each token row is
// sent once per destination that owns any of its experts, and every route carries (row within its
// destination's rows, local expert id).
//
//   counts[d]   = (routes to d, rows to d)                      int64 [world][2]
//   order[s]    = route (t * topk + j) at send position s        int32 [P]
//   inv[p]      = send position of route p (-1: expert id out of range, MIMO_ERANGE)
//   send_tok[r] = token of send row r (rows of destination 0 first) int32 [P]; rows = sum counts[:, 1]
//   send_tag[s] = (row within the destination's rows, expert id - d * per_rank)   int32 [P][2]
//
// Kernels: per 1024-token chunk, each thread counts its token's routes per destination (count), one
// CTA scans the chunk totals into per-destination bases (scan), and each chunk writes its tokens'
// positions from block-wide exclusive scans (scatter).  The receiving rank then finds each received
// route's row among the received rows (ep_recv_index); send rows are gathered by gather_rows.
#include "common.cuh"
#include "kernels.h"

namespace mimo {

namespace ep {
constexpr int kTok = 1024;  // tokens per chunk = threads per CTA
constexpr int kMaxWorld = 8;
constexpr int kMaxTopk = 16;

// Destination of expert id e (-1 when e is outside [0, world * per_rank)).
__device__ __forceinline__ int dest_of(int e, int per_rank, int world) {
  return (e >= 0 && e < per_rank * world) ? e / per_rank : -1;
}

// The token's routes per destination: route counts packed 8 bits per destination (topk <= 16 fits),
// two 32-bit words for 8 destinations.
struct TokCounts {
  uint32_t w[2];
  __device__ int get(int d) const { return (w[d >> 2] >> ((d & 3) * 8)) & 0xFF; }
  __device__ void add(int d) { w[d >> 2] += 1u << ((d & 3) * 8); }
};

__device__ __forceinline__ TokCounts token_counts(const int32_t* __restrict__ idx, int t, int T, int topk,
                                                  int per_rank, int world, int32_t* status) {
  TokCounts c{{0u, 0u}};
  if (t >= T) return c;
  for (int j = 0; j < topk; ++j) {
    const int d = dest_of(__ldg(idx + (size_t)t * topk + j), per_rank, world);
    if (d < 0) set_status(status, MIMO_ERANGE);
    else c.add(d);
  }
  return c;
}

// Block-wide exclusive scan of v over the CTA's threads (kTok); returns the exclusive prefix and sets
// total.  `sh` holds kTok / 32 ints.
__device__ __forceinline__ int block_excl_scan(int v, int* sh, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sh[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int s = lane < kTok / 32 ? sh[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < kTok / 32) sh[lane] = s;  // inclusive warp totals
  }
  __syncthreads();
  total = sh[kTok / 32 - 1];
  const int before = warp > 0 ? sh[warp - 1] : 0;
  __syncthreads();  // sh is reused by the next scan
  return before + x - v;
}
}  // namespace ep

// Per chunk c and destination d: (routes, rows) of the chunk's tokens -> cc[(c * world + d) * 2 + q].
__global__ void __launch_bounds__(ep::kTok) ep_count_kernel(const int32_t* __restrict__ idx, int T, int topk,
                                                           int per_rank, int world, int32_t* __restrict__ cc,
                                                           int32_t* status) {
  __shared__ int tot[2 * ep::kMaxWorld];
  if (threadIdx.x < 2 * ep::kMaxWorld) tot[threadIdx.x] = 0;
  __syncthreads();
  const int t = blockIdx.x * ep::kTok + threadIdx.x;
  const ep::TokCounts c = ep::token_counts(idx, t, T, topk, per_rank, world, status);
  for (int d = 0; d < world; ++d) {
    const int r = c.get(d);
    if (r) {
      atomicAdd(&tot[2 * d], r);
      atomicAdd(&tot[2 * d + 1], 1);
    }
  }
  __syncthreads();
  if (threadIdx.x < 2 * world) cc[(size_t)blockIdx.x * 2 * world + threadIdx.x] = tot[threadIdx.x];
}

// One CTA, thread (d, q): chunk bases within destination d's segment (in place in cc), the totals
// (counts, int64) and the segment starts doff[d][q] (destinations in rank order).
__global__ void ep_scan_kernel(int32_t* __restrict__ cc, int nchunks, int world, int64_t* __restrict__ counts,
                               int32_t* __restrict__ doff) {
  __shared__ int tot[2 * ep::kMaxWorld];
  const int i = threadIdx.x;  // = 2 * d + q
  int run = 0;
  if (i < 2 * world) {
    for (int c = 0; c < nchunks; ++c) {
      const int v = cc[(size_t)c * 2 * world + i];
      cc[(size_t)c * 2 * world + i] = run;
      run += v;
    }
    tot[i] = run;
    counts[i] = run;
  }
  __syncthreads();
  if (i < 2 * world) {
    int off = 0;
    for (int d = 0; d < i / 2; ++d) off += tot[2 * d + (i & 1)];
    doff[i] = off;
  }
}

__global__ void __launch_bounds__(ep::kTok) ep_scatter_kernel(const int32_t* __restrict__ idx, int T, int topk,
                                                             int per_rank, int world,
                                                             const int32_t* __restrict__ cc,
                                                             const int32_t* __restrict__ doff,
                                                             int32_t* __restrict__ order, int32_t* __restrict__ inv,
                                                             int32_t* __restrict__ send_tok,
                                                             int32_t* __restrict__ send_tag) {
  __shared__ int sh[ep::kTok / 32];
  const int t = blockIdx.x * ep::kTok + threadIdx.x;
  const ep::TokCounts c = ep::token_counts(idx, t, T, topk, per_rank, world, nullptr);
  int rpos[ep::kMaxWorld], rowpos[ep::kMaxWorld];  // this token's first route / its row, per destination
#pragma unroll
  for (int d = 0; d < ep::kMaxWorld; ++d) {
    if (d < world) {  // world is uniform over the CTA: every thread takes the same scans
      const int r = c.get(d);
      int tr, tw;
      const int er = ep::block_excl_scan(r, sh, tr);
      const int ew = ep::block_excl_scan(r ? 1 : 0, sh, tw);
      const int* base = cc + ((size_t)blockIdx.x * world + d) * 2;
      rpos[d] = doff[2 * d] + base[0] + er;
      rowpos[d] = base[1] + ew;  // within destination d's rows
      if (r && t < T) send_tok[doff[2 * d + 1] + rowpos[d]] = t;
    }
  }
  if (t >= T) return;
  for (int j = 0; j < topk; ++j) {
    const int p = t * topk + j;
    const int e = __ldg(idx + p);
    const int d = ep::dest_of(e, per_rank, world);
    if (d < 0) {
      inv[p] = -1;
      continue;
    }
    int pos = 0, row = 0;
#pragma unroll
    for (int q = 0; q < ep::kMaxWorld; ++q)
      if (q == d) {  // registers stay registers: no dynamic index
        pos = rpos[q]++;
        row = rowpos[q];
      }
    order[pos] = p;
    inv[p] = pos;
    send_tag[2 * (size_t)pos] = row;
    send_tag[2 * (size_t)pos + 1] = e - d * per_rank;
  }
}

size_t ep_plan_workspace_bytes(int T, int world) {
  const int nchunks = std::max(1, (T + ep::kTok - 1) / ep::kTok);
  return ((size_t)nchunks * 2 * world + 2 * ep::kMaxWorld) * sizeof(int32_t);
}

cudaError_t launch_ep_plan(const int32_t* idx, int T, int topk, int per_rank, int world, int64_t* counts,
                           int32_t* order, int32_t* inv, int32_t* send_tok, int32_t* send_tag, void* ws,
                           int32_t* status, cudaStream_t st) {
  if (T < 1 || topk < 1 || topk > ep::kMaxTopk || world < 1 || world > ep::kMaxWorld || per_rank < 1)
    return cudaErrorInvalidValue;
  const int nchunks = (T + ep::kTok - 1) / ep::kTok;
  int32_t* cc = static_cast<int32_t*>(ws);
  int32_t* doff = cc + (size_t)nchunks * 2 * world;
  ep_count_kernel<<<nchunks, ep::kTok, 0, st>>>(idx, T, topk, per_rank, world, cc, status);
  ep_scan_kernel<<<1, 32, 0, st>>>(cc, nchunks, world, counts, doff);
  ep_scatter_kernel<<<nchunks, ep::kTok, 0, st>>>(idx, T, topk, per_rank, world, cc, doff, order, inv, send_tok,
                                                  send_tag);
  return cudaGetLastError();
}

// out[r] = x[rows[r]] (bf16 rows of H values, 16-byte copies); a row index outside [0, x_rows) sets
// MIMO_ERANGE and writes a zero row.
__global__ void __launch_bounds__(256) gather_rows_kernel(const uint16_t* __restrict__ x, long long x_rows, int H,
                                                          const int32_t* __restrict__ rows,
                                                          uint16_t* __restrict__ out, int32_t* status) {
  const long long r = blockIdx.x;
  const int src = __ldg(rows + r);
  const bool ok = src >= 0 && src < x_rows;
  if (!ok && threadIdx.x == 0) set_status(status, MIMO_ERANGE);
  const uint4* s = reinterpret_cast<const uint4*>(x + (size_t)(ok ? src : 0) * H);
  uint4* d = reinterpret_cast<uint4*>(out + (size_t)r * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) d[i] = ok ? __ldg(s + i) : make_uint4(0, 0, 0, 0);
}

// Receiving side: received route i came from rank src (the segment of i in the per-rank route counts
// recv_counts[:, 0]) and names row tag[i][0] of the rows received from src (recv_counts[:, 1]):
// route_row[i] = that row's index in the received rows, eid[i] = tag[i][1].  A tag outside the rows
// received from its rank sets MIMO_ERANGE and gives row -1.
__global__ void __launch_bounds__(256) ep_recv_index_kernel(const int32_t* __restrict__ tag,
                                                            const int64_t* __restrict__ recv_counts, int world,
                                                            long long n, int32_t* __restrict__ route_row,
                                                            int32_t* __restrict__ eid, int32_t* status) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  long long route_end = 0, row_base = 0, nrows = 0;
  int src = world;
  for (int s = 0; s < world; ++s) {
    route_end += recv_counts[2 * s];
    if (i < route_end) {
      src = s;
      nrows = recv_counts[2 * s + 1];
      break;
    }
    row_base += recv_counts[2 * s + 1];
  }
  const int t0 = __ldg(tag + 2 * i);
  const bool ok = src < world && t0 >= 0 && t0 < nrows;
  if (!ok) set_status(status, MIMO_ERANGE);
  route_row[i] = ok ? (int32_t)(row_base + t0) : -1;
  eid[i] = __ldg(tag + 2 * i + 1);
}

cudaError_t launch_gather_rows(const uint16_t* x, long long x_rows, int H, const int32_t* rows, long long n,
                               uint16_t* out, int32_t* status, cudaStream_t st) {
  if (n < 0 || n > 0x7FFFFFFFLL || H % 8) return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  gather_rows_kernel<<<(unsigned)n, 256, 0, st>>>(x, x_rows, H, rows, out, status);
  return cudaGetLastError();
}

cudaError_t launch_ep_recv_index(const int32_t* tag, const int64_t* recv_counts, int world, long long n_recv,
                                 int32_t* route_row, int32_t* eid, int32_t* status, cudaStream_t st) {
  if (n_recv < 0 || n_recv > 0x7FFFFFFFLL || world < 1 || world > ep::kMaxWorld) return cudaErrorInvalidValue;
  if (n_recv == 0) return cudaSuccess;
  ep_recv_index_kernel<<<(unsigned)((n_recv + 255) / 256), 256, 0, st>>>(tag, recv_counts, world, n_recv, route_row,
                                                                         eid, status);
  return cudaGetLastError();
}

}  // namespace mimo
