// MXFP4 expert products on sm_100a: one persistent, warp-specialised tile kernel serves
//   * decode (1-8 rows): kernel A (gate/up + SwiGLU, engine/mimo_stream/kernels.py:33-85) and
//     kernel B (down x router weight, kernels.py:88-123) over DISTINCT experts, each expert's bytes
//     streamed from HBM exactly once per call;
//   * prefill (> 8 rows): the same tiles over (expert, block of up to 64 routes) units, i.e. the
//     gather_qmm pair products of Engine._pair_outputs (engine/mimo_stream/model.py:221-228).
//
// Work item = (unit, tile of 16 weight rows).  A producer warp streams each item's weight rows and
// e8m0 scales (K in chunks of 2048) into a ring of shared-memory stages with 1-D cp.async.bulk copies
// completing on mbarriers (L2 evict-first: expert bytes are read once).  Eight consumer warps split
// each chunk's K range, decode e2m1 nibbles in registers with the Blackwell cvt.rn.f16x2.e2m1x2
// instruction and run f16 tensor-core MMAs (weights = A, 16 rows; routed tokens = B, 8 per block)
// with float32 accumulation; every 32-element group's product is scaled by its e8m0 scale in float32,
// as the reference applies the scale per group.  A fixed-order cross-warp reduction feeds the
// epilogue (SwiGLU for gate/up; weight / bf16 rounding for down).
//
// Activations enter the MMA as f16: every bf16 value in [2^-14, 65504] is exact in f16; values below
// that range keep 2^-24 absolute resolution; values beyond +-65504 set MIMO_ERANGE.
#include "common.cuh"
#include "kernels.h"

namespace mimo {

constexpr int kRows = 16;   // weight rows per tile (MMA M)
constexpr int kCW = 8;      // consumer warps
constexpr int kThreads = (kCW + 1) * 32;
constexpr int kKC = 2048;   // K elements per pipeline chunk
constexpr int kGPW = kKC / 32 / kCW;  // 32-element groups per consumer warp per chunk (8)
constexpr int kWS = kKC / 2 + 16;     // smem row stride of packed weights (bytes, +16 pad: no conflicts)
constexpr int kSS = kKC / 32 + 16;    // smem row stride of scales (bytes)
constexpr int kMat = kRows * (kWS + kSS);  // one matrix' tile in a stage (17,920 B)
constexpr int kBarBytes = 1024;

template <int NM>
constexpr int stage_bytes() { return NM * kMat; }
template <int NM, int TB, int NSTAGE>
constexpr int smem_bytes() { return kBarBytes + NSTAGE * stage_bytes<NM>() + kCW * NM * TB * 128 * 4; }

// Correctly rounded bf16 sigmoid of a bf16 value (the reference's 64K-entry sigmoid table,
// kernels.py:138-146, defined as bf16(float32(sigmoid)) of the exact sigmoid).  Fast float path;
// when the float result sits within a few ulp of a bf16 rounding tie, recompute in double.
__device__ __forceinline__ float sigmoid_bf16(float xb) {
  const float s = 1.0f / (1.0f + expf(-xb));
  const uint32_t lo = __float_as_uint(s) & 0xFFFFu;
  float sr = s;
  if (lo > 0x7FF0u && lo < 0x8010u) sr = (float)(1.0 / (1.0 + exp(-(double)xb)));
  return bf16_round(sr);
}

// Kernel A epilogue: gt = bf16(g), ut = bf16(u), h = bf16(bf16(gt * sig(gt)) * ut)  (kernels.py:79-82)
__device__ __forceinline__ float swiglu_ref(float g, float u) {
  const float gt = bf16_round(g);
  const float ut = bf16_round(u);
  const float gs = bf16_round(gt * sigmoid_bf16(gt));
  return bf16_round(gs * ut);
}

__device__ __forceinline__ __half to_f16_checked(float v, int32_t* status) {
  if (fabsf(v) > 65504.f && !isnan(v)) {
    set_status(status, MIMO_ERANGE);
    v = copysignf(65504.f, v);
  }
  return __float2half_rn(v);
}

// B-operand row of route q of a unit (MMA column), or null when q is past the unit's routes.
__device__ __forceinline__ const __half* b_row(const ExpertParams& p, int p0, int cnt, int q) {
  if (q >= cnt) return nullptr;
  const int r = p.rtok ? __ldg(p.rtok + p0 + q) : (p0 + q);
  return p.bsrc + (size_t)r * p.K;
}

template <int NM, int TB, int NSTAGE, int MODE>
__global__ void __launch_bounds__(kThreads, 1) expert_tiles_kernel(const ExpertParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + NSTAGE;
  volatile int* s_abort = reinterpret_cast<volatile int*>(empty + NSTAGE);
  uint8_t* stages = smem + kBarBytes;
  float* red = reinterpret_cast<float*>(stages + NSTAGE * stage_bytes<NM>());

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = p.num_units ? min(__ldg(p.num_units), p.units_cap) : p.units_cap;
  const long long items = (long long)units * p.tiles;
  const long long it0 = items * blockIdx.x / gridDim.x;
  const long long it1 = items * (blockIdx.x + 1) / gridDim.x;
  const int nchunks = p.K / kKC;
  const long long nsteps = (it1 - it0) * nchunks;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NSTAGE; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kCW);
    }
    *s_abort = 0;
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kCW) {
    // ------------------------------------------------------------------------------ producer
    const uint64_t pol = l2_evict_first_policy();
    int stage = 0;
    uint32_t ph = 0;
    long long issued = 0;
    for (long long s = 0; s < nsteps; ++s) {
      const long long item = it0 + s / nchunks;
      const int c = (int)(s % nchunks);
      const int unit = (int)(item / p.tiles), tile = (int)(item % p.tiles);
      int slot = __ldg(p.unit_slot + unit);
      if (slot < 0 || slot >= p.S) {
        if (lane == 0 && c == 0) set_status(p.status, MIMO_ERANGE);
        slot = 0;  // keep the pipeline in step; consumers discard this item
      }
      if (*s_abort) break;
      if (!mbar_wait(&empty[stage], ph ^ 1u)) {
        if (lane == 0) set_status(p.status, MIMO_ETIMEOUT);
        *s_abort = 1;
        break;
      }
      if (lane == 0) mbar_arrive_expect_tx(&full[stage], NM * kRows * (kKC / 2 + kKC / 32));
      __syncwarp();
      uint8_t* sb = stages + stage * stage_bytes<NM>();
      for (int ci = lane; ci < NM * 2 * kRows; ci += 32) {
        const int m = ci / (2 * kRows), kind = (ci / kRows) & 1, row = ci % kRows;
        const size_t grow = (size_t)slot * p.N + (size_t)tile * kRows + row;
        uint8_t* mb = sb + m * kMat;
        if (kind == 0)
          bulk_g2s(mb + row * kWS, p.w[m] + grow * (p.K / 2) + (size_t)c * (kKC / 2), kKC / 2,
                   &full[stage], pol);
        else
          bulk_g2s(mb + kRows * kWS + row * kSS, p.s[m] + grow * (p.K / 32) + (size_t)c * (kKC / 32),
                   kKC / 32, &full[stage], pol);
      }
      ++issued;
      if (++stage == NSTAGE) {
        stage = 0;
        ph ^= 1u;
      }
    }
    // Drain: never leave the CTA with bulk copies in flight (matters only after an abort).
    const long long tail = issued < NSTAGE ? issued : NSTAGE;
    for (long long k = 0; k < tail; ++k) {
      const long long f = issued - 1 - k;
      const int st = (int)(f % NSTAGE);
      const uint32_t par = (uint32_t)((f / NSTAGE) & 1);
      if (!mbar_wait(&full[st], par)) {
        if (lane == 0) set_status(p.status, MIMO_ETIMEOUT);
        break;
      }
    }
    return;
  }

  // -------------------------------------------------------------------------------- consumers
  const int g = lane >> 2, t = lane & 3;
  const int tid = threadIdx.x;
  int stage = 0;
  uint32_t ph = 0;
  bool aborted = false;

  int unit = -1, tile = 0, slot = 0, p0 = 0, cnt = 0;
  const __half* brow[TB];
  float acc[NM][TB][4];
  uint4 bcur[kGPW], bnext[kGPW];  // TB == 1: B of the whole chunk, prefetched one step ahead

  auto step_brow = [&](long long s) -> const __half* {  // TB == 1 prefetch helper
    const long long item = it0 + s / nchunks;
    const int un = (int)(item / p.tiles);
    const int q0 = p.unit_p0 ? __ldg(p.unit_p0 + un) : un * p.p0_stride;
    const int cn = min(__ldg(p.unit_cnt + un), 8);
    return b_row(p, q0, cn, g);
  };
  auto load_chunk = [&](const __half* br, int c, uint4 (&dst)[kGPW]) {
#pragma unroll
    for (int jj = 0; jj < kGPW; ++jj) {
      const int kk = c * kKC + (warp * kGPW + jj) * 32 + t * 8;
      dst[jj] = br ? ldg_nc_v4(br + kk) : make_uint4(0u, 0u, 0u, 0u);
    }
  };

  if constexpr (TB == 1) {
    if (nsteps > 0) load_chunk(step_brow(0), 0, bcur);
  }

  for (long long s = 0; s < nsteps; ++s) {
    const long long item = it0 + s / nchunks;
    const int c = (int)(s % nchunks);
    if (c == 0) {
      unit = (int)(item / p.tiles);
      tile = (int)(item % p.tiles);
      slot = __ldg(p.unit_slot + unit);
      p0 = p.unit_p0 ? __ldg(p.unit_p0 + unit) : unit * p.p0_stride;
      cnt = min(__ldg(p.unit_cnt + unit), TB * 8);
#pragma unroll
      for (int b = 0; b < TB; ++b) brow[b] = b_row(p, p0, cnt, b * 8 + g);
#pragma unroll
      for (int m = 0; m < NM; ++m)
#pragma unroll
        for (int b = 0; b < TB; ++b)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[m][b][i] = 0.f;
    }
    if constexpr (TB == 1) {
      if (s + 1 < nsteps) load_chunk(step_brow(s + 1), (int)((s + 1) % nchunks), bnext);
    }
    if (!aborted && !mbar_wait(&full[stage], ph)) {
      aborted = true;
      set_status(p.status, MIMO_ETIMEOUT);
      *s_abort = 1;
    }
    if (!aborted) {
      const uint8_t* sb = stages + stage * stage_bytes<NM>();
      uint4 bv[TB], bvn[TB];
      if constexpr (TB > 1) {
#pragma unroll
        for (int b = 0; b < TB; ++b) {
          const int kk = c * kKC + (warp * kGPW) * 32 + t * 8;
          bv[b] = brow[b] ? ldg_nc_v4(brow[b] + kk) : make_uint4(0u, 0u, 0u, 0u);
        }
      }
#pragma unroll
      for (int jj = 0; jj < kGPW; ++jj) {
        const int j = warp * kGPW + jj;
        if constexpr (TB == 1) {
          bv[0] = bcur[jj];
        } else {
          if (jj + 1 < kGPW) {
#pragma unroll
            for (int b = 0; b < TB; ++b) {
              const int kk = c * kKC + (j + 1) * 32 + t * 8;
              bvn[b] = brow[b] ? ldg_nc_v4(brow[b] + kk) : make_uint4(0u, 0u, 0u, 0u);
            }
          }
        }
#pragma unroll
        for (int m = 0; m < NM; ++m) {
          const uint8_t* mb = sb + m * kMat;
          const uint32_t w0 = *reinterpret_cast<const uint32_t*>(mb + g * kWS + j * 16 + t * 4);
          const uint32_t w1 = *reinterpret_cast<const uint32_t*>(mb + (g + 8) * kWS + j * 16 + t * 4);
          const float sc0 = e8m0_to_f32(mb[kRows * kWS + g * kSS + j]);
          const float sc1 = e8m0_to_f32(mb[kRows * kWS + (g + 8) * kSS + j]);
          uint32_t ra[4], rb[4];
          e2m1x8_to_f16x2(w0, ra);
          e2m1x8_to_f16x2(w1, rb);
#pragma unroll
          for (int b = 0; b < TB; ++b) {
            float tmp[4];
            const float z[4] = {0.f, 0.f, 0.f, 0.f};
            mma_16816(tmp, ra[0], rb[0], ra[1], rb[1], bv[b].x, bv[b].y, z);
            mma_16816(tmp, ra[2], rb[2], ra[3], rb[3], bv[b].z, bv[b].w, tmp);
            acc[m][b][0] = fmaf(tmp[0], sc0, acc[m][b][0]);
            acc[m][b][1] = fmaf(tmp[1], sc0, acc[m][b][1]);
            acc[m][b][2] = fmaf(tmp[2], sc1, acc[m][b][2]);
            acc[m][b][3] = fmaf(tmp[3], sc1, acc[m][b][3]);
          }
        }
        if constexpr (TB > 1) {
#pragma unroll
          for (int b = 0; b < TB; ++b) bv[b] = bvn[b];
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == NSTAGE) {
      stage = 0;
      ph ^= 1u;
    }
    if constexpr (TB == 1) {
#pragma unroll
      for (int jj = 0; jj < kGPW; ++jj) bcur[jj] = bnext[jj];
    }

    if (c == nchunks - 1) {
      // fixed-order cross-warp reduction, then the epilogue
      float* rw_ = red + warp * (NM * TB * 128);
#pragma unroll
      for (int m = 0; m < NM; ++m)
#pragma unroll
        for (int b = 0; b < TB; ++b) {
          float* r = rw_ + (m * TB + b) * 128;
          r[g * 8 + 2 * t] = acc[m][b][0];
          r[g * 8 + 2 * t + 1] = acc[m][b][1];
          r[(g + 8) * 8 + 2 * t] = acc[m][b][2];
          r[(g + 8) * 8 + 2 * t + 1] = acc[m][b][3];
        }
      named_bar_sync(1, kCW * 32);
      const bool bad = (slot < 0 || slot >= p.S);
      if (!aborted && !bad) {
        for (int o = tid; o < kRows * 8 * TB; o += kCW * 32) {
          const int row = o % kRows, q = o / kRows;  // q = route within unit (block q/8, column q%8)
          if (q < cnt) {
            const int b = q >> 3, col = q & 7;
            float v[NM];
#pragma unroll
            for (int m = 0; m < NM; ++m) {
              float sum = 0.f;
#pragma unroll
              for (int w = 0; w < kCW; ++w) sum += red[w * (NM * TB * 128) + (m * TB + b) * 128 + row * 8 + col];
              v[m] = sum;
            }
            const size_t op = (size_t)(p0 + q) * p.N + (size_t)tile * kRows + row;
            if constexpr (MODE == 0) {
              p.h_out[op] = to_f16_checked(swiglu_ref(v[0], v[NM - 1]), p.status);
            } else if constexpr (MODE == 1) {
              const float d = p.pairs_rounding ? bf16_round(v[0]) : v[0];
              p.part_out[op] = d * __ldg(p.rw + p0 + q);
            } else {
              p.ypair_out[op] = (uint16_t)f32_to_bf16(v[0]);
            }
          }
        }
      }
      named_bar_sync(1, kCW * 32);
    }
  }
}

template <int NM, int TB, int NSTAGE, int MODE>
static cudaError_t launch_tiles(const ExpertParams& p, int grid, cudaStream_t st) {
  auto kfn = expert_tiles_kernel<NM, TB, NSTAGE, MODE>;
  constexpr int smem = smem_bytes<NM, TB, NSTAGE>();
  static_assert(smem <= 232448, "shared memory budget");
  cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kfn<<<grid, kThreads, smem, st>>>(p);
  return cudaGetLastError();
}

// x (bf16) -> f16 B-operand rows, with the f16 range check.
__global__ void to_f16_kernel(const uint16_t* __restrict__ x, __half* __restrict__ y, size_t n,
                              int32_t* status) {
  const size_t i = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (i >= n) return;
  const uint4 v = *reinterpret_cast<const uint4*>(x + i);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const __half lo = to_f16_checked(__uint_as_float(w[k] << 16), status);
    const __half hi = to_f16_checked(__uint_as_float(w[k] & 0xFFFF0000u), status);
    o[k] = (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
  }
  *reinterpret_cast<uint4*>(y + i) = make_uint4(o[0], o[1], o[2], o[3]);
}

cudaError_t launch_to_f16(const uint16_t* x, __half* y, size_t n, int32_t* status, cudaStream_t st) {
  const size_t threads = (n + 7) / 8;
  to_f16_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(x, y, n, status);
  return cudaGetLastError();
}

cudaError_t launch_expert_tiles(const ExpertParams& p, int kind, int num_sms, cudaStream_t st) {
  switch (kind) {
    case 0: return launch_tiles<2, 1, 5, 0>(p, num_sms, st);   // decode gate/up
    case 1: return launch_tiles<1, 1, 11, 1>(p, num_sms, st);  // decode down
    case 2: return launch_tiles<2, 8, 4, 0>(p, num_sms, st);   // prefill gate/up
    case 3: return launch_tiles<1, 8, 9, 2>(p, num_sms, st);   // prefill down
    default: return cudaErrorInvalidValue;
  }
}

// ------------------------------------------------------------------------------------ combine
// Decode (kernels.py:196-199): y[t, m] = bf16(sum_k part[gidx[t, k], m]) in route order; with
// gidx == null, the scatter-add of kernels.py:196-197 summed in (u, r) order.
__global__ void combine_decode_kernel(const float* __restrict__ part, const int32_t* __restrict__ gidx,
                                      const int32_t* __restrict__ urows, const int32_t* __restrict__ ucnt,
                                      const int32_t* __restrict__ num_unique, int ucap, int R, int M,
                                      int topk, int H, uint16_t* __restrict__ y) {
  const int t = blockIdx.y;
  const int m = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (t >= M || m >= H) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  auto add = [&](int slot) {
    const float4 v = *reinterpret_cast<const float4*>(part + (size_t)slot * H + m);
    acc.x = __fadd_rn(acc.x, v.x);
    acc.y = __fadd_rn(acc.y, v.y);
    acc.z = __fadd_rn(acc.z, v.z);
    acc.w = __fadd_rn(acc.w, v.w);
  };
  if (gidx) {
    for (int k = 0; k < topk; ++k) {
      const int sl = gidx[t * topk + k];
      if (sl >= 0) add(sl);
    }
  } else {
    const int U = num_unique ? min(*num_unique, ucap) : ucap;
    for (int u = 0; u < U; ++u) {
      const int n = min(ucnt[u], R);
      for (int r = 0; r < n; ++r)
        if (urows[u * R + r] == t) add(u * R + r);
    }
  }
  const uint32_t o0 = f32_to_bf16(acc.x) | (f32_to_bf16(acc.y) << 16);
  const uint32_t o1 = f32_to_bf16(acc.z) | (f32_to_bf16(acc.w) << 16);
  *reinterpret_cast<uint2*>(y + (size_t)t * H + m) = make_uint2(o0, o1);
}

cudaError_t launch_combine_decode(const float* part, const int32_t* gidx, const int32_t* urows,
                                  const int32_t* ucnt, const int32_t* num_unique, int ucap, int R,
                                  int M, int topk, int H, uint16_t* y, cudaStream_t st) {
  dim3 grid((H / 4 + 255) / 256, M);
  combine_decode_kernel<<<grid, 256, 0, st>>>(part, gidx, urows, ucnt, num_unique, ucap, R, M, topk, H,
                                              y);
  return cudaGetLastError();
}

// Prefill (model.py:266-271): y[t, m] = bf16(sum_k fp32(ypair[inv[t, k], m]) * w[t, k]) in k order.
__global__ void combine_prefill_kernel(const uint16_t* __restrict__ ypair, const int32_t* __restrict__ inv,
                                       const float* __restrict__ w, int T, int topk, int H,
                                       uint16_t* __restrict__ y) {
  const int t = blockIdx.y;
  const int m = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (t >= T || m >= H) return;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int k = 0; k < topk; ++k) {
    const int pos = inv[t * topk + k];
    if (pos < 0) continue;
    const float wk = w[t * topk + k];
    const uint4 v = *reinterpret_cast<const uint4*>(ypair + (size_t)pos * H + m);
    const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc[2 * i] = __fadd_rn(acc[2 * i], __fmul_rn(__uint_as_float(vv[i] << 16), wk));
      acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], __fmul_rn(__uint_as_float(vv[i] & 0xFFFF0000u), wk));
    }
  }
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = f32_to_bf16(acc[2 * i]) | (f32_to_bf16(acc[2 * i + 1]) << 16);
  *reinterpret_cast<uint4*>(y + (size_t)t * H + m) = make_uint4(o[0], o[1], o[2], o[3]);
}

cudaError_t launch_combine_prefill(const uint16_t* ypair, const int32_t* inv, const float* w, int T,
                                   int topk, int H, uint16_t* y, cudaStream_t st) {
  dim3 grid((H / 8 + 255) / 256, T);
  combine_prefill_kernel<<<grid, 256, 0, st>>>(ypair, inv, w, T, topk, H, y);
  return cudaGetLastError();
}

}  // namespace mimo
