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
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"

namespace mimo {

constexpr int kRows = 16;   // weight rows per tile (MMA M)
constexpr int kCW = 8;      // consumer warps
constexpr int kThreads = (kCW + 1) * 32;
constexpr int kBarBytes = 1024;
constexpr int kHdrBytes = 64;  // per-stage header: slot, p0, cnt, tile (written by the producer)

// Shared-memory geometry of one pipeline stage for a K chunk of KC elements.
template <int KC>
struct Geo {
  static constexpr int GPW = KC / 32 / kCW;   // 32-element groups per consumer warp per chunk
  static constexpr int WS = KC / 2 + 16;      // row stride of packed weights (+16 B: conflict-free reads)
  static constexpr int SS = KC / 32 + 16;     // row stride of e8m0 scales
  static constexpr int MAT = kRows * (WS + SS);
  static constexpr int BS = KC * 2 + 64;      // row stride of staged f16 B rows (+64 B: conflict-free)
  static_assert(GPW >= 1 && (KC / 32) % kCW == 0, "chunk must split evenly over the consumer warps");
};

template <int NM, int TB, int KC>
constexpr int stage_bytes() {
  return kHdrBytes + NM * Geo<KC>::MAT + (TB == 1 ? 8 * Geo<KC>::BS : 0);
}
template <int NM, int TB, int NSTAGE, int KC>
constexpr int smem_bytes() {
  return kBarBytes + NSTAGE * stage_bytes<NM, TB, KC>() + kCW * NM * TB * 128 * 4;
}

__device__ __forceinline__ __half to_f16_checked(float v, int32_t* status) {
  if (fabsf(v) > 65504.f && !isnan(v)) {
    set_status(status, MIMO_ERANGE);
    v = copysignf(65504.f, v);
  }
  return __float2half_rn(v);
}

// B-operand row index of route q of a unit.  A row outside [0, brows) (brows > 0) sets MIMO_ERANGE and
// reads row 0 instead, so a bad route table never reads past the activations.
__device__ __forceinline__ int b_row_index(const ExpertParams& p, int p0, int q) {
  int r = p.rtok ? __ldg(p.rtok + p0 + q) : (p0 + q);
  if (p.brows > 0 && (r < 0 || r >= p.brows)) {
    set_status(p.status, MIMO_ERANGE);
    r = 0;
  }
  return r;
}

// Routes a unit may hold: its route slots are [p0, p0 + limit).  Units at a fixed stride (decode:
// p0 = unit * R) hold at most R, so a count above R would write into the next unit's rows.
__device__ __forceinline__ int unit_route_count(const int32_t* unit_cnt, int unit, int limit, int32_t* status) {
  const int c = __ldg(unit_cnt + unit);
  if (c > limit) {
    set_status(status, MIMO_ERANGE);
    return limit;
  }
  return max(c, 0);
}

// Work item decoding shared by producer and consumers.
__device__ __forceinline__ void item_info(const ExpertParams& p, long long item, int& unit, int& tile,
                                          int& slot, int& p0, int& cnt, int tb) {
  unit = (int)(item / p.tiles);
  tile = (int)(item % p.tiles);
  slot = __ldg(p.unit_slot + unit);
  p0 = p.unit_p0 ? __ldg(p.unit_p0 + unit) : unit * p.p0_stride;
  cnt = unit_route_count(p.unit_cnt, unit, p.unit_p0 ? tb * 8 : min(tb * 8, p.p0_stride), p.status);
}

template <int NM, int TB, int NSTAGE, int MODE, int KC>
__global__ void __launch_bounds__(kThreads, 1) expert_tiles_kernel(const ExpertParams p) {
  using G = Geo<KC>;
  constexpr int SB = stage_bytes<NM, TB, KC>();
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + NSTAGE;
  volatile int* s_abort = reinterpret_cast<volatile int*>(empty + NSTAGE);
  uint8_t* stages = smem + kBarBytes;
  float* red = reinterpret_cast<float*>(stages + NSTAGE * SB);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = p.num_units ? min(__ldg(p.num_units), p.units_cap) : p.units_cap;
  const long long items = (long long)units * p.tiles;
  const long long it0 = items * blockIdx.x / gridDim.x;
  const long long it1 = items * (blockIdx.x + 1) / gridDim.x;
  const int nchunks = p.K / KC;
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
    int unit = 0, tile = 0, slot = 0, p0 = 0, cnt = 0, brow = 0;
    for (long long s = 0; s < nsteps; ++s) {
      const long long item = it0 + s / nchunks;
      const int c = (int)(s % nchunks);
      if (c == 0) {
        item_info(p, item, unit, tile, slot, p0, cnt, TB);
        if constexpr (TB == 1) brow = (lane < cnt) ? b_row_index(p, p0, lane) : 0;
      }
      int cslot = slot;
      if (cslot < 0 || cslot >= p.S) {
        if (lane == 0 && c == 0) set_status(p.status, MIMO_ERANGE);
        cslot = 0;  // keep the pipeline in step; consumers discard this item
      }
      if (*s_abort) break;
      if (!mbar_wait(&empty[stage], ph ^ 1u)) {
        if (lane == 0) set_status(p.status, MIMO_ETIMEOUT);
        *s_abort = 1;
        break;
      }
      uint8_t* sb = stages + stage * SB;
      if (lane == 0) {
        int* hdr = reinterpret_cast<int*>(sb);
        hdr[0] = slot;
        hdr[1] = p0;
        hdr[2] = cnt;
        hdr[3] = tile;
        const uint32_t bbytes = (TB == 1) ? (uint32_t)cnt * KC * 2 : 0u;
        mbar_arrive_expect_tx(&full[stage], NM * kRows * (KC / 2 + KC / 32) + bbytes);
      }
      __syncwarp();
      uint8_t* wb = sb + kHdrBytes;
      for (int ci = lane; ci < NM * 2 * kRows; ci += 32) {
        const int m = ci / (2 * kRows), kind = (ci / kRows) & 1, row = ci % kRows;
        const size_t grow = (size_t)cslot * p.N + (size_t)tile * kRows + row;
        uint8_t* mb = wb + m * G::MAT;
        if (kind == 0)
          bulk_g2s(mb + row * G::WS, p.w[m] + grow * (p.K / 2) + (size_t)c * (KC / 2), KC / 2,
                   &full[stage], pol);
        else
          bulk_g2s(mb + kRows * G::WS + row * G::SS, p.s[m] + grow * (p.K / 32) + (size_t)c * (KC / 32),
                   KC / 32, &full[stage], pol);
      }
      if constexpr (TB == 1) {
        if (lane < cnt)
          bulk_g2s_keep(wb + NM * G::MAT + lane * G::BS, p.bsrc + (size_t)brow * p.K + (size_t)c * KC,
                        KC * 2, &full[stage]);
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
  int tile = 0, slot = 0, p0 = 0, cnt = 0;
  const __half* brow[TB];
  float acc[NM][TB][4];

  for (long long s = 0; s < nsteps; ++s) {
    const int c = (int)(s % nchunks);
    if (!aborted && !mbar_wait(&full[stage], ph)) {
      aborted = true;
      set_status(p.status, MIMO_ETIMEOUT);
      *s_abort = 1;
    }
    const uint8_t* sb = stages + stage * SB;
    if (c == 0) {
      if constexpr (TB == 1) {
        const int* hdr = reinterpret_cast<const int*>(sb);
        slot = hdr[0];
        p0 = hdr[1];
        cnt = hdr[2];
        tile = hdr[3];
      } else {
        int unit;
        item_info(p, it0 + s / nchunks, unit, tile, slot, p0, cnt, TB);
#pragma unroll
        for (int b = 0; b < TB; ++b)
          brow[b] = (b * 8 + g < cnt) ? p.bsrc + (size_t)b_row_index(p, p0, b * 8 + g) * p.K : nullptr;
      }
#pragma unroll
      for (int m = 0; m < NM; ++m)
#pragma unroll
        for (int b = 0; b < TB; ++b)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[m][b][i] = 0.f;
    }
    if (!aborted) {
      const uint8_t* wb = sb + kHdrBytes;
      uint4 bv[TB], bvn[TB];
      if constexpr (TB > 1) {
#pragma unroll
        for (int b = 0; b < TB; ++b) {
          const int kk = c * KC + (warp * G::GPW) * 32 + t * 8;
          bv[b] = brow[b] ? ldg_nc_v4(brow[b] + kk) : make_uint4(0u, 0u, 0u, 0u);
        }
      }
#pragma unroll
      for (int jj = 0; jj < G::GPW; ++jj) {
        const int j = warp * G::GPW + jj;
        if constexpr (TB == 1) {
          bv[0] = (g < cnt) ? lds_v4(wb + NM * G::MAT + g * G::BS + j * 64 + t * 16)
                            : make_uint4(0u, 0u, 0u, 0u);
        } else {
          if (jj + 1 < G::GPW) {
#pragma unroll
            for (int b = 0; b < TB; ++b) {
              const int kk = c * KC + (j + 1) * 32 + t * 8;
              bvn[b] = brow[b] ? ldg_nc_v4(brow[b] + kk) : make_uint4(0u, 0u, 0u, 0u);
            }
          }
        }
#pragma unroll
        for (int m = 0; m < NM; ++m) {
          const uint8_t* mb = wb + m * G::MAT;
          const uint32_t w0 = *reinterpret_cast<const uint32_t*>(mb + g * G::WS + j * 16 + t * 4);
          const uint32_t w1 = *reinterpret_cast<const uint32_t*>(mb + (g + 8) * G::WS + j * 16 + t * 4);
          const float sc0 = e8m0_to_f32(mb[kRows * G::WS + g * G::SS + j]);
          const float sc1 = e8m0_to_f32(mb[kRows * G::WS + (g + 8) * G::SS + j]);
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

template <int NM, int TB, int NSTAGE, int MODE, int KC>
static cudaError_t launch_tiles(const ExpertParams& p, int grid, cudaStream_t st) {
  auto kfn = expert_tiles_kernel<NM, TB, NSTAGE, MODE, KC>;
  constexpr int smem = smem_bytes<NM, TB, NSTAGE, KC>();
  static_assert(smem <= 232448, "shared memory budget");
  if (p.K % KC != 0) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kfn<<<grid, kThreads, smem, st>>>(p);
  return cudaGetLastError();
}

// ==================================================================================================
// TMA-fed decode kernel (1-8 rows per distinct expert).
//
// Work item = (distinct expert u, tile of 16 weight rows), K streamed in chunks of 2048 elements.  Per
// chunk the producer issues one TMA box per matrix for the packed e2m1 bytes (16 rows x 8 panels of
// 128 B, 128B-swizzled so that row r's 16-byte chunk j sits at chunk j ^ (r % 8)) and one for the e8m0
// scales; the activation rows of the expert (<= 8 routed rows, full K, f16) are staged once per expert
// into a padded buffer.  Consumer warp w takes panel w (8 groups of 32 elements) of each chunk.
constexpr int kDKC = 2048;
constexpr int kDPanels = kDKC / 256;           // 8 = one panel per consumer warp
constexpr int kDWBox = kDPanels * kRows * 128;  // 16 KiB of packed weights per matrix per stage
constexpr int kDSBox = kRows * (kDKC / 32);     // 1 KiB of scales per matrix per stage
static_assert(kDPanels == kCW, "one 128-byte panel per consumer warp");

template <int NM>
constexpr int dstage_bytes() { return NM * (kDWBox + kDSBox); }
template <int KMAX>
constexpr int dbrow_bytes() { return KMAX * 2 + 64; }  // +64 B: conflict-free 16-byte reads across rows
template <int NM, int NSTAGE, int KMAX, int CW>
constexpr int dsmem_bytes() {
  return kBarBytes + ((8 * dbrow_bytes<KMAX>() + 1023) / 1024) * 1024 + NSTAGE * dstage_bytes<NM>() +
         CW * NM * 128 * 4;
}

// CW consumer warps (8 or 16): warp w takes panel w / (CW/8) and, within it, 8 / (CW/8) of the 8 groups.
template <int NM, int NSTAGE, int MODE, int KMAX, int CW>
__global__ void __launch_bounds__((CW + 1) * 32, 1) expert_decode_tma_kernel(const __grid_constant__ DecodeParams p) {
  constexpr int WPP = CW / 8;     // warps per panel
  constexpr int GPWD = 8 / WPP;   // groups per warp per chunk
  static_assert(CW == 8 || CW == 16, "8 or 16 consumer warps");
  constexpr int SB = dstage_bytes<NM>();
  constexpr int BR = dbrow_bytes<KMAX>();
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + NSTAGE;
  uint64_t* bfull = empty + NSTAGE;
  uint64_t* bempty = bfull + 1;
  int* hdr = reinterpret_cast<int*>(bempty + 1);  // [NSTAGE][4]: slot, p0, cnt, tile
  volatile int* s_abort = hdr + 4 * NSTAGE;
  uint8_t* bbuf = smem + kBarBytes;
  uint8_t* stages = bbuf + ((8 * BR + 1023) / 1024) * 1024;
  float* red = reinterpret_cast<float*>(stages + NSTAGE * SB);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = p.num_units ? min(__ldg(p.num_units), p.units_cap) : p.units_cap;
  const long long items = (long long)units * p.tiles;
  const long long it0 = items * blockIdx.x / gridDim.x;
  const long long it1 = items * (blockIdx.x + 1) / gridDim.x;
  const int nchunks = p.K / kDKC;
  const long long nsteps = (it1 - it0) * nchunks;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NSTAGE; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], CW);
    }
    mbar_init(bfull, 1);
    mbar_init(bempty, CW);
    *s_abort = 0;
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == CW) {
    // ------------------------------------------------------------------------------ producer
    if (lane == 0) {
      for (int m = 0; m < NM; ++m) {
        tma_prefetch_map(&p.wmap[m]);
        tma_prefetch_map(&p.smap[m]);
      }
    }
    const uint64_t pol = l2_evict_first_policy();
    int stage = 0;
    uint32_t ph = 0, bph = 0;
    long long issued = 0;
    int cur_unit = -1, slot = 0, cnt = 0, p0 = 0;
    bool b_pending = false;
    for (long long s = 0; s < nsteps; ++s) {
      const long long item = it0 + s / nchunks;
      const int c = (int)(s % nchunks);
      const int unit = (int)(item / p.tiles), tile = (int)(item % p.tiles);
      if (*s_abort) break;
      if (unit != cur_unit) {
        slot = __ldg(p.unit_slot + unit);
        cnt = unit_route_count(p.unit_cnt, unit, min(8, p.p0_stride), p.status);
        p0 = unit * p.p0_stride;
        int brow = (lane < cnt) ? (p.rtok ? __ldg(p.rtok + p0 + lane) : p0 + lane) : 0;
        if (p.brows > 0 && (brow < 0 || brow >= p.brows)) {  // never read past the activation rows
          set_status(p.status, MIMO_ERANGE);
          brow = 0;
        }
        // the consumers release the previous expert's rows when they start this one
        if (!mbar_wait(bempty, bph ^ 1u)) {
          if (lane == 0) set_status(p.status, MIMO_ETIMEOUT);
          *s_abort = 1;
          break;
        }
        if (lane == 0) mbar_arrive_expect_tx(bfull, (uint32_t)cnt * p.K * 2);
        __syncwarp();
        if (lane < cnt) bulk_g2s_keep(bbuf + lane * BR, p.bsrc + (size_t)brow * p.K, p.K * 2, bfull);
        b_pending = true;
        bph ^= 1u;
        cur_unit = unit;
        if ((slot < 0 || slot >= p.S) && lane == 0) set_status(p.status, MIMO_ERANGE);
      }
      const int cslot = (slot < 0 || slot >= p.S) ? 0 : slot;  // bad items stream slot 0, then are discarded
      if (!mbar_wait(&empty[stage], ph ^ 1u)) {
        if (lane == 0) set_status(p.status, MIMO_ETIMEOUT);
        *s_abort = 1;
        break;
      }
      if (lane == 0) {
        hdr[stage * 4 + 0] = slot;
        hdr[stage * 4 + 1] = p0;
        hdr[stage * 4 + 2] = cnt;
        hdr[stage * 4 + 3] = tile;
        uint8_t* sb = stages + stage * SB;
        mbar_arrive_expect_tx(&full[stage], NM * (kDWBox + kDSBox));
        const int row0 = cslot * p.N + tile * kRows;
        for (int m = 0; m < NM; ++m) {
          uint8_t* wdst = sb + m * kDWBox;
          if (!p.per_panel) {
            tma_load_3d(wdst, &p.wmap[m], 0, row0, c * kDPanels, &full[stage], pol);
          } else {
            for (int q = 0; q < kDPanels; ++q)
              tma_load_2d(wdst + q * kRows * 128, &p.wmap[m], (c * kDPanels + q) * 128, row0, &full[stage], pol);
          }
          tma_load_2d(sb + NM * kDWBox + m * kDSBox, &p.smap[m], c * (kDKC / 32), row0, &full[stage], pol);
        }
      }
      __syncwarp();
      ++issued;
      if (++stage == NSTAGE) {
        stage = 0;
        ph ^= 1u;
      }
    }
    // Drain: never leave the CTA with copies in flight (matters only after an abort).
    const long long tail = issued < NSTAGE ? issued : NSTAGE;
    for (long long k = 0; k < tail; ++k) {
      const long long f = issued - 1 - k;
      if (!mbar_wait(&full[(int)(f % NSTAGE)], (uint32_t)((f / NSTAGE) & 1))) {
        if (lane == 0) set_status(p.status, MIMO_ETIMEOUT);
        break;
      }
    }
    if (b_pending && !mbar_wait(bfull, bph ^ 1u) && lane == 0) set_status(p.status, MIMO_ETIMEOUT);
    return;
  }

  // -------------------------------------------------------------------------------- consumers
  const int g = lane >> 2, t = lane & 3;
  const int tid = threadIdx.x;
  int stage = 0;
  uint32_t ph = 0, bph = 0;
  bool aborted = false;
  int cur_unit = -1, tile = 0, slot = 0, p0 = 0, cnt = 0;
  float acc[NM][4];

  for (long long s = 0; s < nsteps; ++s) {
    const long long item = it0 + s / nchunks;
    const int c = (int)(s % nchunks);
    const int unit = (int)(item / p.tiles);
    if (unit != cur_unit) {
      if (cur_unit >= 0) {
        __syncwarp();
        if (lane == 0) mbar_arrive(bempty);
      }
      if (!aborted && !mbar_wait(bfull, bph)) {
        aborted = true;
        set_status(p.status, MIMO_ETIMEOUT);
        *s_abort = 1;
      }
      bph ^= 1u;
      cur_unit = unit;
    }
    if (!aborted && !mbar_wait(&full[stage], ph)) {
      aborted = true;
      set_status(p.status, MIMO_ETIMEOUT);
      *s_abort = 1;
    }
    if (c == 0) {
      slot = hdr[stage * 4 + 0];
      p0 = hdr[stage * 4 + 1];
      cnt = hdr[stage * 4 + 2];
      tile = hdr[stage * 4 + 3];
#pragma unroll
      for (int m = 0; m < NM; ++m)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[m][i] = 0.f;
    }
    if (!aborted) {
      const uint8_t* sb = stages + stage * SB;
      const int panel = warp / WPP, jbase = (warp % WPP) * GPWD;
      // scales of this warp's groups for rows g and g+8
      uint32_t sc_lo[NM][2], sc_hi[NM][2];
#pragma unroll
      for (int m = 0; m < NM; ++m) {
        const uint8_t* sm_ = sb + NM * kDWBox + m * kDSBox + panel * 8 + jbase;
        if constexpr (GPWD == 8) {
          const uint2 a = *reinterpret_cast<const uint2*>(sm_ + g * (kDKC / 32));
          const uint2 b = *reinterpret_cast<const uint2*>(sm_ + (g + 8) * (kDKC / 32));
          sc_lo[m][0] = a.x; sc_lo[m][1] = a.y; sc_hi[m][0] = b.x; sc_hi[m][1] = b.y;
        } else {
          sc_lo[m][0] = *reinterpret_cast<const uint32_t*>(sm_ + g * (kDKC / 32));
          sc_hi[m][0] = *reinterpret_cast<const uint32_t*>(sm_ + (g + 8) * (kDKC / 32));
          sc_lo[m][1] = sc_hi[m][1] = 0u;
        }
      }
      // e8m0 -> float32 as (byte << 23); bytes 0 (2^-127) and 255 (NaN) take the exact slow path.
      bool special = false;
#pragma unroll
      for (int m = 0; m < NM; ++m)
#pragma unroll
        for (int h = 0; h < (GPWD == 8 ? 2 : 1); ++h) {
          const uint32_t a = sc_lo[m][h], b = sc_hi[m][h];
          special |= (((a - 0x01010101u) & ~a) | ((~a - 0x01010101u) & a) | ((b - 0x01010101u) & ~b) |
                      ((~b - 0x01010101u) & b)) & 0x80808080u;
        }
      const uint8_t* brow = bbuf + g * BR + (size_t)c * kDKC * 2;
#pragma unroll
      for (int q = 0; q < GPWD; ++q) {
        const int jj = jbase + q;      // group within the panel
        const int j = panel * 8 + jj;  // group within the chunk
        const uint4 bv = (g < cnt) ? lds_v4(brow + j * 64 + t * 16) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int m = 0; m < NM; ++m) {
          const uint8_t* pan = sb + m * kDWBox + panel * (kRows * 128);
          const int sw = (jj ^ (g & 7)) * 16 + t * 4;
          const uint32_t w0 = *reinterpret_cast<const uint32_t*>(pan + g * 128 + sw);
          const uint32_t w1 = *reinterpret_cast<const uint32_t*>(pan + (g + 8) * 128 + sw);
          const uint32_t b0 = sc_lo[m][q >> 2], b1 = sc_hi[m][q >> 2];
          float s0, s1;
          if (!special) {
            s0 = __uint_as_float(__byte_perm(b0, 0u, 0x0444u | ((q & 3) << 12)) >> 1);
            s1 = __uint_as_float(__byte_perm(b1, 0u, 0x0444u | ((q & 3) << 12)) >> 1);
          } else {
            s0 = e8m0_to_f32((b0 >> ((q & 3) * 8)) & 0xFFu);
            s1 = e8m0_to_f32((b1 >> ((q & 3) * 8)) & 0xFFu);
          }
          uint32_t ra[4], rb[4];
          e2m1x8_to_f16x2(w0, ra);
          e2m1x8_to_f16x2(w1, rb);
          float tmp[4];
          const float z[4] = {0.f, 0.f, 0.f, 0.f};
          mma_16816(tmp, ra[0], rb[0], ra[1], rb[1], bv.x, bv.y, z);
          mma_16816(tmp, ra[2], rb[2], ra[3], rb[3], bv.z, bv.w, tmp);
          acc[m][0] = fmaf(tmp[0], s0, acc[m][0]);
          acc[m][1] = fmaf(tmp[1], s0, acc[m][1]);
          acc[m][2] = fmaf(tmp[2], s1, acc[m][2]);
          acc[m][3] = fmaf(tmp[3], s1, acc[m][3]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == NSTAGE) {
      stage = 0;
      ph ^= 1u;
    }

    if (c == nchunks - 1) {
      float* rw_ = red + warp * (NM * 128);
#pragma unroll
      for (int m = 0; m < NM; ++m) {
        float* r = rw_ + m * 128;
        r[g * 8 + 2 * t] = acc[m][0];
        r[g * 8 + 2 * t + 1] = acc[m][1];
        r[(g + 8) * 8 + 2 * t] = acc[m][2];
        r[(g + 8) * 8 + 2 * t + 1] = acc[m][3];
      }
      named_bar_sync(1, CW * 32);
      const bool bad = (slot < 0 || slot >= p.S);
      if (!aborted && !bad && tid < kRows * 8) {
        const int row = tid % kRows, q = tid / kRows;
        if (q < cnt) {
          float v[NM];
#pragma unroll
          for (int m = 0; m < NM; ++m) {
            float sum = 0.f;
#pragma unroll
            for (int w = 0; w < CW; ++w) sum += red[w * (NM * 128) + m * 128 + row * 8 + q];
            v[m] = sum;
          }
          const size_t op = (size_t)(p0 + q) * p.N + (size_t)tile * kRows + row;
          if constexpr (MODE == 0) {
            p.h_out[op] = to_f16_checked(swiglu_ref(v[0], v[NM - 1]), p.status);
          } else {
            const float d = p.pairs_rounding ? bf16_round(v[0]) : v[0];
            p.part_out[op] = d * __ldg(p.rw + p0 + q);
          }
        }
      }
      named_bar_sync(1, CW * 32);
    }
  }
}

template <int NM, int NSTAGE, int MODE, int KMAX, int CW>
static cudaError_t launch_dtma(const DecodeParams& p, int grid, cudaStream_t st) {
  auto kfn = expert_decode_tma_kernel<NM, NSTAGE, MODE, KMAX, CW>;
  constexpr int smem = dsmem_bytes<NM, NSTAGE, KMAX, CW>();
  static_assert(smem <= 232448, "shared memory budget");
  if (p.K % kDKC != 0 || p.K > KMAX) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kfn<<<grid, (CW + 1) * 32, smem, st>>>(p);
  return cudaGetLastError();
}

// Consumer warps per CTA (8 or 16); tuning knob MIMO_MOE_DECODE_WARPS, default 8.
static int decode_warps() {
  static int w = [] {
    const char* e = getenv("MIMO_MOE_DECODE_WARPS");
    return (e && atoi(e) == 16) ? 16 : 8;
  }();
  return w;
}

cudaError_t launch_decode_tma(const DecodeParams& p, int kind, int num_sms, cudaStream_t st) {
  const bool w16 = decode_warps() == 16;
  if (kind == 0) return w16 ? launch_dtma<2, 4, 0, 4096, 16>(p, num_sms, st) : launch_dtma<2, 4, 0, 4096, 8>(p, num_sms, st);
  if (kind == 1) return w16 ? launch_dtma<1, 10, 1, 2048, 16>(p, num_sms, st) : launch_dtma<1, 10, 1, 2048, 8>(p, num_sms, st);
  return cudaErrorInvalidValue;
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
    case 0: return launch_tiles<2, 1, 6, 0, 1024>(p, num_sms, st);   // decode gate/up
    case 1: return launch_tiles<1, 1, 8, 1, 1024>(p, num_sms, st);   // decode down
    case 2: return launch_tiles<2, 8, 4, 0, 2048>(p, num_sms, st);   // prefill gate/up
    case 3: return launch_tiles<1, 8, 9, 2, 2048>(p, num_sms, st);   // prefill down
    default: return cudaErrorInvalidValue;
  }
}

// ------------------------------------------------------------------------------------ combine
// Decode (kernels.py:196-199): y[t, m] = bf16(sum_k part[gidx[t, k], m]) in route order; with
// gidx == null, the scatter-add of kernels.py:196-197 summed in (u, r) order.  part holds ucap * R
// rows: a gidx entry at or beyond that sets MIMO_ERANGE and is skipped (negative entries are skipped
// silently, as unused routes).
__global__ void combine_decode_kernel(const float* __restrict__ part, const int32_t* __restrict__ gidx,
                                      const int32_t* __restrict__ urows, const int32_t* __restrict__ ucnt,
                                      const int32_t* __restrict__ num_unique, int ucap, int R, int M,
                                      int topk, int H, uint16_t* __restrict__ y, int32_t* status) {
  pdl_wait();  // the partials come from the preceding kernel
  pdl_launch_dependents();
  const int t = blockIdx.x;  // rows on x: gridDim.y stops at 65535
  const int m = (blockIdx.y * blockDim.x + threadIdx.x) * 4;
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
    const long long rows = (long long)ucap * R;
    for (int k = 0; k < topk; ++k) {
      const int sl = gidx[t * topk + k];
      if (sl >= rows) {
        if (m == 0) set_status(status, MIMO_ERANGE);
        continue;
      }
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
                                  int M, int topk, int H, uint16_t* y, int32_t* status, cudaStream_t st) {
  dim3 grid(M, (H / 4 + 255) / 256);
  return launch_k(combine_decode_kernel, grid, dim3(256), 0, st, part, gidx, urows, ucnt, num_unique, ucap, R, M,
                  topk, H, y, status);
}

// y[m] = bf16(sum over k in order of part[row]) with row = gidx[m * topk + k] (skipped when < 0), or
// m * topk + k without gidx (kernels.py:194-199).  part holds part_rows rows; a gidx entry at or beyond
// that sets MIMO_ERANGE (when status is given) and is skipped.
__global__ void combine_rows_kernel(const float* __restrict__ part, const int32_t* __restrict__ gidx, int M,
                                    int topk, int H, long long part_rows, uint16_t* __restrict__ y,
                                    int32_t* status) {
  const int t = blockIdx.x;  // rows on x: gridDim.y stops at 65535
  const int m = (blockIdx.y * blockDim.x + threadIdx.x) * 4;
  if (t >= M || m >= H) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k = 0; k < topk; ++k) {
    const int sl = gidx ? gidx[t * topk + k] : t * topk + k;
    if (sl >= part_rows) {
      if (m == 0) set_status(status, MIMO_ERANGE);
      continue;
    }
    if (sl < 0) continue;
    const float4 v = *reinterpret_cast<const float4*>(part + (size_t)sl * H + m);
    acc.x = __fadd_rn(acc.x, v.x);
    acc.y = __fadd_rn(acc.y, v.y);
    acc.z = __fadd_rn(acc.z, v.z);
    acc.w = __fadd_rn(acc.w, v.w);
  }
  const uint32_t o0 = f32_to_bf16(acc.x) | (f32_to_bf16(acc.y) << 16);
  const uint32_t o1 = f32_to_bf16(acc.z) | (f32_to_bf16(acc.w) << 16);
  *reinterpret_cast<uint2*>(y + (size_t)t * H + m) = make_uint2(o0, o1);
}

cudaError_t launch_combine_rows(const float* part, const int32_t* gidx, int M, int topk, int H,
                                long long part_rows, uint16_t* y, int32_t* status, cudaStream_t st) {
  dim3 grid(M, (H / 4 + 255) / 256);
  combine_rows_kernel<<<grid, 256, 0, st>>>(part, gidx, M, topk, H, part_rows, y, status);
  return cudaGetLastError();
}

// Prefill (model.py:266-271): y[t, m] = bf16(sum_k fp32(ypair[inv[t, k], m]) * w[t, k]) in k order.
__global__ void combine_prefill_kernel(const uint16_t* __restrict__ ypair, const int32_t* __restrict__ inv,
                                       const float* __restrict__ w, int T, int topk, int H,
                                       uint16_t* __restrict__ y) {
  const int t = blockIdx.x;  // rows on x: gridDim.y stops at 65535
  const int m = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (t >= T || m >= H) return;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int k = 0; k < topk; ++k) {
    const int pos = inv[t * topk + k];
    if (pos < 0) continue;
    const float wk = w ? w[t * topk + k] : 1.f;
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
  dim3 grid(T, (H / 8 + 255) / 256);
  combine_prefill_kernel<<<grid, 256, 0, st>>>(ypair, inv, w, T, topk, H, y);
  return cudaGetLastError();
}

}  // namespace mimo
