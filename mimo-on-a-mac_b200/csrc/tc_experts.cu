// MXFP4 expert products on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Weights stay in their MXFP4 form end to end: TMA copies the packed e2m1 bytes of a 128-row x
// 128-value tile into shared memory in the padded layout the block-scaled MMA reads
// (CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B: 8 data bytes + 8 gap bytes per 16 values, 128B swizzle),
// and tcgen05.mma.kind::mxf8f6f4.block_scale applies the pool's e8m0 scales in hardware.
// Activations are split into two e4m3 terms, each with one ue8m0 scale per 32 values
// (x = hi * s1 + lo * s2; two 4-bit-significand terms carry all 8 significant bits of a bf16 value
// unless a value is 2^9 or more below its block's largest), and enter the MMA as 2 * NTOK columns;
// the epilogue adds the two columns of each route.
//
// Roles (one CTA per SM, persistent over work items = (unit, 128-row weight tile)):
//   warp 0      TMA producer: per 128-value K chunk, the weight tiles of NM matrices and the unit's
//               activation-term tile into a ring of NSTAGE stages; per group of 4 chunks, 16-byte
//               wide boxes of the weight and activation scale rows into a 2-entry scale ring;
//   warp 1      scale-factor builder: per stage, rearranges the chunk's 4 e8m0 bytes of each of the
//               128 weight rows and of the (padded to 128) activation rows into the 512-byte block
//               that tcgen05.cp.32x128b.warpx4 turns into the TMEM scale layout (block byte
//               (m % 32) * 16 + (m / 32) * 4 + kb for row m, K block kb); its arrival is the second
//               of the stage's `full` barrier, so the MMA issuer waits on one barrier per stage;
//   warps 2-3   MMA issuers (one lane each, warp 3 also allocates TMEM): tcgen05.cp of the scale
//               blocks and 4 MMAs of K = 32 per stage into the issuer's own accumulator of a double
//               buffer (gate / up, or even / odd stages of down), tcgen05.commit to free the stage;
//   warps 4-11  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lanes 32 * (w % 4) + 0..31,
//               i.e. weight rows, for half of the routes), then
//               MODE 0  SwiGLU with the reference's roundings (engine/mimo_stream/kernels.py:79-82)
//                       and the split of h into two e4m3 terms for the down pass;
//               MODE 1  down x route weight (kernels.py:120), fp32 partials for the fixed-order
//                       combine;
//               MODE 2  bf16 pair outputs (engine/mimo_stream/model.py:228).
// The producer does its per-item work (coordinates, slot, row base) once per item: at decode sizes a
// stage lasts ~600 cycles and the single issuing threads are the critical path.
// Every wait is bounded; an expired wait sets MIMO_ETIMEOUT and the CTA drains and returns.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace mimo {
namespace tc {

constexpr int kM = 128;           // weight rows per tile (MMA M)
constexpr int kKC = 128;          // K values per stage
constexpr int kATile = kM * kKC;  // shared bytes of one padded e2m1 tile (16 KiB)
constexpr int kAGlobal = kATile / 2;  // global (packed) bytes of one tile: the TMA transaction count
constexpr int kEpiWarps = 8;  // two per TMEM lane quadrant, each taking half of the routes
constexpr int kThreads = (4 + kEpiWarps) * 32;
constexpr int kBarBytes = 2048;   // barriers + TMEM slot, then 1 KiB alignment slack

// Ring depths of kinds 0..3 (decode gate/up, decode down, prefill gate/up, prefill down).
#ifndef MIMO_TC_ST0
#define MIMO_TC_ST0 6
#endif
#ifndef MIMO_TC_ST1
#define MIMO_TC_ST1 5
#endif
#ifndef MIMO_TC_ST2
#define MIMO_TC_ST2 4
#endif
#ifndef MIMO_TC_ST3
#define MIMO_TC_ST3 3
#endif
#ifndef MIMO_TC_EPI_PREFILL
#define MIMO_TC_EPI_PREFILL 16  // epilogue warps of the prefill kernels
#endif
#ifndef MIMO_TC_PST2
#define MIMO_TC_PST2 5  // ring depth of the paired prefill gate/up kernel
#endif
#ifndef MIMO_TC_PST3
#define MIMO_TC_PST3 4  // ring depth of the paired prefill down kernel
#endif
#ifndef MIMO_TC_STF
#define MIMO_TC_STF 5  // ring depth of the fused decode kernel, e4m3 activation terms
#endif
#ifndef MIMO_TC_STF4
#define MIMO_TC_STF4 9  // ring depth of the fused decode kernel, e2m1 activation terms (packed weights)
#endif
#ifndef MIMO_TC_WEIGHT_EVICT_FIRST
#define MIMO_TC_WEIGHT_EVICT_FIRST 1  // decode streams each weight once: L2 evict-first
#endif
constexpr int kStages[4] = {MIMO_TC_ST0, MIMO_TC_ST1, MIMO_TC_ST2, MIMO_TC_ST3};

// A stage holds two "slots", one per MMA issuer: (matrix j, chunk c) for gate/up (NM = 2, one K
// chunk per stage) or (matrix 0, chunk c + j) for down (NM = 1, two K chunks per stage).
// Stage layout: [A tile slot 0 | A tile slot 1 | KPS activation tiles], 1024-byte aligned tiles.
template <int NM>
constexpr int kps() { return 2 / NM; }  // K chunks per stage
template <int NM, int N>
constexpr int stage_bytes() { return 2 * kATile + kps<NM>() * N * kKC; }
template <int NM, int N>
constexpr int scale_box_bytes() { return NM * kM * 16 + N * 16; }  // one 4-chunk group's scale boxes
template <int NM>
constexpr int sf_block_bytes() { return (2 + kps<NM>()) * 512; }  // per stage: 2 weight + KPS act. blocks
template <int NM, int N, int NSTAGE>
constexpr int smem_bytes() {
  return kBarBytes + 1024 + NSTAGE * stage_bytes<NM, N>() + 2 * scale_box_bytes<NM, N>() +
         NSTAGE * sf_block_bytes<NM>();
}
// Accumulator buffers: two (the epilogue of one item overlaps the MMAs of the next) when TMEM has
// room, else one (the epilogue copies its columns to registers and frees the buffer at once).
template <int N, int NSTAGE>
constexpr int abuf() { return 4 * N + NSTAGE * 16 <= 512 ? 2 : 1; }
template <int N, int NSTAGE>
constexpr int tmem_cols_needed() { return abuf<N, NSTAGE>() * 2 * N + NSTAGE * 16; }  // accumulators + scales
template <int N, int NSTAGE>
constexpr uint32_t tmem_cols() {
  constexpr int n = tmem_cols_needed<N, NSTAGE>();
  return n <= 32 ? 32 : n <= 64 ? 64 : n <= 128 ? 128 : n <= 256 ? 256 : 512;
}

// Splits v into hi/lo e4m3 bytes and their block scale bytes; the 32 lanes form one block.
__device__ __forceinline__ void split_warp_block(float v, uint32_t& hi, uint32_t& lo, uint32_t& b1, uint32_t& b2) {
  // Non-negative floats order like their bit patterns: one redux.sync gives the block maximum.
  const float amax = __uint_as_float(__reduce_max_sync(0xFFFFFFFFu, __float_as_uint(fabsf(v))));
  b1 = block_scale_byte(amax);
  hi = f32_to_e4m3(v * inv_exp2_byte(b1));
  const float r = v - e4m3_to_f32(hi) * exp2_byte(b1);
  const float rmax = __uint_as_float(__reduce_max_sync(0xFFFFFFFFu, __float_as_uint(fabsf(r))));
  b2 = block_scale_byte(rmax);
  lo = f32_to_e4m3(r * inv_exp2_byte(b2));
}

// ------------------------------------------------------------------------------------ kernel
// Work item i -> (unit, weight tile).  Without groups, unit-major.  With groups (prefill: the units
// of one expert are consecutive), the items of a group are taken tile-major, so the units of one
// expert read each weight tile back to back and all but the first find it in L2.
__device__ __forceinline__ void item_coords(const TcParams& p, long long i, int& unit, int& tile) {
  const int ur = (int)(i / p.tiles);
  if (p.unit_first) {
    const int u0 = __ldg(p.unit_first + ur);
    const int n = __ldg(p.unit_nsub + ur);
    const long long j = i - (long long)u0 * p.tiles;
    tile = (int)(j / n);
    unit = u0 + (int)(j % n);
  } else {
    unit = ur;
    tile = (int)(i % p.tiles);
  }
}

// Routes of a unit, at most `cap`: units at a fixed stride (unit_p0 null: p0 = unit * p0_stride) own
// p0_stride route slots, so a count above that sets MIMO_ERANGE and is cut (it would write into the
// next unit's rows, or past the last one's).
__device__ __forceinline__ int unit_routes(const TcParams& p, int unit, int cap) {
  const int lim = p.unit_p0 ? cap : min(cap, p.p0_stride);
  const int c = __ldg(p.unit_cnt + unit);
  if (c > lim) {
    set_status(p.status, MIMO_ERANGE);
    return lim;
  }
  return max(c, 0);
}

namespace fz {
__device__ __forceinline__ int ld_acquire(const int32_t* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;\n" ::: "memory");
}
}  // namespace fz

// Decode combine (kernels.py:194-199) of output rows [128 tile, 128 tile + 128), run by the epilogue
// warps (ew = 0 .. nw - 1) of the CTA whose tile stores complete the count p.cdone[tile] (one per unit
// and tile).  Before counting, every thread's partial stores are fenced; the winner fences again and
// reads the partials through L2.  The sum over a token's routes is in the order of the separate combine
// kernel, so the output is bit-identical to it.
__device__ __noinline__ void combine_tile(const TcParams& p, int tile, int units, int ew, int lane, int nw,
                                          volatile int* s_last) {
  __threadfence();
  named_bar_sync(1, nw * 32);
  if (ew == 0 && lane == 0) *s_last = atomicAdd(p.cdone + tile, 1) == units - 1;
  named_bar_sync(1, nw * 32);
  const bool last = *s_last;
  named_bar_sync(1, nw * 32);  // s_last is rewritten for the next item only after everyone read it
  if (!last) return;
  __threadfence();
  const long long rows = (long long)p.units_cap * p.p0_stride;  // rows of part
  const int col0 = tile * kM;
  for (int o = ew * 32 + lane; o < p.cM * kM; o += nw * 32) {
    const int m = o / kM, j = col0 + o % kM;
    float sum = 0.f;
    if (p.cgidx) {
      for (int k = 0; k < p.ctopk; ++k) {
        const int sl = __ldg(p.cgidx + m * p.ctopk + k);
        if (sl >= rows) {
          set_status(p.status, MIMO_ERANGE);
          continue;
        }
        if (sl >= 0) sum = __fadd_rn(sum, __ldcg(p.part + (size_t)sl * p.Nw + j));
      }
    } else {
      for (int u = 0; u < units; ++u) {
        const int n = min(__ldg(p.cucnt + u), p.p0_stride);
        for (int r = 0; r < n; ++r)
          if (__ldg(p.curows + u * p.p0_stride + r) == m)
            sum = __fadd_rn(sum, __ldcg(p.part + (size_t)(u * p.p0_stride + r) * p.Nw + j));
      }
    }
    p.cy[(size_t)m * p.Nw + j] = (uint16_t)f32_to_bf16(sum);
  }
}

// EPI epilogue warps (a multiple of 4): EPI / 4 per TMEM lane quadrant, each taking NTOK / (EPI / 4) of
// the routes.  Prefill uses 16: its per-route SwiGLU and term split are long dependent chains, and
// four warps per SM sub-partition hide their latency where two cannot.
template <int NM, int NTOK, int NSTAGE, int MODE, int EPI>
__global__ void __launch_bounds__((4 + EPI) * 32, 1) tc_expert_kernel(const __grid_constant__ TcParams p) {
  constexpr int N = 2 * NTOK;
  constexpr int KPS = kps<NM>();
  constexpr int SB = stage_bytes<NM, N>();
  constexpr int SCB = scale_box_bytes<NM, N>();
  constexpr int SFB = sf_block_bytes<NM>();
  constexpr uint32_t TCOLS = tmem_cols<N, NSTAGE>();
  constexpr int QH = NTOK / (EPI / 4);       // routes per epilogue warp
  constexpr int QC = QH < 16 ? QH : 16;      // routes per TMEM load in the epilogue
  static_assert(EPI % 4 == 0 && NTOK % (EPI / 4) == 0 && QH % QC == 0, "epilogue split");
  static_assert(NM * KPS == 2, "two slots per stage");
  static_assert(N % 16 == 0 && N <= 256 && QH % QC == 0, "MMA N");
  // MODE 3 / 4 (decode / prefill down, paired row tiles): an item is 256 output rows, slot m holding
  // rows [128 m, 128 m + 128) of it with one K chunk per stage; the two accumulators are separate rows.
  constexpr bool PAIRED = MODE == 3 || MODE == 4;
  static_assert(!PAIRED || NM == 2, "paired row tiles take the two slots");
  constexpr int TROWS = PAIRED ? 2 * kM : kM;  // weight rows per item
  constexpr int MROW = PAIRED ? kM : 0;        // row offset of slot 1's tile (gate/up: same rows)
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // [NSTAGE] tiles landed + scale blocks written
  uint64_t* empty = full + NSTAGE;                     // [NSTAGE] both issuers' MMAs of the stage done
  uint64_t* sc_full = empty + NSTAGE;                  // [2] scale boxes of a 4-chunk group landed
  uint64_t* sc_empty = sc_full + 2;                    // [2] scale boxes read
  uint64_t* acc_full = sc_empty + 2;                   // [2]
  uint64_t* acc_empty = acc_full + 2;                  // [2]
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* base = reinterpret_cast<uint8_t*>(((uintptr_t)(smem + kBarBytes) + 1023) & ~(uintptr_t)1023);
  uint8_t* stages = base;                   // NSTAGE x [2 A tiles | KPS B tiles]
  uint8_t* scbox = stages + NSTAGE * SB;    // 2 x [NM x A scale box | B scale box]
  uint8_t* sfblk = scbox + 2 * SCB;         // NSTAGE x [2 weight scale blocks | KPS activation blocks]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NSTAGE; ++i) {
      mbar_init(&full[i], 2);   // the producer's expect-tx arrival + the scale builder's arrival
      mbar_init(&empty[i], 2);  // one commit per issuer
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sc_full[b], 1);
      mbar_init(&sc_empty[b], 1);
      mbar_init(&acc_full[b], 2);
      mbar_init(&acc_empty[b], EPI);
    }
    mbar_init(drain, 2);
    *s_abort = 0;
    mbar_fence_init();
  }
  if (warp == 3) {
    tmem_alloc(tmem_slot, TCOLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Early down (MODE 3 with ready counters): no wait for the whole gate/up grid.  The unit tables were
  // written before the gate/up launch started its work (each launch of the chain waits for its
  // predecessor before it lets its successor start), and a unit's h terms are waited for per unit by
  // the producer below; nothing else this kernel reads comes from the gate/up launch.
  const bool early = MODE == 3 && p.ready != nullptr;
  if (!early) pdl_wait();  // the unit tables and activation terms come from the preceding kernel
  pdl_launch_dependents();
  const uint32_t tbase = *tmem_slot;
  // after the wait: the unit count is written by the preceding kernel
  const int units = p.num_units ? min(__ldcg(p.num_units), p.units_cap) : p.units_cap;
  const long long items = (long long)units * p.tiles;
  // Items are dealt round-robin: at any time the CTAs work on consecutive items (the tiles and units
  // of the same experts), so a weight tile shared by an expert's units and a unit's activation tile
  // shared by its weight tiles are read from L2 by CTAs running side by side.  CTA-local item n is
  // item blockIdx.x + n * gridDim.x.
  const long long my_items = items > blockIdx.x ? (items - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  const int ns = p.K / (kKC * KPS);  // stages per item; K chunks per item are a multiple of 4
  const long long nsteps = my_items * ns;
  constexpr int ABUF = abuf<N, NSTAGE>();
  constexpr uint32_t kSfCol0 = ABUF * 2 * N;  // accumulator (buf, j) at columns (2 * buf + j) * N

  if (warp == 0) {
    // ------------------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_a =
          (p.weights_once && MIMO_TC_WEIGHT_EVICT_FIRST) ? l2_evict_first_policy() : l2_evict_normal_policy();
      const uint64_t pol_b = l2_evict_normal_policy();
      for (int m = 0; m < NM; ++m) {
        tma_prefetch_map(&p.amap[m]);
        tma_prefetch_map(&p.smap[m]);
      }
      tma_prefetch_map(&p.bmap);
      tma_prefetch_map(&p.bsmap);
      int stage = 0;
      uint32_t ph = 0;
      long long issued = 0, groups = 0;
      bool stop = false;
      // Per item: coordinates, slot and row base once; per stage only the ring bookkeeping.
      for (long long n = 0; n < my_items && !stop; ++n) {
        const long long it = blockIdx.x + n * gridDim.x;
        int unit, tile;
        item_coords(p, it, unit, tile);
        int slot = __ldg(p.unit_slot + unit);
        if (slot < 0 || slot >= p.S) {
          set_status(p.status, MIMO_ERANGE);
          slot = 0;
        }
        const int row0 = slot * p.Nw + tile * TROWS;
        const int brow = p.btok ? 0 : unit * N;
        if (early) {  // the unit's h must be complete: every gate/up epilogue warp of its tiles signalled
          bool ok = fz::ld_acquire(p.ready + unit) >= p.ready_need;
          if (!ok) {
            const uint64_t t0 = global_timer_ns();
            while (!(ok = fz::ld_acquire(p.ready + unit) >= p.ready_need)) {
              if (*s_abort || global_timer_ns() - t0 > 2000000000ull) break;
              __nanosleep(64);
            }
          }
          if (!ok) {
            set_status(p.status, MIMO_ETIMEOUT);
            *s_abort = 1;
            break;
          }
          fz::fence_proxy_async_global();  // h was written by generic stores; TMA reads it
        }
        for (int ks = 0; ks < ns; ++ks) {
          if (*s_abort) {
            stop = true;
            break;
          }
          const int kc = ks * KPS;  // first K chunk of the stage
          if ((kc & 3) == 0) {      // scale boxes for chunks kc..kc+3: 16 bytes of each row
            const int e = (int)(groups & 1);
            if (!mbar_wait(&sc_empty[e], (uint32_t)(((groups >> 1) & 1) ^ 1))) {
              set_status(p.status, MIMO_ETIMEOUT);
              *s_abort = 1;
              stop = true;
              break;
            }
            uint8_t* sc = scbox + e * SCB;
            mbar_arrive_expect_tx(&sc_full[e], NM * kM * 16 + N * 16);
            for (int m = 0; m < NM; ++m)
              tma_load_2d(sc + m * kM * 16, &p.smap[m], kc * 4, row0 + m * MROW, &sc_full[e], pol_b);
            tma_load_2d(sc + NM * kM * 16, &p.bsmap, kc * 4, brow, &sc_full[e], pol_b);
            ++groups;
          }
          if (!mbar_wait(&empty[stage], ph ^ 1u)) {
            set_status(p.status, MIMO_ETIMEOUT);
            *s_abort = 1;
            stop = true;
            break;
          }
          uint8_t* sb = stages + stage * SB;
          mbar_arrive_expect_tx(&full[stage], 2 * kAGlobal + KPS * N * kKC);
          if constexpr (KPS == 1) {
            tma_load_2d(sb, &p.amap[0], kc * kKC, row0, &full[stage], pol_a);
            tma_load_2d(sb + kATile, &p.amap[1], kc * kKC, row0 + MROW, &full[stage], pol_a);
            tma_load_2d(sb + 2 * kATile, &p.bmap, kc * kKC, brow, &full[stage], pol_b);
          } else {  // 3-D boxes [2 chunks][rows][128 B]: both chunks' tiles in one copy each
            tma_load_3d(sb, &p.amap[0], 0, row0, kc, &full[stage], pol_a);
            tma_load_3d(sb + 2 * kATile, &p.bmap, 0, brow, kc, &full[stage], pol_b);
          }
          ++issued;
          if (++stage == NSTAGE) {
            stage = 0;
            ph ^= 1u;
          }
        }
      }
      // Shared memory must not be released with copies still landing.
      bool ok = true;
      for (long long k = 0; ok && k < (issued < NSTAGE ? issued : NSTAGE); ++k) {
        const long long f = issued - 1 - k;
        ok = mbar_wait(&full[(int)(f % NSTAGE)], (uint32_t)((f / NSTAGE) & 1));
      }
      for (long long k = 0; ok && k < (groups < 2 ? groups : 2); ++k) {
        const long long g = groups - 1 - k;
        ok = mbar_wait(&sc_full[(int)(g & 1)], (uint32_t)((g >> 1) & 1));
      }
      if (!ok) set_status(p.status, MIMO_ETIMEOUT);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------ scale-factor builder
    // From the landed boxes ([row][16 B], chunk c at bytes 4c..4c+3), lane l writes 16-byte row l of
    // each 512-byte block: the chunk's 4 bytes for rows l, l+32, l+64, l+96.  Blocks of a stage:
    // [weight scales of slot 0 | slot 1 | activation scales of chunk 0 (| chunk 1)].
    int stage = 0;
    uint32_t ph = 0;
    for (long long s = 0; s < nsteps; ++s) {
      if (*s_abort) break;
      const uint32_t kc = (uint32_t)(s * KPS);  // running chunk index; groups of 4 align with items
      const int c = (int)(kc & 3);
      const uint32_t g = kc >> 2;
      const int e = (int)(g & 1);
      if (c == 0 && !mbar_wait(&sc_full[e], (g >> 1) & 1)) {
        if (lane == 0) set_status(p.status, MIMO_ETIMEOUT);
        *s_abort = 1;
        break;
      }
      if (!mbar_wait(&empty[stage], ph ^ 1u)) {
        if (lane == 0) set_status(p.status, MIMO_ETIMEOUT);
        *s_abort = 1;
        break;
      }
      const uint8_t* sc = scbox + e * SCB;
      uint8_t* blk = sfblk + stage * SFB;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int m = NM == 2 ? j : 0, cj = c + (KPS == 2 ? j : 0);
        const uint8_t* box = sc + m * kM * 16 + cj * 4;
        uint4 v;
        v.x = *reinterpret_cast<const uint32_t*>(box + (lane + 0) * 16);
        v.y = *reinterpret_cast<const uint32_t*>(box + (lane + 32) * 16);
        v.z = *reinterpret_cast<const uint32_t*>(box + (lane + 64) * 16);
        v.w = *reinterpret_cast<const uint32_t*>(box + (lane + 96) * 16);
        *reinterpret_cast<uint4*>(blk + j * 512 + lane * 16) = v;
      }
#pragma unroll
      for (int j = 0; j < KPS; ++j) {
        const uint8_t* box = sc + NM * kM * 16 + (c + j) * 4;
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int n = lane + 32 * q;
          w[q] = n < N ? *reinterpret_cast<const uint32_t*>(box + n * 16) : 0x7F7F7F7Fu;
        }
        *reinterpret_cast<uint4*>(blk + (2 + j) * 512 + lane * 16) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&full[stage]);
        if (c + KPS == 4) mbar_arrive(&sc_empty[e]);
      }
      if (++stage == NSTAGE) {
        stage = 0;
        ph ^= 1u;
      }
    }
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------------------------ MMA issuers
    // One issuing thread runs tcgen05.mma at ~77 cycles per instruction at small N; two overlap.
    // Issuer j owns slot j of every stage (gate / up matrix, or the stage's first / second K chunk
    // of down) and accumulator j of each buffer (the epilogue adds the two partial sums for down).
    // Each copies the scales its own MMAs read, so no ordering is needed between the two threads.
    const int j = warp - 2;
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0;
      bool aborted = false;
      for (long long n = 0; n < my_items && !aborted; ++n) {
        const int buf = ABUF == 2 ? (int)(n & 1) : 0;
        const uint32_t use = ABUF == 2 ? (uint32_t)((n >> 1) & 1) : (uint32_t)(n & 1);
        if (!mbar_wait(&acc_empty[buf], use ^ 1u)) {
          set_status(p.status, MIMO_ETIMEOUT);
          *s_abort = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tbase + (uint32_t)(2 * buf + j) * N;
        for (int ks = 0; ks < ns; ++ks) {
          if (!mbar_wait(&full[stage], ph)) {
            set_status(p.status, MIMO_ETIMEOUT);
            *s_abort = 1;
            aborted = true;
            break;
          }
          tc_fence_after();
          const uint32_t sb = smem_u32(stages + stage * SB);
          const uint32_t blk = smem_u32(sfblk + stage * SFB);
          const uint32_t sf_col = tbase + kSfCol0 + (uint32_t)stage * 16 + 8 * j;
          const int bj = KPS == 2 ? j : 0;  // activation tile / scale block of this slot's chunk
          tc_cp_sf(sf_col, desc_sf(blk + j * 512));             // weight scales of the slot
          tc_cp_sf(sf_col + 4, desc_sf(blk + (2 + bj) * 512));  // activation scales of its chunk
          const uint32_t a0 = sb + j * kATile, b0 = sb + 2 * kATile + bj * N * kKC;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc_mma_mx(d, desc_sw128(a0 + kk * 32), desc_sw128(b0 + kk * 32), idesc_mx(N, kk),
                      sf_col | ((uint32_t)kk << 30), (sf_col + 4) | ((uint32_t)kk << 30), (ks | kk) != 0);
          tc_commit(&empty[stage]);
          if (++stage == NSTAGE) {
            stage = 0;
            ph ^= 1u;
          }
        }
        if (!aborted) tc_commit(&acc_full[buf]);
      }
      // Nothing may still read shared memory or TMEM when the CTA releases them.
      tc_commit(drain);
      if (!mbar_wait(drain, 0)) set_status(p.status, MIMO_ETIMEOUT);
    }
  } else if (warp >= 4) {
    // --------------------------------------------------------------------------------- epilogue
    const int quad = warp & 3;                     // TMEM lanes this warp may read
    const int qlo = ((warp - 4) >> 2) * QH;        // its half of the routes: [qlo, qlo + QH)
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    bool aborted = false;
    for (long long n = 0; n < my_items; ++n) {
      const long long it = blockIdx.x + n * gridDim.x;
      const int buf = ABUF == 2 ? (int)(n & 1) : 0;
      const uint32_t use = ABUF == 2 ? (uint32_t)((n >> 1) & 1) : (uint32_t)(n & 1);
      int unit, tile;
      item_coords(p, it, unit, tile);
      const int slot = __ldg(p.unit_slot + unit);
      const int cnt = unit_routes(p, unit, NTOK);
      const int p0 = p.unit_p0 ? __ldg(p.unit_p0 + unit) : unit * p.p0_stride;
      if (!aborted && !mbar_wait(&acc_full[buf], use)) {
        set_status(p.status, MIMO_ETIMEOUT);
        aborted = true;
      }
      tc_fence_after();
      const bool live = !aborted && slot >= 0 && slot < p.S;
      const int row = tile * TROWS + quad * 32 + lane;  // output feature of this lane (slot 0's row)
      if (MODE == 0 && live && p.btok) {
        // Columns are tokens: route q reads its token's hi/lo columns.
#pragma unroll 1
        for (int q = qlo; q < qlo + QH; ++q) {
          float h = 0.f;
          if (q < cnt) {
            const int t = __ldg(p.btok + p0 + q);
            if (t >= 0 && t < (p.btok_rows > 0 ? min(p.btok_rows, NTOK) : NTOK)) {
              float gh[1], gl[1], uh[1], ul[1];
              const uint32_t c0 = tbase + lane_base + (uint32_t)(2 * buf) * N + t;
              tmem_ld<1>(c0, gh);
              tmem_ld<1>(c0 + NTOK, gl);
              tmem_ld<1>(c0 + N, uh);
              tmem_ld<1>(c0 + N + NTOK, ul);
              tmem_wait_ld();
              h = swiglu_ref(gh[0] + gl[0], uh[0] + ul[0]);
              if (!isfinite(h)) set_status(p.status, MIMO_ERANGE);
            } else if (lane == 0) {
              set_status(p.status, MIMO_ERANGE);
            }
          }
          uint32_t th, tl, b1, b2;
          split_warp_block(h, th, tl, b1, b2);
          const size_t rh = (size_t)unit * N + q, rl = rh + NTOK;
          p.hq[rh * p.Nw + row] = (uint8_t)th;
          p.hq[rl * p.Nw + row] = (uint8_t)tl;
          if (lane == 0) {
            p.hs[rh * (p.Nw / 32) + row / 32] = (uint8_t)b1;
            p.hs[rl * (p.Nw / 32) + row / 32] = (uint8_t)b2;
          }
        }
      }
      // One route's outputs from accumulators 0 / 1 (gate / up, or the two K halves of down), each
      // as its hi and lo term columns.  MODE 0 is warp-collective (block maxima over the lanes).
      auto emit = [&](int q, float h0, float h1, float l0, float l1) {
        if constexpr (MODE == 0) {
          float h = 0.f;
          if (q < cnt) {
            h = swiglu_ref(h0 + l0, h1 + l1);
            if (!isfinite(h)) set_status(p.status, MIMO_ERANGE);
          }
          uint32_t th, tl, b1, b2;
          split_warp_block(h, th, tl, b1, b2);
          const size_t rh = (size_t)unit * N + q, rl = rh + NTOK;
          p.hq[rh * p.Nw + row] = (uint8_t)th;
          p.hq[rl * p.Nw + row] = (uint8_t)tl;
          if (lane == 0) {
            p.hs[rh * (p.Nw / 32) + row / 32] = (uint8_t)b1;
            p.hs[rl * (p.Nw / 32) + row / 32] = (uint8_t)b2;
          }
        } else if constexpr (MODE == 3) {
          if (q < cnt) {  // two rows: slot 0's and slot 1's, each hi + lo
            const int orow = p.out_row ? __ldg(p.out_row + p0 + q) : p0 + q;
            const float w = __ldg(p.rw + p0 + q);
            const float d0 = h0 + l0, d1 = h1 + l1;
            const float v0 = (p.pairs_rounding ? bf16_round(d0) : d0) * w;
            const float v1 = (p.pairs_rounding ? bf16_round(d1) : d1) * w;
            float* dst = p.peer_part ? p.peer_part[orow / p.peer_rows] + (size_t)(orow % p.peer_rows) * p.Nw
                                     : p.part + (size_t)orow * p.Nw;
            dst[row] = v0;
            dst[row + kM] = v1;
          }
        } else if constexpr (MODE == 4) {
          if (q < cnt) {  // bf16 pair outputs of the two rows (model.py:221-228)
            uint16_t* dst = p.ypair + (size_t)(p0 + q) * p.Nw;
            dst[row] = (uint16_t)f32_to_bf16(h0 + l0);
            dst[row + kM] = (uint16_t)f32_to_bf16(h1 + l1);
          }
        } else {
          if (q < cnt) {
            const float d = (h0 + l0) + (h1 + l1);  // each K half's hi + lo, then the halves
            const int orow = MODE == 1 && p.out_row ? __ldg(p.out_row + p0 + q) : p0 + q;
            if constexpr (MODE == 1) {
              const float v = (p.pairs_rounding ? bf16_round(d) : d) * __ldg(p.rw + p0 + q);
              if (p.peer_part)  // straight into the owner rank's receive buffer (NVLink store)
                p.peer_part[orow / p.peer_rows][(size_t)(orow % p.peer_rows) * p.Nw + row] = v;
              else
                p.part[(size_t)orow * p.Nw + row] = v;
            } else {
              const size_t op = (size_t)orow * p.Nw + row;
              p.ypair[op] = (uint16_t)f32_to_bf16(d);
            }
          }
        }
      };
      const bool chunks = live && !(MODE == 0 && p.btok);
      if constexpr (ABUF == 2) {
#pragma unroll 1
        for (int q0 = qlo; q0 < qlo + QH && chunks; q0 += QC) {
          float hi[2][QC], lo[2][QC];  // accumulators 0 and 1 of the buffer
#pragma unroll
          for (int a = 0; a < 2; ++a) {
            const uint32_t c = tbase + lane_base + (uint32_t)(2 * buf + a) * N + q0;
            tmem_ld<QC>(c, hi[a]);
            tmem_ld<QC>(c + NTOK, lo[a]);
          }
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < QC; ++i) emit(q0 + i, hi[0][i], hi[1][i], lo[0][i], lo[1][i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
      } else {
        // Single buffer: copy all of this warp's columns out, free the accumulator, then compute.
        float hv[2][QH], lv[2][QH];
        if (chunks) {
#pragma unroll
          for (int q0 = 0; q0 < QH; q0 += QC) {
#pragma unroll
            for (int a = 0; a < 2; ++a) {
              float th[QC], tl[QC];
              const uint32_t c = tbase + lane_base + (uint32_t)(2 * buf + a) * N + qlo + q0;
              tmem_ld<QC>(c, th);
              tmem_ld<QC>(c + NTOK, tl);
#pragma unroll
              for (int i = 0; i < QC; ++i) {
                hv[a][q0 + i] = th[i];
                lv[a][q0 + i] = tl[i];
              }
            }
          }
          tmem_wait_ld();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
        if (chunks) {
#pragma unroll
          for (int i = 0; i < QH; ++i) emit(qlo + i, hv[0][i], hv[1][i], lv[0][i], lv[1][i]);
        }
      }
      if constexpr (MODE == 1) {
        if (p.cy) combine_tile(p, tile, units, warp - 4, lane, EPI, s_abort + 1);
      }
      if constexpr (MODE == 0) {
        if (p.ready) {  // publish this warp's share of the unit's h (every item, so no wait is left open)
          __threadfence();
          fz::fence_proxy_async_global();
          __syncwarp();
          if (lane == 0) atomicAdd(p.ready + unit, 1);
        }
      }
    }
    if constexpr (MODE == 1) {  // no units: no tile completes, and the sum over no routes is 0
      if (p.cy && units == 0 && blockIdx.x == 0)
        for (int o = (warp - 4) * 32 + lane; o < p.cM * p.Nw; o += EPI * 32) p.cy[o] = 0;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 3) {
    tc_fence_after();
    tmem_dealloc(tbase, TCOLS);
  }
}

// ------------------------------------------------------------------- fused decode (gate/up -> down)
// One persistent launch runs both passes of a decode call.  Work items: the gate/up tiles (unit,
// 128 rows of I; 2 matrices x K = H) and the down tiles (unit, 128 rows of H; K = I).  CTA c takes
// its gate/up tiles c, c + G, ... first, then its down tiles; the down tiles are dealt from the CTA
// after the last one that got an extra gate/up tile, so the CTAs with less gate/up work start down
// work first.  A down tile needs the unit's whole h: every gate/up epilogue warp adds 1 to
// ready[unit] after its h stores (8 warps x I/128 tiles per unit), and the producer waits for that
// count (acquire, bounded) before loading the unit's h terms.  Each CTA finishes issuing its gate/up
// tiles before it waits on any unit, and the grid is one CTA per SM (all resident), so every wait
// ends; a wait that outlasts the limit sets MIMO_ETIMEOUT and the CTA drains and returns.
//
// Two operand formats (template FP4):
//   FP4 = false  kind::mxf8f6f4: weights in the padded e2m1 layout (16 KiB per 128 x 128 tile in shared
//                memory for 8 KiB of weights), activations as two e4m3 terms (N = 16);
//   FP4 = true   kind::mxf4: weights packed as stored (8 KiB per tile, 64B swizzle), activations as five
//                e2m1 terms (N = 40).  Twice the weight bytes fit in the same shared memory, so each SM
//                keeps about twice as many weight bytes in flight, which is what bounds decode: an
//                SM's streaming rate is its bytes in flight over the memory latency.
static_assert(kFp4Terms == kTcFp4Terms, "term count");
namespace fz {
template <bool FP4>
struct Fmt {
  static constexpr int kTerms = FP4 ? kFp4Terms : 2;
  static constexpr int kN = kTerms * kTcDecodeRoutes;       // MMA N: 8 routes x terms
  static constexpr int kATileS = FP4 ? kM * kKC / 2 : kATile;  // shared bytes of one weight tile
  static constexpr int kBRow = FP4 ? kKC / 2 : kKC;          // bytes of one term row per K chunk
  static constexpr int kBTile = kN * kBRow;
  static constexpr int kSB = 2 * kATileS + 2 * kBTile;       // stage: 2 A tiles + up to 2 B tiles
  static constexpr int kSCB = 2 * kM * 16 + kN * 16;         // scale boxes of one 4-chunk group
  static constexpr int kSFB = 4 * 512;                        // scale blocks of one stage
  static_assert(kSB % 1024 == 0 || (FP4 && kSB % 512 == 0), "tile alignment");
};
template <int NSTAGE, bool FP4>
constexpr int smem_bytes() {
  using F = Fmt<FP4>;
  return kBarBytes + 1024 + NSTAGE * F::kSB + 2 * F::kSCB + NSTAGE * F::kSFB;
}

struct Sched {
  int tiles_gu, tiles_dn, ns_gu, ns_dn;  // tiles per unit; stages per item
  long long my_gu, my_dn, cdn;           // this CTA's item counts; its first down item
  __device__ __forceinline__ long long items() const { return my_gu + my_dn; }
  // item n of this CTA -> (down?, unit, tile)
  __device__ __forceinline__ void at(long long n, bool& dn, int& unit, int& tile) const {
    if (n < my_gu) {
      const long long i = blockIdx.x + n * gridDim.x;
      dn = false;
      unit = (int)(i / tiles_gu);
      tile = (int)(i % tiles_gu);
    } else {
      const long long j = cdn + (n - my_gu) * gridDim.x;
      dn = true;
      unit = (int)(j / tiles_dn);
      tile = (int)(j % tiles_dn);
    }
  }
};

__device__ __forceinline__ Sched schedule(const TcParams& gu, const TcParams& dn, int units) {
  Sched s;
  s.tiles_gu = gu.tiles;
  s.tiles_dn = dn.tiles;
  s.ns_gu = gu.K / kKC;
  s.ns_dn = dn.K / (2 * kKC);
  const long long G = gridDim.x, c = blockIdx.x;
  const long long n_gu = (long long)units * gu.tiles, n_dn = (long long)units * dn.tiles;
  s.my_gu = n_gu > c ? (n_gu - c + G - 1) / G : 0;
  s.cdn = (c - n_gu % G + G) % G;
  s.my_dn = n_dn > s.cdn ? (n_dn - s.cdn + G - 1) / G : 0;
  return s;
}

}  // namespace fz

template <int NSTAGE, bool FP4>
__global__ void __launch_bounds__(kThreads, 1) tc_decode_fused_kernel(const __grid_constant__ TcFusedParams f) {
  using F = fz::Fmt<FP4>;
  constexpr int NTOK = kTcDecodeRoutes, N = F::kN, NT = F::kTerms;
  constexpr int SB = F::kSB, SCB = F::kSCB, SFB = F::kSFB, AT = F::kATileS, BT = F::kBTile;
  constexpr uint32_t TCOLS = tmem_cols<N, NSTAGE>();
  constexpr int ABUF = abuf<N, NSTAGE>();
  constexpr int QH = NTOK / 2;
  static_assert(ABUF == 2, "double-buffered accumulators");
  const TcParams& g = f.gu;
  const TcParams& d = f.dn;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + NSTAGE;
  uint64_t* sc_full = empty + NSTAGE;
  uint64_t* sc_empty = sc_full + 2;
  uint64_t* acc_full = sc_empty + 2;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* base = reinterpret_cast<uint8_t*>(((uintptr_t)(smem + kBarBytes) + 1023) & ~(uintptr_t)1023);
  uint8_t* stages = base;
  uint8_t* scbox = stages + NSTAGE * SB;
  uint8_t* sfblk = scbox + 2 * SCB;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NSTAGE; ++i) {
      mbar_init(&full[i], 2);
      mbar_init(&empty[i], 2);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sc_full[b], 1);
      mbar_init(&sc_empty[b], 1);
      mbar_init(&acc_full[b], 2);
      mbar_init(&acc_empty[b], kEpiWarps);
    }
    mbar_init(drain, 2);
    *s_abort = 0;
    mbar_fence_init();
  }
  if (warp == 3) {
    tmem_alloc(tmem_slot, TCOLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();  // the unit tables and activation terms come from the preceding kernel
  pdl_launch_dependents();
  const uint32_t tbase = *tmem_slot;
  constexpr uint32_t kSfCol0 = ABUF * 2 * N;
  // after the wait: the unit count is written by the preceding kernel
  const int units = g.num_units ? min(__ldg(g.num_units), g.units_cap) : g.units_cap;
  const fz::Sched sch = fz::schedule(g, d, units);
  const long long my_items = sch.items();
  const int ready_target = kEpiWarps * g.tiles;


  if (warp == 0) {
    // ------------------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_a = MIMO_TC_WEIGHT_EVICT_FIRST ? l2_evict_first_policy() : l2_evict_normal_policy();
      const uint64_t pol_b = l2_evict_normal_policy();
      for (int m = 0; m < 2; ++m) {
        tma_prefetch_map(&g.amap[m]);
        tma_prefetch_map(&g.smap[m]);
      }
      tma_prefetch_map(&g.bmap);
      tma_prefetch_map(&g.bsmap);
      tma_prefetch_map(&d.amap[0]);
      tma_prefetch_map(&d.smap[0]);
      tma_prefetch_map(&d.bmap);
      tma_prefetch_map(&d.bsmap);
      int stage = 0;
      uint32_t ph = 0;
      long long issued = 0, groups = 0;
      bool stop = false;
      for (long long n = 0; n < my_items && !stop; ++n) {
        bool dn;
        int unit, tile;
        sch.at(n, dn, unit, tile);
        const TcParams& p = dn ? d : g;
        int slot = __ldg(p.unit_slot + unit);
        if (slot < 0 || slot >= p.S) {
          set_status(p.status, MIMO_ERANGE);
          slot = 0;
        }
        if (dn) {  // the unit's h must be complete: all its gate/up epilogue warps have signalled
          bool ok = fz::ld_acquire(f.ready + unit) >= ready_target;
          if (!ok) {
            const uint64_t t0 = global_timer_ns();
            while (!(ok = fz::ld_acquire(f.ready + unit) >= ready_target)) {
              if (*s_abort || global_timer_ns() - t0 > 2000000000ull) break;
              __nanosleep(64);
            }
          }
          if (!ok) {
            set_status(p.status, MIMO_ETIMEOUT);
            *s_abort = 1;
            break;
          }
          fz::fence_proxy_async_global();  // h was written by generic stores; TMA reads it
        }
        const int NM = dn ? 1 : 2, KPS = dn ? 2 : 1;
        const int ns = dn ? sch.ns_dn : sch.ns_gu;
        const int row0 = slot * p.Nw + tile * kM;
        const int brow = (!dn && p.btok) ? 0 : unit * N;
        for (int ks = 0; ks < ns; ++ks) {
          if (*s_abort) {
            stop = true;
            break;
          }
          const int kc = ks * KPS;
          if ((kc & 3) == 0) {
            const int e = (int)(groups & 1);
            if (!mbar_wait(&sc_empty[e], (uint32_t)(((groups >> 1) & 1) ^ 1))) {
              set_status(p.status, MIMO_ETIMEOUT);
              *s_abort = 1;
              stop = true;
              break;
            }
            uint8_t* sc = scbox + e * SCB;
            mbar_arrive_expect_tx(&sc_full[e], NM * kM * 16 + N * 16);
            for (int m = 0; m < NM; ++m) tma_load_2d(sc + m * kM * 16, &p.smap[m], kc * 4, row0, &sc_full[e], pol_b);
            tma_load_2d(sc + NM * kM * 16, &p.bsmap, kc * 4, brow, &sc_full[e], pol_b);
            ++groups;
          }
          if (!mbar_wait(&empty[stage], ph ^ 1u)) {
            set_status(p.status, MIMO_ETIMEOUT);
            *s_abort = 1;
            stop = true;
            break;
          }
          uint8_t* sb = stages + stage * SB;
          mbar_arrive_expect_tx(&full[stage], 2 * kAGlobal + KPS * BT);
          if constexpr (FP4) {  // 2-D boxes of 64 bytes (128 values) per row
            if (!dn) {
              tma_load_2d(sb, &p.amap[0], kc * 64, row0, &full[stage], pol_a);
              tma_load_2d(sb + AT, &p.amap[1], kc * 64, row0, &full[stage], pol_a);
              tma_load_2d(sb + 2 * AT, &p.bmap, kc * 64, brow, &full[stage], pol_b);
            } else {
              for (int c = 0; c < 2; ++c) {
                tma_load_2d(sb + c * AT, &p.amap[0], (kc + c) * 64, row0, &full[stage], pol_a);
                tma_load_2d(sb + 2 * AT + c * BT, &p.bmap, (kc + c) * 64, brow, &full[stage], pol_b);
              }
            }
          } else {
            if (!dn) {
              tma_load_2d(sb, &p.amap[0], kc * kKC, row0, &full[stage], pol_a);
              tma_load_2d(sb + kATile, &p.amap[1], kc * kKC, row0, &full[stage], pol_a);
              tma_load_2d(sb + 2 * kATile, &p.bmap, kc * kKC, brow, &full[stage], pol_b);
            } else {
              tma_load_3d(sb, &p.amap[0], 0, row0, kc, &full[stage], pol_a);
              tma_load_3d(sb + 2 * kATile, &p.bmap, 0, brow, kc, &full[stage], pol_b);
            }
          }
          ++issued;
          if (++stage == NSTAGE) {
            stage = 0;
            ph ^= 1u;
          }
        }
      }
      bool ok = true;
      for (long long k = 0; ok && k < (issued < NSTAGE ? issued : NSTAGE); ++k) {
        const long long q = issued - 1 - k;
        ok = mbar_wait(&full[(int)(q % NSTAGE)], (uint32_t)((q / NSTAGE) & 1));
      }
      for (long long k = 0; ok && k < (groups < 2 ? groups : 2); ++k) {
        const long long q = groups - 1 - k;
        ok = mbar_wait(&sc_full[(int)(q & 1)], (uint32_t)((q >> 1) & 1));
      }
      if (!ok) set_status(g.status, MIMO_ETIMEOUT);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------ scale-factor builder
    int stage = 0;
    uint32_t ph = 0;
    uint32_t grp = 0;  // running 4-chunk group
    bool stop = false;
    for (long long n = 0; n < my_items && !stop; ++n) {
      bool dn;
      int unit, tile;
      sch.at(n, dn, unit, tile);
      const int NM = dn ? 1 : 2, KPS = dn ? 2 : 1;
      const int ns = dn ? sch.ns_dn : sch.ns_gu;
      for (int ks = 0; ks < ns; ++ks) {
        if (*s_abort) {
          stop = true;
          break;
        }
        const int c = (ks * KPS) & 3;
        const int e = (int)(grp & 1);
        if (c == 0 && !mbar_wait(&sc_full[e], (grp >> 1) & 1)) {
          if (lane == 0) set_status(g.status, MIMO_ETIMEOUT);
          *s_abort = 1;
          stop = true;
          break;
        }
        if (!mbar_wait(&empty[stage], ph ^ 1u)) {
          if (lane == 0) set_status(g.status, MIMO_ETIMEOUT);
          *s_abort = 1;
          stop = true;
          break;
        }
        const uint8_t* sc = scbox + e * SCB;
        uint8_t* blk = sfblk + stage * SFB;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int m = NM == 2 ? j : 0, cj = c + (KPS == 2 ? j : 0);
          const uint8_t* box = sc + m * kM * 16 + cj * 4;
          uint4 v;
          v.x = *reinterpret_cast<const uint32_t*>(box + (lane + 0) * 16);
          v.y = *reinterpret_cast<const uint32_t*>(box + (lane + 32) * 16);
          v.z = *reinterpret_cast<const uint32_t*>(box + (lane + 64) * 16);
          v.w = *reinterpret_cast<const uint32_t*>(box + (lane + 96) * 16);
          *reinterpret_cast<uint4*>(blk + j * 512 + lane * 16) = v;
        }
        for (int j = 0; j < KPS; ++j) {
          const uint8_t* box = sc + NM * kM * 16 + (c + j) * 4;
          uint32_t w[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int r = lane + 32 * q;
            w[q] = r < N ? *reinterpret_cast<const uint32_t*>(box + r * 16) : 0x7F7F7F7Fu;
          }
          *reinterpret_cast<uint4*>(blk + (2 + j) * 512 + lane * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&full[stage]);
          if (c + KPS == 4) mbar_arrive(&sc_empty[e]);
        }
        if (c + KPS == 4) ++grp;
        if (++stage == NSTAGE) {
          stage = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------------------------ MMA issuers
    const int j = warp - 2;
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0;
      bool aborted = false;
      for (long long n = 0; n < my_items && !aborted; ++n) {
        bool dn;
        int unit, tile;
        sch.at(n, dn, unit, tile);
        const int KPS = dn ? 2 : 1;
        const int ns = dn ? sch.ns_dn : sch.ns_gu;
        const int buf = (int)(n & 1);
        const uint32_t use = (uint32_t)((n >> 1) & 1);
        if (!mbar_wait(&acc_empty[buf], use ^ 1u)) {
          set_status(g.status, MIMO_ETIMEOUT);
          *s_abort = 1;
          break;
        }
        tc_fence_after();
        const uint32_t dacc = tbase + (uint32_t)(2 * buf + j) * N;
        for (int ks = 0; ks < ns; ++ks) {
          if (!mbar_wait(&full[stage], ph)) {
            set_status(g.status, MIMO_ETIMEOUT);
            *s_abort = 1;
            aborted = true;
            break;
          }
          tc_fence_after();
          const uint32_t sb = smem_u32(stages + stage * SB);
          const uint32_t blk = smem_u32(sfblk + stage * SFB);
          const uint32_t sf_col = tbase + kSfCol0 + (uint32_t)stage * 16 + 8 * j;
          const int bj = KPS == 2 ? j : 0;
          tc_cp_sf(sf_col, desc_sf(blk + j * 512));
          tc_cp_sf(sf_col + 4, desc_sf(blk + (2 + bj) * 512));
          const uint32_t a0 = sb + j * AT, b0 = sb + 2 * AT + bj * BT;
          if constexpr (FP4) {  // 2 MMAs of K = 64: scale bytes 0-1, then 2-3 of each row's cell
#pragma unroll
            for (int kk = 0; kk < 2; ++kk)
              tc_mma_mxf4(dacc, desc_sw64(a0 + kk * 32), desc_sw64(b0 + kk * 32), idesc_mxf4(kM, N, 2 * kk),
                          sf_col | ((uint32_t)(2 * kk) << 30), (sf_col + 4) | ((uint32_t)(2 * kk) << 30),
                          (ks | kk) != 0);
          } else {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              tc_mma_mx(dacc, desc_sw128(a0 + kk * 32), desc_sw128(b0 + kk * 32), idesc_mx(N, kk),
                        sf_col | ((uint32_t)kk << 30), (sf_col + 4) | ((uint32_t)kk << 30), (ks | kk) != 0);
          }
          tc_commit(&empty[stage]);
          if (++stage == NSTAGE) {
            stage = 0;
            ph ^= 1u;
          }
        }
        if (!aborted) tc_commit(&acc_full[buf]);
      }
      tc_commit(drain);
      if (!mbar_wait(drain, 0)) set_status(g.status, MIMO_ETIMEOUT);
    }
  } else if (warp >= 4) {
    // --------------------------------------------------------------------------------- epilogue
    const int quad = warp & 3;
    const int qlo = ((warp - 4) >> 2) * QH;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    bool aborted = false;
    for (long long n = 0; n < my_items; ++n) {
      bool dn;
      int unit, tile;
      sch.at(n, dn, unit, tile);
      const TcParams& p = dn ? d : g;
      const int buf = (int)(n & 1);
      const uint32_t use = (uint32_t)((n >> 1) & 1);
      const int slot = __ldg(p.unit_slot + unit);
      const int cnt = unit_routes(p, unit, NTOK);
      const int p0 = p.unit_p0 ? __ldg(p.unit_p0 + unit) : unit * p.p0_stride;
      if (!aborted && !mbar_wait(&acc_full[buf], use)) {
        set_status(g.status, MIMO_ETIMEOUT);
        aborted = true;
      }
      tc_fence_after();
      const bool live = !aborted && slot >= 0 && slot < p.S;
      const int row = tile * kM + quad * 32 + lane;
      // Per accumulator a and MMA column c (a route, or a token when B rows are tokens): the sum of
      // its term columns c, 8 + c, ... in term order.
      float acc[2][NTOK];
      if (live) {
#pragma unroll
        for (int a = 0; a < 2; ++a) {
          float t8[NTOK];
          const uint32_t col = tbase + lane_base + (uint32_t)(2 * buf + a) * N;
          tmem_ld<NTOK>(col, t8);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < NTOK; ++c) acc[a][c] = t8[c];
#pragma unroll
          for (int t = 1; t < NT; ++t) {
            tmem_ld<NTOK>(col + t * NTOK, t8);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < NTOK; ++c) acc[a][c] += t8[c];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      if (live) {
#pragma unroll 1
        for (int q = qlo; q < qlo + QH; ++q) {
          int col = q;  // B rows per route; with by-token rows, route q's token
          bool ok = q < cnt;
          if (!dn && g.btok && ok) {
            col = __ldg(g.btok + p0 + q);
            if (col < 0 || col >= (g.btok_rows > 0 ? min(g.btok_rows, NTOK) : NTOK)) {
              if (lane == 0) set_status(g.status, MIMO_ERANGE);
              ok = false;
              col = 0;
            }
          }
          float a0 = 0.f, a1 = 0.f;
#pragma unroll
          for (int c = 0; c < NTOK; ++c)
            if (c == col) {
              a0 = acc[0][c];
              a1 = acc[1][c];
            }
          if (!dn) {
            // gate/up: SwiGLU with the reference's roundings (kernels.py:79-82), then h as the down
            // pass's activation terms
            float h = 0.f;
            if (ok) {
              h = swiglu_ref(a0, a1);
              if (!isfinite(h)) set_status(g.status, MIMO_ERANGE);
            }
            const size_t r0 = (size_t)unit * N + q;  // term t of route q: row r0 + t * NTOK
            if constexpr (FP4) {
#pragma unroll 1
              for (int t = 0; t < NT; ++t) {
                const float amax = __uint_as_float(__reduce_max_sync(0xFFFFFFFFu, __float_as_uint(fabsf(h))));
                const uint32_t b = e2m1_scale_byte(amax);
                const uint32_t code = f32x2_to_e2m1x2(h * inv_exp2_byte(b), 0.f) & 0xFu;
                h -= e2m1x2_to_f32x2(code).x * exp2_byte(b);
                uint32_t word = code << (4 * (lane & 7));  // 8 lanes = 8 values = one 32-bit word
                word |= __shfl_xor_sync(0xFFFFFFFFu, word, 1);
                word |= __shfl_xor_sync(0xFFFFFFFFu, word, 2);
                word |= __shfl_xor_sync(0xFFFFFFFFu, word, 4);
                const size_t rr = r0 + (size_t)t * NTOK;
                if ((lane & 7) == 0) *reinterpret_cast<uint32_t*>(g.hq + rr * (g.Nw / 2) + row / 2) = word;
                if (lane == 0) g.hs[rr * (g.Nw / 32) + row / 32] = (uint8_t)b;
              }
            } else {
              uint32_t th, tl, b1, b2;
              split_warp_block(h, th, tl, b1, b2);
              const size_t rl = r0 + NTOK;
              g.hq[r0 * g.Nw + row] = (uint8_t)th;
              g.hq[rl * g.Nw + row] = (uint8_t)tl;
              if (lane == 0) {
                g.hs[r0 * (g.Nw / 32) + row / 32] = (uint8_t)b1;
                g.hs[rl * (g.Nw / 32) + row / 32] = (uint8_t)b2;
              }
            }
          } else if (ok) {
            // down x route weight (kernels.py:120): the two K halves' partial sums
            const float v0 = a0 + a1;
            const int orow = d.out_row ? __ldg(d.out_row + p0 + q) : p0 + q;
            const float v = (d.pairs_rounding ? bf16_round(v0) : v0) * __ldg(d.rw + p0 + q);
            if (d.peer_part)
              d.peer_part[orow / d.peer_rows][(size_t)(orow % d.peer_rows) * d.Nw + row] = v;
            else
              d.part[(size_t)orow * d.Nw + row] = v;
          }
        }
      }
      if (!dn) {  // publish this warp's share of the unit's h to the down tiles
        __threadfence();
        fz::fence_proxy_async_global();
        __syncwarp();
        if (lane == 0) atomicAdd(f.ready + unit, 1);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 3) {
    tc_fence_after();
    tmem_dealloc(tbase, TCOLS);
  }
}

// ------------------------------------------------------------ stream-K decode (gate/up -> down)
// Both decode passes in one persistent launch with every CTA streaming the same number of weight bytes.
// The unit of work is a K group of 512 values (4 chunks of 128) of one 128-row tile: a gate/up group
// reads 2 x 128 x 512 e2m1 weights (68 KB with scales), a down group 128 x 512 (34 KB).  The gate/up
// groups of all units, in (unit, tile, group) order, are cut into `gridDim.x` contiguous ranges of
// equal length (CTA c takes [n c / G, n (c + 1) / G)), and so are the down groups.  At decode sizes a
// tile-granular schedule leaves SMs idle or doubly loaded (B = 1: 128 gate/up tiles on 148 SMs); the
// group ranges differ by at most one group.
//
// Canonical accumulation.  Each group accumulates in its own TMEM buffer (a ring of kNAcc), and the
// epilogue turns it into q_g = hi + lo per route column (gate and up; for down, the two K-parity
// accumulators' (hi + lo) added).  A tile's value is the right fold q_0 + (q_1 + (... + q_last)) of its
// groups, whichever CTAs computed them, so the result does not depend on where the ranges are cut (it
// is the same for every unit count and grid, hence bit-identical between one GPU and the expert-
// parallel path, which runs this kernel on other unit tables).  Within a tile every CTA streams its
// groups in descending order and folds as they complete.
//
// Hand-off.  A range that starts inside a tile holds that tile's tail: the CTA streams it first, folds
// it and publishes the partial fold R (its epilogue warp w stores its half of the 8 route columns of its
// TMEM lane quadrant into part_{g,d}[cta] and release-stores flag[cta][w] = 1).  The CTA before it,
// whose range ends in the same tile and which therefore reaches the tile last, starts its part of the
// fold from R (acquired with a bounded wait before its first group of the tile; by then R has long been
// written), so a split tile completes as soon as its last group does.  The CTA holding group 0 owns the
// tile and runs its epilogue (SwiGLU + h terms, or down x route weight).  A range that lies inside one
// tile waits for R of its right neighbour before its own fold.
//
// Down after gate/up.  A down group of unit u needs u's whole h: every gate/up tile owner's epilogue
// warps add 1 to ready[u] after their h stores (8 warps x tiles per unit), and the producer acquires
// that count before loading u's h terms.  Once its gate/up stages are issued, the producer asks L2 for
// the first kL2Prefetch bytes of its down weight tiles (HBM is otherwise idle while the gate/up pass
// drains), and while the count is short it still issues the stages' weight tiles and scale boxes and
// defers only the h loads (it flushes them, waiting for the count, before it would block on a ring
// slot those stages hold).  One CTA per SM (all resident) and gate/up before down in every CTA make
// every wait finite; a wait past its limit sets MIMO_ETIMEOUT, the CTA issues what it deferred, drains
// and returns.
namespace sk {
constexpr int kNTOK = kTcDecodeRoutes;           // route (or token) columns per unit
constexpr int kN = 2 * kNTOK;                    // MMA N: the hi and lo term of each column
constexpr int kNAcc = 8;                         // accumulator buffers, one K group each
constexpr int kScRing = 4;                       // scale-box ring entries (one group each)
constexpr int kGroupChunks = kSkGroupK / kKC;    // 4
constexpr int kSB = 2 * kATile + 2 * kN * kKC;   // stage: 2 weight tiles + 1 (gate/up) or 2 (down) term tiles
constexpr int kSCB = 2 * kM * 16 + kN * 16;      // scale boxes of one group
constexpr int kSFB = 4 * 512;                    // scale blocks of one stage
#ifndef MIMO_TC_SK_L2_PREFETCH
#define MIMO_TC_SK_L2_PREFETCH 0  // measured on B200: no gain at B = 1 or 8 (the burst delays the hand-offs)
#endif
#ifndef MIMO_TC_SK_WAVES
#define MIMO_TC_SK_WAVES 1
#endif
constexpr int kL2Prefetch = MIMO_TC_SK_L2_PREFETCH;  // down weight bytes per CTA asked of L2 ahead of time
template <int NSTAGE>
constexpr int smem_bytes() { return kBarBytes + 1024 + NSTAGE * kSB + kScRing * kSCB + NSTAGE * kSFB; }
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSfCol0 = kNAcc * 2 * kN;     // scale-factor columns after the accumulators

// One phase's schedule.  The phase's tiles (unit-major) are dealt in `rounds` full waves, CTA c taking
// whole tiles c, c + G, c + 2G, ... (G = gridDim.x; CTAs side by side work on neighbouring tiles);
// the remaining tiles' groups (from group `base` on) are cut into `parts` contiguous ranges, taken by
// CTAs 0 .. parts - 1 (the others get none).  parts = min(G, groups / (groups per tile / 2)): every
// range holds at least half a tile, so a tile spans at most three ranges and no empty range sits
// between the parts of a tile.
struct Phase {
  long long n;     // stream-K groups (after the full waves)
  long long base;  // first stream-K group
  int gpt;         // groups per tile
  int tiles;       // tiles per unit
  int rounds;      // full waves of whole tiles
  int parts;
  __device__ __forceinline__ void init(long long all_tiles, int groups_per_tile, int tiles_per_unit, bool waves) {
    gpt = groups_per_tile;
    tiles = tiles_per_unit;
    rounds = waves ? (int)(all_tiles / gridDim.x) : 0;
    base = (long long)rounds * gridDim.x * gpt;
    n = all_tiles * gpt - base;
    const long long half = max(1, gpt / 2);
    parts = (int)max(1ll, min((long long)gridDim.x, n / half));
  }
  __device__ __forceinline__ long long start(int c) const { return base + n * min(c, parts) / parts; }
  // the CTA whose stream-K range holds group g (base <= g < base + n)
  __device__ __forceinline__ int cta_of(long long g) const {
    const long long r = g - base;
    int c = (int)(r * parts / n);
    while (c + 1 < parts && start(c + 1) <= g) ++c;
    while (c > 0 && start(c) > g) --c;
    return c;
  }
  // groups this CTA streams in the phase
  __device__ __forceinline__ long long count(int c) const { return (long long)rounds * gpt + start(c + 1) - start(c); }
};
// Segment = the groups of one tile inside a CTA's work, [lo, hi); streamed from hi - 1 down to lo.
struct Seg {
  long long t, t0, lo, hi;  // tile, its first group, the segment's groups
};
// A CTA's segments in order: its whole tiles of the full waves, then its stream-K range by tile.
struct SegIter {
  const Phase* Q;
  int r;
  long long gi, b;
  __device__ __forceinline__ SegIter(const Phase& q, int c) : Q(&q), r(0), gi(q.start(c)), b(q.start(c + 1)) {}
  __device__ __forceinline__ bool next(Seg& s) {
    if (r < Q->rounds) {
      s.t = (long long)r * gridDim.x + blockIdx.x;
      s.t0 = s.t * Q->gpt;
      s.lo = s.t0;
      s.hi = s.t0 + Q->gpt;
      ++r;
      return true;
    }
    if (gi >= b) return false;
    s.t = gi / Q->gpt;
    s.t0 = s.t * Q->gpt;
    s.lo = gi;
    s.hi = min(b, s.t0 + Q->gpt);
    gi = s.hi;
    return true;
  }
};

__device__ __forceinline__ void st_release_gpu(int32_t* p, int32_t v) {
  asm volatile("st.release.gpu.global.s32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
// Bounded acquire-wait until *p != 0.
__device__ __forceinline__ bool wait_flag(const int32_t* p, volatile int* s_abort) {
  if (fz::ld_acquire(p)) return true;
  const uint64_t t0 = global_timer_ns();
  while (!fz::ld_acquire(p)) {
    if (*s_abort || global_timer_ns() - t0 > 2000000000ull) return false;
    __nanosleep(32);
  }
  return true;
}
}  // namespace sk

template <int NSTAGE>
__global__ void __launch_bounds__(kThreads, 1) tc_decode_sk_kernel(const __grid_constant__ TcSkParams f) {
  using namespace sk;
  constexpr int NTOK = kNTOK, N = kN;
  const TcParams& g = f.gu;
  const TcParams& d = f.dn;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + NSTAGE;
  uint64_t* sc_full = empty + NSTAGE;
  uint64_t* sc_empty = sc_full + kScRing;
  uint64_t* acc_full = sc_empty + kScRing;
  uint64_t* acc_empty = acc_full + kNAcc;
  uint64_t* drain = acc_empty + kNAcc;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* s_last = s_abort + 1;  // this CTA completed an output row tile (fused combine)
  uint8_t* base = reinterpret_cast<uint8_t*>(((uintptr_t)(smem + kBarBytes) + 1023) & ~(uintptr_t)1023);
  uint8_t* stages = base;
  uint8_t* scbox = stages + NSTAGE * kSB;
  uint8_t* sfblk = scbox + kScRing * kSCB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NSTAGE; ++i) {
      mbar_init(&full[i], 2);   // producer expect-tx + scale builder
      mbar_init(&empty[i], 2);  // one commit per issuer
    }
    for (int b = 0; b < kScRing; ++b) {
      mbar_init(&sc_full[b], 1);
      mbar_init(&sc_empty[b], 1);
    }
    for (int b = 0; b < kNAcc; ++b) {
      mbar_init(&acc_full[b], 2);
      mbar_init(&acc_empty[b], kEpiWarps);
    }
    mbar_init(drain, 2);
    *s_abort = 0;
    mbar_fence_init();
  }
  if (warp == 3) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();  // unit tables and activation terms come from the preceding kernel
  pdl_launch_dependents();
  const uint32_t tbase = *tmem_slot;
  const int units = g.num_units ? min(__ldg(g.num_units), g.units_cap) : g.units_cap;
  Phase P[2];
  P[0].init((long long)units * g.tiles, g.K / kSkGroupK, g.tiles, MIMO_TC_SK_WAVES);
  P[1].init((long long)units * d.tiles, d.K / kSkGroupK, d.tiles, MIMO_TC_SK_WAVES);
  const int ready_target = kEpiWarps * g.tiles;

  if (warp == 0) {
    // ------------------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_a = MIMO_TC_WEIGHT_EVICT_FIRST ? l2_evict_first_policy() : l2_evict_normal_policy();
      const uint64_t pol_b = l2_evict_normal_policy();
      for (int m = 0; m < 2; ++m) {
        tma_prefetch_map(&g.amap[m]);
        tma_prefetch_map(&g.smap[m]);
      }
      tma_prefetch_map(&g.bmap);
      tma_prefetch_map(&g.bsmap);
      tma_prefetch_map(&d.amap[0]);
      tma_prefetch_map(&d.smap[0]);
      tma_prefetch_map(&d.bmap);
      tma_prefetch_map(&d.bsmap);
      // h-term loads of a down unit whose h is not complete yet: kind 0 = term tile (3-D box), 1 = term
      // scale box (2-D); issued by flush() once ready[pend_unit] reaches the target.
      struct Pend {
        uint8_t* dst;
        int kind, c0, c1, c2;
        uint64_t* bar;
      };
      Pend pend[NSTAGE + kScRing];
      int npend = 0, pend_unit = -1;
      bool stop = false;
      auto flush = [&](bool force) {
        if (npend == 0) return;
        bool ok = fz::ld_acquire(f.ready + pend_unit) >= ready_target;
        if (!ok && !force) {
          const uint64_t t0 = global_timer_ns();
          while (!(ok = fz::ld_acquire(f.ready + pend_unit) >= ready_target)) {
            if (*s_abort || global_timer_ns() - t0 > 2000000000ull) break;
            __nanosleep(64);
          }
          if (!ok) {
            set_status(g.status, MIMO_ETIMEOUT);
            *s_abort = 1;
            stop = true;
          }
        }
        fz::fence_proxy_async_global();  // h was written by generic stores; TMA reads it
        // After an abort the loads still go out (in-bounds rows, unfinished values), so that every
        // stage barrier completes and the drain below never waits on a copy that was not issued.
        for (int i = 0; i < npend; ++i) {
          const Pend& q = pend[i];
          if (q.kind == 0) tma_load_3d(q.dst, &d.bmap, q.c0, q.c1, q.c2, q.bar, pol_b);
          else tma_load_2d(q.dst, &d.bsmap, q.c0, q.c1, q.bar, pol_b);
        }
        npend = 0;
      };
      // Wait for a ring slot; deferred loads go out first when the slot is not free at once.
      auto wait_free = [&](uint64_t* bar, uint32_t par) -> bool {
        if (npend && !mbar_try_wait(bar, par)) flush(false);
        if (stop || !mbar_wait(bar, par)) {
          set_status(g.status, MIMO_ETIMEOUT);
          *s_abort = 1;
          stop = true;
          return false;
        }
        return true;
      };
      int stage = 0;
      uint32_t ph = 0;
      long long issued = 0, groups = 0;
      for (int phase = 0; phase < 2 && !stop; ++phase) {
        const TcParams& p = phase ? d : g;
        const Phase& Q = P[phase];
        const int NM = phase ? 1 : 2, KPS = phase ? 2 : 1;
        if (phase && kL2Prefetch > 0) {
          // the down weights of this CTA's first groups, into L2 while the gate/up pass drains
          long long bytes = 0;
          SegIter it(Q, cta);
          Seg s;
          while (bytes < kL2Prefetch && it.next(s)) {
            const int unit = (int)(s.t / Q.tiles), tile = (int)(s.t % Q.tiles);
            int slot = __ldg(d.unit_slot + unit);
            slot = (slot < 0 || slot >= d.S) ? 0 : slot;
            const int row0 = slot * d.Nw + tile * kM;
            for (long long gk = s.hi - 1; gk >= s.lo && bytes < kL2Prefetch; --gk) {
              const int kc0 = (int)(gk - s.t0) * kGroupChunks;
              tma_prefetch_l2_2d(&d.smap[0], kc0 * 4, row0);
              for (int st = 0; st < kGroupChunks / KPS; ++st) tma_prefetch_l2_3d(&d.amap[0], 0, row0, kc0 + st * KPS);
              bytes += kGroupChunks * kAGlobal;
            }
          }
        }
        SegIter it(Q, cta);
        Seg sg;
        while (!stop && it.next(sg)) {
          const int unit = (int)(sg.t / Q.tiles), tile = (int)(sg.t % Q.tiles);
          int slot = __ldg(p.unit_slot + unit);
          if (slot < 0 || slot >= p.S) {
            set_status(p.status, MIMO_ERANGE);
            slot = 0;
          }
          const int row0 = slot * p.Nw + tile * kM;
          const int brow = (!phase && p.btok) ? 0 : unit * N;
          bool ready_ok = true;
          if (phase) {
            if (npend && pend_unit != unit) flush(false);
            ready_ok = fz::ld_acquire(f.ready + unit) >= ready_target;
            if (ready_ok) fz::fence_proxy_async_global();
            else pend_unit = unit;
          }
          for (long long gk = sg.hi - 1; gk >= sg.lo && !stop; --gk) {
            const int kc0 = (int)(gk - sg.t0) * kGroupChunks;
            if (phase && !ready_ok && (ready_ok = fz::ld_acquire(f.ready + unit) >= ready_target)) {
              flush(false);  // became ready: send what waited, then load directly
              fz::fence_proxy_async_global();
            }
            // scale boxes of the group: 16 bytes (4 chunks) of every weight row and term row
            const int e = (int)(groups % kScRing);
            if (!wait_free(&sc_empty[e], (uint32_t)(((groups / kScRing) & 1) ^ 1))) break;
            uint8_t* sc = scbox + e * kSCB;
            mbar_arrive_expect_tx(&sc_full[e], NM * kM * 16 + N * 16);
            for (int m = 0; m < NM; ++m) tma_load_2d(sc + m * kM * 16, &p.smap[m], kc0 * 4, row0, &sc_full[e], pol_b);
            if (ready_ok) tma_load_2d(sc + NM * kM * 16, &p.bsmap, kc0 * 4, brow, &sc_full[e], pol_b);
            else pend[npend++] = Pend{sc + NM * kM * 16, 1, kc0 * 4, brow, 0, &sc_full[e]};
            ++groups;
            for (int s = 0; s < kGroupChunks / KPS; ++s) {
              const int kc = kc0 + s * KPS;
              if (*s_abort) {
                stop = true;
                break;
              }
              if (!wait_free(&empty[stage], ph ^ 1u)) break;
              uint8_t* sb = stages + stage * kSB;
              mbar_arrive_expect_tx(&full[stage], 2 * kAGlobal + KPS * N * kKC);
              if (!phase) {
                tma_load_2d(sb, &p.amap[0], kc * kKC, row0, &full[stage], pol_a);
                tma_load_2d(sb + kATile, &p.amap[1], kc * kKC, row0, &full[stage], pol_a);
                tma_load_2d(sb + 2 * kATile, &p.bmap, kc * kKC, brow, &full[stage], pol_b);
              } else {  // 3-D boxes [2 chunks][rows][128 B]
                tma_load_3d(sb, &p.amap[0], 0, row0, kc, &full[stage], pol_a);
                if (ready_ok) tma_load_3d(sb + 2 * kATile, &p.bmap, 0, brow, kc, &full[stage], pol_b);
                else pend[npend++] = Pend{sb + 2 * kATile, 0, 0, brow, kc, &full[stage]};
              }
              ++issued;
              if (++stage == NSTAGE) {
                stage = 0;
                ph ^= 1u;
              }
            }
          }
        }
      }
      flush(stop);  // nothing may stay unissued: the drain waits on every stage barrier
      bool ok = true;
      for (long long k = 0; ok && k < (issued < NSTAGE ? issued : NSTAGE); ++k) {
        const long long q = issued - 1 - k;
        ok = mbar_wait(&full[(int)(q % NSTAGE)], (uint32_t)((q / NSTAGE) & 1));
      }
      for (long long k = 0; ok && k < (groups < kScRing ? groups : kScRing); ++k) {
        const long long q = groups - 1 - k;
        ok = mbar_wait(&sc_full[(int)(q % kScRing)], (uint32_t)((q / kScRing) & 1));
      }
      if (!ok) set_status(g.status, MIMO_ETIMEOUT);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------ scale-factor builder
    // Per stage, the 512-byte blocks tcgen05.cp.32x128b.warpx4 turns into the TMEM scale layout: the
    // chunk's 4 bytes of weight rows l, l+32, l+64, l+96 (two weight slots) and of the term rows.
    int stage = 0;
    uint32_t ph = 0;
    uint32_t grp = 0;
    bool stop = false;
    for (int phase = 0; phase < 2 && !stop; ++phase) {
      const Phase& Q = P[phase];
      const int NM = phase ? 1 : 2, KPS = phase ? 2 : 1;
      const long long ng = Q.count(cta);
      for (long long k = 0; k < ng && !stop; ++k) {
        const int e = (int)(grp % kScRing);
        if (!mbar_wait(&sc_full[e], (grp / kScRing) & 1)) {
          if (lane == 0) set_status(g.status, MIMO_ETIMEOUT);
          *s_abort = 1;
          break;
        }
        const uint8_t* sc = scbox + e * kSCB;
        for (int s = 0; s < kGroupChunks / KPS; ++s) {
          if (*s_abort || !mbar_wait(&empty[stage], ph ^ 1u)) {
            if (!*s_abort && lane == 0) set_status(g.status, MIMO_ETIMEOUT);
            *s_abort = 1;
            stop = true;
            break;
          }
          const int c = s * KPS;
          uint8_t* blk = sfblk + stage * kSFB;
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int m = NM == 2 ? j : 0, cj = c + (KPS == 2 ? j : 0);
            const uint8_t* box = sc + m * kM * 16 + cj * 4;
            uint4 v;
            v.x = *reinterpret_cast<const uint32_t*>(box + (lane + 0) * 16);
            v.y = *reinterpret_cast<const uint32_t*>(box + (lane + 32) * 16);
            v.z = *reinterpret_cast<const uint32_t*>(box + (lane + 64) * 16);
            v.w = *reinterpret_cast<const uint32_t*>(box + (lane + 96) * 16);
            *reinterpret_cast<uint4*>(blk + j * 512 + lane * 16) = v;
          }
          for (int j = 0; j < KPS; ++j) {
            const uint8_t* box = sc + NM * kM * 16 + (c + j) * 4;
            uint32_t w[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int r = lane + 32 * q;
              w[q] = r < N ? *reinterpret_cast<const uint32_t*>(box + r * 16) : 0x7F7F7F7Fu;
            }
            *reinterpret_cast<uint4*>(blk + (2 + j) * 512 + lane * 16) = make_uint4(w[0], w[1], w[2], w[3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&full[stage]);
            if (c + KPS == kGroupChunks) mbar_arrive(&sc_empty[e]);
          }
          if (++stage == NSTAGE) {
            stage = 0;
            ph ^= 1u;
          }
        }
        ++grp;
      }
    }
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------------------------ MMA issuers
    // Issuer j: gate/up matrix j, or the chunk of parity j of each down stage; a fresh accumulation in
    // accumulator buffer (group mod kNAcc) for every group.
    const int j = warp - 2;
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0;
      long long gcount = 0;
      bool aborted = false;
      for (int phase = 0; phase < 2 && !aborted; ++phase) {
        const Phase& Q = P[phase];
        const int KPS = phase ? 2 : 1;
        const long long ng = Q.count(cta);
        for (long long k = 0; k < ng && !aborted; ++k, ++gcount) {
          const int bufi = (int)(gcount % kNAcc);
          const uint32_t use = (uint32_t)((gcount / kNAcc) & 1);
          if (!mbar_wait(&acc_empty[bufi], use ^ 1u)) {
            set_status(g.status, MIMO_ETIMEOUT);
            *s_abort = 1;
            aborted = true;
            break;
          }
          tc_fence_after();
          const uint32_t dacc = tbase + (uint32_t)(2 * bufi + j) * N;
          for (int s = 0; s < kGroupChunks / KPS; ++s) {
            if (!mbar_wait(&full[stage], ph)) {
              set_status(g.status, MIMO_ETIMEOUT);
              *s_abort = 1;
              aborted = true;
              break;
            }
            tc_fence_after();
            const uint32_t sb = smem_u32(stages + stage * kSB);
            const uint32_t blk = smem_u32(sfblk + stage * kSFB);
            const uint32_t sf_col = tbase + kSfCol0 + (uint32_t)stage * 16 + 8 * j;
            const int bj = KPS == 2 ? j : 0;  // term tile / scale block of this issuer's chunk
            tc_cp_sf(sf_col, desc_sf(blk + j * 512));
            tc_cp_sf(sf_col + 4, desc_sf(blk + (2 + bj) * 512));
            const uint32_t a0 = sb + j * kATile, b0 = sb + 2 * kATile + bj * N * kKC;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              tc_mma_mx(dacc, desc_sw128(a0 + kk * 32), desc_sw128(b0 + kk * 32), idesc_mx(N, kk),
                        sf_col | ((uint32_t)kk << 30), (sf_col + 4) | ((uint32_t)kk << 30), (s | kk) != 0);
            tc_commit(&empty[stage]);
            if (++stage == NSTAGE) {
              stage = 0;
              ph ^= 1u;
            }
          }
          if (!aborted) tc_commit(&acc_full[bufi]);
        }
      }
      tc_commit(drain);
      if (!mbar_wait(drain, 0)) set_status(g.status, MIMO_ETIMEOUT);
    }
  } else {
    // --------------------------------------------------------------------------------- epilogue
    // Warp w: TMEM lane quadrant w % 4 (weight rows), route half (w - 4) / 4 for the final epilogue;
    // both warps of a quadrant fold all 8 columns (a route's token column can be any of them).
    const int ew = warp - 4;
    const int quad = warp & 3, half = ew >> 2;
    const int qlo = half * (NTOK / 2);
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    bool aborted = false;
    long long gcount = 0;
    if (f.y && units == 0 && cta == 0)  // no routes: the combined output is zero
      for (int o = ew * 32 + lane; o < f.M * d.Nw; o += kEpiWarps * 32) f.y[o] = 0;
    for (int phase = 0; phase < 2; ++phase) {
      const TcParams& p = phase ? d : g;
      const Phase& Q = P[phase];
      float* part = phase ? f.part_d : f.part_g;
      int32_t* flag = phase ? f.flag_d : f.flag_g;
      const int NV = phase ? 1 : 2;  // folded values per column: gate and up, or the down sum
      SegIter it(Q, cta);
      Seg sg;
      while (it.next(sg)) {
        const int unit = (int)(sg.t / Q.tiles), tile = (int)(sg.t % Q.tiles);
        float acc[2][NTOK];
        bool have = false;  // acc holds a partial fold
        if (sg.hi < sg.t0 + Q.gpt) {
          // the tile's groups after ours belong to the next range: start from its published fold R
          const int c2 = Q.cta_of(sg.hi);
          const bool ok = !aborted && sk::wait_flag(flag + (size_t)c2 * kEpiWarps + quad, s_abort) &&
                          sk::wait_flag(flag + (size_t)c2 * kEpiWarps + quad + 4, s_abort);
          if (!ok && !aborted) {
            set_status(g.status, MIMO_ETIMEOUT);
            aborted = true;
          }
          const float* src = part + ((size_t)c2 * 4 + quad) * (NV * NTOK * 32);
#pragma unroll
          for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int c = 0; c < NTOK; ++c) acc[m][c] = (ok && m < NV) ? __ldcg(src + (m * NTOK + c) * 32 + lane) : 0.f;
          have = true;
        } else {
#pragma unroll
          for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int c = 0; c < NTOK; ++c) acc[m][c] = 0.f;
        }
        for (long long gk = sg.hi - 1; gk >= sg.lo; --gk, ++gcount) {
          const int bufi = (int)(gcount % kNAcc);
          const uint32_t use = (uint32_t)((gcount / kNAcc) & 1);
          if (!aborted && !mbar_wait(&acc_full[bufi], use)) {
            set_status(g.status, MIMO_ETIMEOUT);
            aborted = true;
          }
          tc_fence_after();
          float q[2][NTOK];
          if (!aborted) {
            float hv[2][NTOK], lv[2][NTOK];
#pragma unroll
            for (int m = 0; m < 2; ++m) {
              const uint32_t col = tbase + lane_base + (uint32_t)(2 * bufi + m) * N;
              tmem_ld<NTOK>(col, hv[m]);
              tmem_ld<NTOK>(col + NTOK, lv[m]);
            }
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < NTOK; ++c) {
              if (phase == 0) {
                q[0][c] = hv[0][c] + lv[0][c];
                q[1][c] = hv[1][c] + lv[1][c];
              } else {
                q[0][c] = (hv[0][c] + lv[0][c]) + (hv[1][c] + lv[1][c]);
                q[1][c] = 0.f;
              }
            }
          } else {
#pragma unroll
            for (int m = 0; m < 2; ++m)
#pragma unroll
              for (int c = 0; c < NTOK; ++c) q[m][c] = 0.f;
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[bufi]);
#pragma unroll
          for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int c = 0; c < NTOK; ++c) acc[m][c] = have ? q[m][c] + acc[m][c] : q[m][c];  // right fold
          have = true;
        }
        if (sg.lo > sg.t0) {
          // our range starts inside this tile: publish the partial fold for the CTA before us
          float* dst = part + ((size_t)cta * 4 + quad) * (NV * NTOK * 32);
#pragma unroll
          for (int m = 0; m < 2; ++m)
            if (m < NV)
#pragma unroll
              for (int c = 0; c < NTOK / 2; ++c) dst[(m * NTOK + qlo + c) * 32 + lane] = acc[m][qlo + c];
          __threadfence();
          __syncwarp();
          if (lane == 0) st_release_gpu(flag + (size_t)cta * kEpiWarps + ew, 1);
          continue;
        }
        // tile owner: the epilogue
        const int slot = __ldg(p.unit_slot + unit);
        const int cnt = unit_routes(p, unit, NTOK);
        const int p0 = p.unit_p0 ? __ldg(p.unit_p0 + unit) : unit * p.p0_stride;
        const bool live = !aborted && slot >= 0 && slot < p.S;
        const int row = tile * kM + quad * 32 + lane;
        if (live) {
#pragma unroll 1
          for (int qq = qlo; qq < qlo + NTOK / 2; ++qq) {
            int col = qq;  // B rows per route; with by-token rows, route qq's token
            bool ok = qq < cnt;
            if (!phase && g.btok && ok) {
              col = __ldg(g.btok + p0 + qq);
              if (col < 0 || col >= (g.btok_rows > 0 ? min(g.btok_rows, NTOK) : NTOK)) {
                if (lane == 0) set_status(g.status, MIMO_ERANGE);
                ok = false;
                col = 0;
              }
            }
            float a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int c = 0; c < NTOK; ++c)
              if (c == col) {
                a0 = acc[0][c];
                a1 = acc[1][c];
              }
            if (!phase) {
              // SwiGLU with the reference's roundings (kernels.py:79-82), then h as the down pass's terms
              float h = 0.f;
              if (ok) {
                h = swiglu_ref(a0, a1);
                if (!isfinite(h)) set_status(g.status, MIMO_ERANGE);
              }
              uint32_t th, tl, b1, b2;
              split_warp_block(h, th, tl, b1, b2);
              const size_t r0 = (size_t)unit * N + qq, rl = r0 + NTOK;
              g.hq[r0 * g.Nw + row] = (uint8_t)th;
              g.hq[rl * g.Nw + row] = (uint8_t)tl;
              if (lane == 0) {
                g.hs[r0 * (g.Nw / 32) + row / 32] = (uint8_t)b1;
                g.hs[rl * (g.Nw / 32) + row / 32] = (uint8_t)b2;
              }
            } else if (ok) {
              // down x route weight (kernels.py:120)
              const int orow = d.out_row ? __ldg(d.out_row + p0 + qq) : p0 + qq;
              const float v = (d.pairs_rounding ? bf16_round(a0) : a0) * __ldg(d.rw + p0 + qq);
              if (d.peer_part)
                d.peer_part[orow / d.peer_rows][(size_t)(orow % d.peer_rows) * d.Nw + row] = v;
              else
                d.part[(size_t)orow * d.Nw + row] = v;
            }
          }
        }
        if (!phase) {  // publish this warp's share of the unit's h to the down groups
          __threadfence();
          fz::fence_proxy_async_global();
          __syncwarp();
          if (lane == 0) atomicAdd(f.ready + unit, 1);
        } else if (f.y) {
          // fused combine: the CTA completing the last unit's tile of these output rows sums them
          __threadfence();
          named_bar_sync(1, kEpiWarps * 32);
          if (ew == 0 && lane == 0) *s_last = atomicAdd(f.done + tile, 1) == units - 1;
          named_bar_sync(1, kEpiWarps * 32);
          if (*s_last && !aborted) {
            __threadfence();
            const long long rows = (long long)p.units_cap * f.R;  // part rows
            const int col0 = tile * kM;
            for (int o = ew * 32 + lane; o < f.M * kM; o += kEpiWarps * 32) {
              const int m = o / kM, j = col0 + o % kM;
              float sum = 0.f;
              if (f.gidx) {
                for (int k = 0; k < f.topk; ++k) {
                  const int sl = __ldg(f.gidx + m * f.topk + k);
                  if (sl >= rows) {
                    set_status(g.status, MIMO_ERANGE);
                    continue;
                  }
                  if (sl >= 0) sum = __fadd_rn(sum, __ldcg(d.part + (size_t)sl * d.Nw + j));
                }
              } else {
                for (int u = 0; u < units; ++u) {
                  const int n = min(__ldg(f.ucnt + u), f.R);
                  for (int r = 0; r < n; ++r)
                    if (__ldg(f.urows + u * f.R + r) == m)
                      sum = __fadd_rn(sum, __ldcg(d.part + (size_t)(u * f.R + r) * d.Nw + j));
                }
              }
              f.y[(size_t)m * d.Nw + j] = (uint16_t)f32_to_bf16(sum);
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 3) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

// ------------------------------------------------------------ prefill on SM pairs (cta_group::2)
// The prefill passes on pairs of SMs.  A cluster of two CTAs takes one 256-row weight tile per item:
// rows [0, 128) of the tile sit in CTA 0's shared memory and rows [128, 256) in CTA 1's, and the unit's
// N = 128 activation-term rows are split in N between them (hi terms in CTA 0, lo terms in CTA 1).
// CTA 0 issues tcgen05.mma.cta_group::2 with M = 256: each SM's tensor core multiplies its own 128
// weight rows by all 128 term rows (it reads the other half of B from its peer) into its own TMEM.
// Against the single-SM kernel, each MMA instruction does twice the work and each SM loads half as
// many activation bytes per stage.  The B scale factors of all 128 term rows are kept in both CTAs'
// TMEM (each CTA loads and builds them), the A scale factors of its own rows in each.
// Barriers: each CTA's copies complete on its own stage `full` barrier; CTA 0's `full` also waits for
// a 4-byte st.async from CTA 1's scale builder, sent once CTA 1's stage has landed and its scale blocks
// are written (the asynchronous store releases at cluster scope without stalling the builder; a
// remote mbarrier arrive held it ~1 us per stage and made it the pair's bottleneck).  The
// accumulator's `acc_empty` lives in CTA 0 (CTA 1's epilogue warps arrive there remotely, once per
// item); `empty`, `acc_full` and `drain` exist in both CTAs and CTA 0's issuers commit to both.
// Every wait is bounded; both CTAs always reach the final cluster barrier.
namespace pr {
constexpr int kNB = kTcPrefillRoutes;  // term rows per CTA: N / 2
constexpr int kN = 2 * kTcPrefillRoutes;
template <int NM>
constexpr int stage_bytes() { return 2 * kATile + kps<NM>() * kNB * kKC; }
template <int NM>
constexpr int scale_box_bytes() { return NM * kM * 16 + kN * 16; }
template <int NM, int NSTAGE>
constexpr int smem_bytes() {
  return kBarBytes + 1024 + NSTAGE * stage_bytes<NM>() + 2 * scale_box_bytes<NM>() + NSTAGE * sf_block_bytes<NM>();
}
// kind::mxf8f6f4 block-scaled instruction descriptor for the pair: M = 256 (bits 24-28 hold M / 16).
__device__ __forceinline__ uint32_t idesc_mx2(int n, uint32_t kb) {
  return (idesc_mx(n, kb) & ~(0x1Fu << 24)) | ((uint32_t)(256 >> 4) << 24);
}
}  // namespace pr

template <int NM, int NSTAGE, int MODE, int EPI>
__global__ void __launch_bounds__((4 + EPI) * 32, 1) tc_pair_kernel(const __grid_constant__ TcParams p) {
  constexpr int NTOK = kTcPrefillRoutes;
  constexpr int N = pr::kN;
  constexpr int NB = pr::kNB;
  constexpr int KPS = kps<NM>();
  constexpr int SB = pr::stage_bytes<NM>();
  constexpr int SCB = pr::scale_box_bytes<NM>();
  constexpr int SFB = sf_block_bytes<NM>();
  constexpr uint32_t TCOLS = 512;
  constexpr int QH = NTOK / (EPI / 4);
  constexpr int QC = QH < 16 ? QH : 16;
  static_assert(2 * N + NSTAGE * 16 <= (int)TCOLS, "TMEM: one accumulator buffer + scale columns");
  static_assert(EPI % 4 == 0 && NTOK % (EPI / 4) == 0 && QH % QC == 0, "epilogue split");
  static_assert(NM * KPS == 2 && MODE != 1, "two slots per stage; prefill modes");
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // [NSTAGE] own tiles landed (+ CTA 0: both scale builders)
  uint64_t* empty = full + NSTAGE;                     // [NSTAGE] both issuers' MMAs of the stage done
  uint64_t* sc_full = empty + NSTAGE;                  // [2] this CTA's scale boxes landed
  uint64_t* sc_empty = sc_full + 2;                    // [2] scale boxes read
  uint64_t* acc_full = sc_empty + 2;                   // accumulators written (both issuers)
  uint64_t* acc_empty = acc_full + 1;                  // (CTA 0) both CTAs' epilogues copied them out
  uint64_t* drain = acc_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* fwd = tmem_slot + 2;  // [NSTAGE] (CTA 0) words CTA 1's stage signals land in
  uint8_t* base = reinterpret_cast<uint8_t*>(((uintptr_t)(smem + kBarBytes) + 1023) & ~(uintptr_t)1023);
  uint8_t* stages = base;                 // NSTAGE x [2 A tiles | KPS B half-tiles]
  uint8_t* scbox = stages + NSTAGE * SB;  // 2 x [NM x A scale box | B scale box]
  uint8_t* sfblk = scbox + 2 * SCB;       // NSTAGE x [2 weight scale blocks | KPS activation blocks]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool lead = rank == 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NSTAGE; ++i) {
      mbar_init(&full[i], lead ? 2 : 1);  // own expect-tx arrival (+ CTA 0: its scale builder)
      mbar_init(&empty[i], 2);  // one commit per issuer
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sc_full[b], 1);
      mbar_init(&sc_empty[b], 1);
    }
    mbar_init(acc_full, 2);
    mbar_init(acc_empty, 2 * EPI);
    mbar_init(drain, 2);
    *s_abort = 0;
    mbar_fence_init();
  }
  if (warp == 3) {
    tmem_alloc2(tmem_slot, TCOLS);
    tmem_relinquish2();
  }
  tc_fence_before();
  cluster_sync();  // barriers initialised and TMEM allocated in both CTAs before any remote use
  tc_fence_after();
  pdl_wait();  // the unit tables and activation terms come from the preceding kernel
  pdl_launch_dependents();
  const uint32_t tbase = *tmem_slot;
  const int units = p.num_units ? min(__ldg(p.num_units), p.units_cap) : p.units_cap;
  const long long items = (long long)units * p.tiles;  // p.tiles: 256-row tiles per expert
  const long long pair = cluster_id_x(), npairs = cluster_count_x();
  const long long my_items = items > pair ? (items - pair + npairs - 1) / npairs : 0;
  const int ns = p.K / (kKC * KPS);
  const long long nsteps = my_items * ns;
  const uint32_t full0 = mapa_shared(smem_u32(full), 0);  // CTA 0's barriers, cluster addresses
  const uint32_t acc_empty0 = mapa_shared(smem_u32(acc_empty), 0);
  const uint32_t fwd0 = mapa_shared(smem_u32(fwd), 0);
  constexpr uint32_t kSfCol0 = 2 * N;  // accumulator j at columns j * N

  if (warp == 0) {
    // ------------------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol = l2_evict_normal_policy();
      for (int m = 0; m < NM; ++m) {
        tma_prefetch_map(&p.amap[m]);
        tma_prefetch_map(&p.smap[m]);
      }
      tma_prefetch_map(&p.bmap);
      tma_prefetch_map(&p.bsmap);
      int stage = 0;
      uint32_t ph = 0;
      long long issued = 0, groups = 0;
      bool stop = false;
      for (long long n = 0; n < my_items && !stop; ++n) {
        const long long it = pair + n * npairs;
        int unit, tile;
        item_coords(p, it, unit, tile);
        int slot = __ldg(p.unit_slot + unit);
        if (slot < 0 || slot >= p.S) {
          set_status(p.status, MIMO_ERANGE);
          slot = 0;
        }
        const int row0 = slot * p.Nw + tile * (2 * kM) + (int)rank * kM;  // this CTA's 128 weight rows
        const int brow = unit * N;                                       // the unit's term rows
        for (int ks = 0; ks < ns; ++ks) {
          if (*s_abort) {
            stop = true;
            break;
          }
          const int kc = ks * KPS;
          if ((kc & 3) == 0) {  // scale boxes for chunks kc..kc+3: own weight rows, all term rows
            const int e = (int)(groups & 1);
            if (!mbar_wait(&sc_empty[e], (uint32_t)(((groups >> 1) & 1) ^ 1))) {
              set_status(p.status, MIMO_ETIMEOUT);
              *s_abort = 1;
              stop = true;
              break;
            }
            uint8_t* sc = scbox + e * SCB;
            mbar_arrive_expect_tx(&sc_full[e], NM * kM * 16 + N * 16);
            for (int m = 0; m < NM; ++m) tma_load_2d(sc + m * kM * 16, &p.smap[m], kc * 4, row0, &sc_full[e], pol);
            tma_load_2d(sc + NM * kM * 16, &p.bsmap, kc * 4, brow, &sc_full[e], pol);
            ++groups;
          }
          if (!mbar_wait(&empty[stage], ph ^ 1u)) {
            set_status(p.status, MIMO_ETIMEOUT);
            *s_abort = 1;
            stop = true;
            break;
          }
          uint8_t* sb = stages + stage * SB;
          // CTA 0's stage also waits for CTA 1's 4-byte signal (its tiles landed, scale blocks written).
          mbar_arrive_expect_tx(&full[stage], 2 * kAGlobal + KPS * NB * kKC + (lead ? 4 : 0));
          if constexpr (KPS == 1) {
            tma_load_2d(sb, &p.amap[0], kc * kKC, row0, &full[stage], pol);
            tma_load_2d(sb + kATile, &p.amap[1], kc * kKC, row0, &full[stage], pol);
            tma_load_2d(sb + 2 * kATile, &p.bmap, kc * kKC, brow + (int)rank * NB, &full[stage], pol);
          } else {
            tma_load_3d(sb, &p.amap[0], 0, row0, kc, &full[stage], pol);
            tma_load_3d(sb + 2 * kATile, &p.bmap, 0, brow + (int)rank * NB, kc, &full[stage], pol);
          }
          ++issued;
          if (++stage == NSTAGE) {
            stage = 0;
            ph ^= 1u;
          }
        }
      }
      // Shared memory must not be released with copies still landing.
      bool ok = true;
      for (long long k = 0; ok && k < (issued < NSTAGE ? issued : NSTAGE); ++k) {
        const long long f = issued - 1 - k;
        ok = mbar_wait(&full[(int)(f % NSTAGE)], (uint32_t)((f / NSTAGE) & 1));
      }
      for (long long k = 0; ok && k < (groups < 2 ? groups : 2); ++k) {
        const long long g = groups - 1 - k;
        ok = mbar_wait(&sc_full[(int)(g & 1)], (uint32_t)((g >> 1) & 1));
      }
      if (!ok) set_status(p.status, MIMO_ETIMEOUT);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------ scale-factor builder
    // As in the single-SM kernel (this CTA's weight rows; all N term rows).  CTA 0's builder arrives on
    // its own full barrier; CTA 1's first waits for its own stage to land, then arrives on CTA 0's.
    int stage = 0;
    uint32_t ph = 0;
    for (long long s = 0; s < nsteps; ++s) {
      if (*s_abort) break;
      const uint32_t kc = (uint32_t)(s * KPS);
      const int c = (int)(kc & 3);
      const uint32_t g = kc >> 2;
      const int e = (int)(g & 1);
      if (c == 0 && !mbar_wait(&sc_full[e], (g >> 1) & 1)) {
        if (lane == 0) set_status(p.status, MIMO_ETIMEOUT);
        *s_abort = 1;
        break;
      }
      if (!mbar_wait(&empty[stage], ph ^ 1u)) {
        if (lane == 0) set_status(p.status, MIMO_ETIMEOUT);
        *s_abort = 1;
        break;
      }
      const uint8_t* sc = scbox + e * SCB;
      uint8_t* blk = sfblk + stage * SFB;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int m = NM == 2 ? j : 0, cj = c + (KPS == 2 ? j : 0);
        const uint8_t* box = sc + m * kM * 16 + cj * 4;
        uint4 v;
        v.x = *reinterpret_cast<const uint32_t*>(box + (lane + 0) * 16);
        v.y = *reinterpret_cast<const uint32_t*>(box + (lane + 32) * 16);
        v.z = *reinterpret_cast<const uint32_t*>(box + (lane + 64) * 16);
        v.w = *reinterpret_cast<const uint32_t*>(box + (lane + 96) * 16);
        *reinterpret_cast<uint4*>(blk + j * 512 + lane * 16) = v;
      }
#pragma unroll
      for (int j = 0; j < KPS; ++j) {
        const uint8_t* box = sc + NM * kM * 16 + (c + j) * 4;
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) w[q] = *reinterpret_cast<const uint32_t*>(box + (lane + 32 * q) * 16);
        *reinterpret_cast<uint4*>(blk + (2 + j) * 512 + lane * 16) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if (c + KPS == 4) mbar_arrive(&sc_empty[e]);
        if (lead) {
          mbar_arrive(&full[stage]);
        } else if (mbar_wait(&full[stage], ph)) {
          // A remote arrive blocked this thread ~1 us per stage; the asynchronous store does not.
          st_async_signal(fwd0 + (uint32_t)stage * 4u, 1u, full0 + (uint32_t)stage * 8u);
        } else {
          set_status(p.status, MIMO_ETIMEOUT);
          *s_abort = 1;
        }
      }
      __syncwarp();
      if (*s_abort) break;
      if (++stage == NSTAGE) {
        stage = 0;
        ph ^= 1u;
      }
    }
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------------------------ MMA issuers
    // CTA 0 only.  Issuer j owns slot j of every stage (gate / up, or the stage's first / second K
    // chunk of down) and accumulator j; its commits go to the barrier in each CTA.
    const int j = warp - 2;
    const uint32_t peer = 1u;
    if (lead && lane == 0) {
      const uint32_t empty_l = mapa_shared(smem_u32(empty), 0), empty_p = mapa_shared(smem_u32(empty), peer);
      const uint32_t accf_l = mapa_shared(smem_u32(acc_full), 0), accf_p = mapa_shared(smem_u32(acc_full), peer);
      int stage = 0;
      uint32_t ph = 0;
      bool aborted = false;
      for (long long n = 0; n < my_items && !aborted; ++n) {
        if (!mbar_wait_cluster(acc_empty, (uint32_t)(n & 1) ^ 1u)) {
          set_status(p.status, MIMO_ETIMEOUT);
          *s_abort = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tbase + (uint32_t)j * N;
        for (int ks = 0; ks < ns; ++ks) {
          if (!mbar_wait_cluster(&full[stage], ph)) {
            set_status(p.status, MIMO_ETIMEOUT);
            *s_abort = 1;
            aborted = true;
            break;
          }
          tc_fence_after();
          const uint32_t sb = smem_u32(stages + stage * SB);
          const uint32_t blk = smem_u32(sfblk + stage * SFB);
          const uint32_t sf_col = tbase + kSfCol0 + (uint32_t)stage * 16 + 8 * j;
          const int bj = KPS == 2 ? j : 0;
          tc_cp_sf2(sf_col, desc_sf(blk + j * 512));
          tc_cp_sf2(sf_col + 4, desc_sf(blk + (2 + bj) * 512));
          const uint32_t a0 = sb + j * kATile, b0 = sb + 2 * kATile + bj * NB * kKC;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc_mma_mx2(d, desc_sw128(a0 + kk * 32), desc_sw128(b0 + kk * 32), pr::idesc_mx2(N, kk),
                       sf_col | ((uint32_t)kk << 30), (sf_col + 4) | ((uint32_t)kk << 30), (ks | kk) != 0);
          tc_commit2(empty_l + (uint32_t)stage * 8u);
          tc_commit2(empty_p + (uint32_t)stage * 8u);
          if (++stage == NSTAGE) {
            stage = 0;
            ph ^= 1u;
          }
        }
        if (!aborted) {
          tc_commit2(accf_l);
          tc_commit2(accf_p);
        }
      }
      // Nothing may still read either CTA's shared memory or TMEM when they are released.
      tc_commit2(mapa_shared(smem_u32(drain), 0));
      tc_commit2(mapa_shared(smem_u32(drain), peer));
      if (!mbar_wait(drain, 0)) set_status(p.status, MIMO_ETIMEOUT);
    } else if (!lead && warp == 2 && lane == 0) {
      // CTA 1 waits for CTA 0's last MMAs, which read its shared memory and write its TMEM (CTA 0's
      // issuers always commit to this barrier at their end).
      if (!mbar_wait(drain, 0)) set_status(p.status, MIMO_ETIMEOUT);
    }
  } else if (warp >= 4) {
    // --------------------------------------------------------------------------------- epilogue
    // This CTA's 128 weight rows of the item's tile, all routes (single accumulator buffer: copy the
    // warp's columns out, release the accumulator to CTA 0's issuers, then compute).
    const int quad = warp & 3;
    const int qlo = ((warp - 4) >> 2) * QH;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    bool aborted = false;
    for (long long n = 0; n < my_items; ++n) {
      const long long it = pair + n * npairs;
      int unit, tile;
      item_coords(p, it, unit, tile);
      const int slot = __ldg(p.unit_slot + unit);
      const int cnt = unit_routes(p, unit, NTOK);
      const int p0 = p.unit_p0 ? __ldg(p.unit_p0 + unit) : unit * p.p0_stride;
      if (!aborted && !mbar_wait(acc_full, (uint32_t)(n & 1))) {
        set_status(p.status, MIMO_ETIMEOUT);
        aborted = true;
      }
      tc_fence_after();
      const bool live = !aborted && slot >= 0 && slot < p.S;
      const int row = tile * (2 * kM) + (int)rank * kM + quad * 32 + lane;  // output feature of this lane
      float hv[2][QH], lv[2][QH];
      if (live) {
#pragma unroll
        for (int q0 = 0; q0 < QH; q0 += QC) {
#pragma unroll
          for (int a = 0; a < 2; ++a) {
            float th[QC], tl[QC];
            const uint32_t c = tbase + lane_base + (uint32_t)a * N + qlo + q0;
            tmem_ld<QC>(c, th);
            tmem_ld<QC>(c + NTOK, tl);
#pragma unroll
            for (int i = 0; i < QC; ++i) {
              hv[a][q0 + i] = th[i];
              lv[a][q0 + i] = tl[i];
            }
          }
        }
        tmem_wait_ld();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty0);
      if (!live) continue;
#pragma unroll
      for (int i = 0; i < QH; ++i) {
        const int q = qlo + i;
        if constexpr (MODE == 0) {
          float h = 0.f;
          if (q < cnt) {
            h = swiglu_ref(hv[0][i] + lv[0][i], hv[1][i] + lv[1][i]);
            if (!isfinite(h)) set_status(p.status, MIMO_ERANGE);
          }
          uint32_t th, tl, b1, b2;
          split_warp_block(h, th, tl, b1, b2);
          const size_t rh = (size_t)unit * N + q, rl = rh + NTOK;
          p.hq[rh * p.Nw + row] = (uint8_t)th;
          p.hq[rl * p.Nw + row] = (uint8_t)tl;
          if (lane == 0) {
            p.hs[rh * (p.Nw / 32) + row / 32] = (uint8_t)b1;
            p.hs[rl * (p.Nw / 32) + row / 32] = (uint8_t)b2;
          }
        } else {
          if (q < cnt) {
            const float dsum = (hv[0][i] + lv[0][i]) + (hv[1][i] + lv[1][i]);  // each K half's hi + lo
            p.ypair[(size_t)(p0 + q) * p.Nw + row] = (uint16_t)f32_to_bf16(dsum);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the other may still reach its shared memory
  if (warp == 3) {
    tc_fence_after();
    tmem_dealloc2(tbase, TCOLS);
  }
}

// Pair kernels: clusters of two CTAs, as many clusters as can be resident at once.
template <int NM, int NSTAGE, int MODE, int EPI>
static cudaError_t launch_pair(const TcParams& p, int num_sms, cudaStream_t st) {
  auto kfn = tc_pair_kernel<NM, NSTAGE, MODE, EPI>;
  constexpr int smem = pr::smem_bytes<NM, NSTAGE>();
  static_assert(smem <= 232448, "shared memory budget");
  static_assert((2 * NSTAGE + 4 + 3) * 8 + 8 + NSTAGE * 4 <= kBarBytes, "barrier area");
  if (p.K % (4 * kKC) != 0 || p.Nw % (2 * kM) != 0 || p.tiles != p.Nw / (2 * kM)) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3((4 + EPI) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  static int nc = 0;
  if (nc <= 0) {
    cfg.gridDim = dim3(num_sms & ~1);
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kfn, &cfg);
    if (e != cudaSuccess) return e;
    nc = n > 0 ? std::min(n, num_sms / 2) : num_sms / 2;
    const char* o = getenv("MIMO_MOE_PAIR_CLUSTERS");  // comparison knob: fewer resident clusters
    if (o && atoi(o) > 0) nc = std::min(nc, atoi(o));
    if (getenv("MIMO_MOE_VERBOSE")) fprintf(stderr, "[mimo_moe] pair kernel NM=%d: %d clusters (occupancy %d)\n", NM, nc, n);
  }
  cfg.gridDim = dim3(2 * nc);
  return cudaLaunchKernelEx(&cfg, kfn, p);
}

template <int NM, int NTOK, int NSTAGE, int MODE, int EPI>
static cudaError_t launch(const TcParams& p, int grid, cudaStream_t st) {
  auto kfn = tc_expert_kernel<NM, NTOK, NSTAGE, MODE, EPI>;
  constexpr int smem = smem_bytes<NM, 2 * NTOK, NSTAGE>();
  static_assert(smem <= 232448, "shared memory budget");
  static_assert(tmem_cols_needed<2 * NTOK, NSTAGE>() <= 512, "TMEM budget");
  static_assert((2 * NSTAGE + 4 + 4 + 1) * 8 + 8 <= kBarBytes, "barrier area");
  constexpr int trows = (MODE == 3 || MODE == 4) ? 2 * kM : kM;
  if (p.K % (4 * kKC) != 0 || p.Nw % trows != 0 || p.tiles != p.Nw / trows) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return launch_k(kfn, dim3(grid), dim3((4 + EPI) * 32), smem, st, p);
}

// ---------------------------------------------------------------------- activation term split
// Block (unit, q): route q of the unit.  Thread t splits 32-value block t of the route's token row;
// routes q >= cnt are left unwritten (their MMA columns are never read).
template <int NTOK>
__global__ void __launch_bounds__(128) split_rows_kernel(const uint16_t* __restrict__ x, int K,
                                                         const int32_t* __restrict__ unit_cnt,
                                                         const int32_t* __restrict__ unit_p0, int p0_stride,
                                                         const int32_t* __restrict__ rtok,
                                                         const int32_t* __restrict__ num_units, int units_cap,
                                                         uint8_t* __restrict__ bq, uint8_t* __restrict__ bs,
                                                         int32_t* status, int x_ld, int x_rows) {
  constexpr int N = 2 * NTOK;
  const int unit = blockIdx.x / NTOK, q = blockIdx.x % NTOK;
  const int units = num_units ? min(*num_units, units_cap) : units_cap;
  if (unit >= units) return;
  const int lim = unit_p0 ? NTOK : min(NTOK, p0_stride);
  const int cnt = min(unit_cnt[unit], lim);
  if (q == 0 && unit_cnt[unit] > lim) set_status(status, MIMO_ERANGE);
  if (q >= cnt) return;
  const int p0 = unit_p0 ? unit_p0[unit] : unit * p0_stride;
  int tok = rtok ? rtok[p0 + q] : p0 + q;
  if (x_rows > 0 && (tok < 0 || tok >= x_rows)) {  // never read past the activation rows
    if (threadIdx.x == 0) set_status(status, MIMO_ERANGE);
    tok = 0;
  }
  const size_t rh = (size_t)unit * N + q, rl = rh + NTOK;
  const int nb = K / 32;
  for (int blk = threadIdx.x; blk < nb; blk += blockDim.x) {
    split_block32(x + (size_t)tok * x_ld + blk * 32, bq + rh * K + blk * 32, bq + rl * K + blk * 32,
                  bs + rh * nb + blk, bs + rl * nb + blk, status);
  }
}

// Block t: token row t -> term rows t (hi) and 8 + t (lo).
__global__ void __launch_bounds__(128) split_tokens_kernel(const uint16_t* __restrict__ x, int K,
                                                           uint8_t* __restrict__ bq, uint8_t* __restrict__ bs,
                                                           int32_t* status) {
  const int t = blockIdx.x, nb = K / 32;
  for (int blk = threadIdx.x; blk < nb; blk += blockDim.x)
    split_block32(x + (size_t)t * K + blk * 32, bq + (size_t)t * K + blk * 32,
                  bq + (size_t)(kTcDecodeRoutes + t) * K + blk * 32, bs + (size_t)t * nb + blk,
                  bs + (size_t)(kTcDecodeRoutes + t) * nb + blk, status);
}

// e2m1 terms (kind::mxf4 decode).  Block t: token row t -> rows j * 8 + t.
__global__ void __launch_bounds__(128) split_tokens_fp4_kernel(const uint16_t* __restrict__ x, int K,
                                                               uint8_t* __restrict__ bq, uint8_t* __restrict__ bs,
                                                               int32_t* status) {
  const int t = blockIdx.x, nb = K / 32;
  for (int blk = threadIdx.x; blk < nb; blk += blockDim.x)
    split_block32_fp4(x + (size_t)t * K + blk * 32, bq + (size_t)t * (K / 2) + blk * 16,
                      (size_t)kTcDecodeRoutes * (K / 2), bs + (size_t)t * nb + blk, (size_t)kTcDecodeRoutes * nb,
                      status);
}
// Block (unit, q): route q of the unit -> rows unit * 40 + j * 8 + q.
__global__ void __launch_bounds__(128) split_rows_fp4_kernel(const uint16_t* __restrict__ x, int K,
                                                             const int32_t* __restrict__ unit_cnt,
                                                             const int32_t* __restrict__ unit_p0, int p0_stride,
                                                             const int32_t* __restrict__ rtok,
                                                             const int32_t* __restrict__ num_units, int units_cap,
                                                             uint8_t* __restrict__ bq, uint8_t* __restrict__ bs,
                                                             int32_t* status, int x_ld, int x_rows) {
  constexpr int NTOK = kTcDecodeRoutes, N = kFp4Terms * NTOK;
  const int unit = blockIdx.x / NTOK, q = blockIdx.x % NTOK;
  const int units = num_units ? min(*num_units, units_cap) : units_cap;
  if (unit >= units) return;
  const int lim = unit_p0 ? NTOK : min(NTOK, p0_stride);
  const int cnt = min(unit_cnt[unit], lim);
  if (q == 0 && unit_cnt[unit] > lim) set_status(status, MIMO_ERANGE);
  if (q >= cnt) return;
  const int p0 = unit_p0 ? unit_p0[unit] : unit * p0_stride;
  int tok = rtok ? rtok[p0 + q] : p0 + q;
  if (x_rows > 0 && (tok < 0 || tok >= x_rows)) {  // never read past the activation rows
    if (threadIdx.x == 0) set_status(status, MIMO_ERANGE);
    tok = 0;
  }
  const size_t r0 = (size_t)unit * N + q;
  const int nb = K / 32;
  for (int blk = threadIdx.x; blk < nb; blk += blockDim.x)
    split_block32_fp4(x + (size_t)tok * x_ld + blk * 32, bq + r0 * (K / 2) + blk * 16, (size_t)NTOK * (K / 2),
                      bs + r0 * nb + blk, (size_t)NTOK * nb, status);
}


}  // namespace tc

// ------------------------------------------------------------------------------ host entry
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("MIMO_MOE_PDL");
    return !(e && std::string(e) == "0");
  }();
  return on;
}

cudaError_t launch_tc_split_tokens_fp4(const uint16_t* x, int T, int K, uint8_t* bq, uint8_t* bs, int32_t* status,
                                       cudaStream_t st) {
  if (T < 1 || T > kTcDecodeRoutes || K % 128 != 0) return cudaErrorInvalidValue;
  tc::split_tokens_fp4_kernel<<<T, 128, 0, st>>>(x, K, bq, bs, status);
  return cudaGetLastError();
}
cudaError_t launch_tc_split_fp4(const uint16_t* x, int K, const int32_t* unit_cnt, const int32_t* unit_p0,
                                int p0_stride, const int32_t* rtok, const int32_t* num_units, int units_cap,
                                uint8_t* bq, uint8_t* bs, int32_t* status, cudaStream_t st, int x_ld, int x_rows) {
  if (K % 128 != 0 || units_cap < 1) return cudaErrorInvalidValue;
  if (x_ld <= 0) x_ld = K;
  if (x_ld < K || x_ld % 8) return cudaErrorInvalidValue;
  tc::split_rows_fp4_kernel<<<units_cap * kTcDecodeRoutes, 128, 0, st>>>(x, K, unit_cnt, unit_p0, p0_stride, rtok,
                                                                         num_units, units_cap, bq, bs, status, x_ld,
                                                                         x_rows);
  return cudaGetLastError();
}
cudaError_t launch_tc_split_tokens(const uint16_t* x, int T, int K, uint8_t* bq, uint8_t* bs, int32_t* status,
                                   cudaStream_t st) {
  if (T < 1 || T > kTcDecodeRoutes || K % 128 != 0) return cudaErrorInvalidValue;
  tc::split_tokens_kernel<<<T, 128, 0, st>>>(x, K, bq, bs, status);
  return cudaGetLastError();
}
cudaError_t launch_tc_split(const uint16_t* x, int K, const int32_t* unit_cnt, const int32_t* unit_p0,
                            int p0_stride, const int32_t* rtok, const int32_t* num_units, int units_cap,
                            int ntok, uint8_t* bq, uint8_t* bs, int32_t* status, cudaStream_t st, int x_ld,
                            int x_rows) {
  if (K % 128 != 0 || units_cap < 1) return cudaErrorInvalidValue;
  if (x_ld <= 0) x_ld = K;
  if (x_ld < K || x_ld % 8) return cudaErrorInvalidValue;  // 16-byte aligned rows
  if (ntok == kTcDecodeRoutes)
    tc::split_rows_kernel<kTcDecodeRoutes><<<units_cap * kTcDecodeRoutes, 128, 0, st>>>(
        x, K, unit_cnt, unit_p0, p0_stride, rtok, num_units, units_cap, bq, bs, status, x_ld, x_rows);
  else if (ntok == kTcPrefillRoutes)
    tc::split_rows_kernel<kTcPrefillRoutes><<<units_cap * kTcPrefillRoutes, 128, 0, st>>>(
        x, K, unit_cnt, unit_p0, p0_stride, rtok, num_units, units_cap, bq, bs, status, x_ld, x_rows);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

template <int kSt, bool FP4>
static cudaError_t launch_fused(const TcFusedParams& f, int num_sms, cudaStream_t st) {
  auto kfn = tc::tc_decode_fused_kernel<kSt, FP4>;
  constexpr int smem = tc::fz::smem_bytes<kSt, FP4>();
  static_assert(smem <= 232448, "shared memory budget");
  static_assert(tc::tmem_cols_needed<tc::fz::Fmt<FP4>::kN, kSt>() <= 512, "TMEM budget");
  static_assert((2 * kSt + 4 + 4 + 1) * 8 + 8 <= tc::kBarBytes, "barrier area");
  const TcParams& g = f.gu;
  const TcParams& d = f.dn;
  if (g.K % (4 * tc::kKC) || d.K % (4 * tc::kKC) || g.Nw % tc::kM || d.Nw % tc::kM || g.tiles != g.Nw / tc::kM ||
      d.tiles != d.Nw / tc::kM || g.Nw != d.K || !f.ready)
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return launch_k(kfn, dim3(num_sms), dim3(tc::kThreads), smem, st, f);
}

#ifndef MIMO_TC_STSK
#define MIMO_TC_STSK 5  // ring depth of the stream-K decode kernel
#endif
cudaError_t launch_tc_decode_sk(const TcSkParams& f, cudaStream_t st) {
  auto kfn = tc::tc_decode_sk_kernel<MIMO_TC_STSK>;
  constexpr int smem = tc::sk::smem_bytes<MIMO_TC_STSK>();
  static_assert(smem <= 232448, "shared memory budget");
  static_assert(tc::sk::kSfCol0 + MIMO_TC_STSK * 16 <= tc::sk::kTmemCols, "TMEM budget");
  static_assert((2 * MIMO_TC_STSK + 2 * tc::sk::kScRing + 2 * tc::sk::kNAcc + 1) * 8 + 8 <= tc::kBarBytes,
                "barrier area");
  const TcParams& g = f.gu;
  const TcParams& d = f.dn;
  if (g.K % kSkGroupK || d.K % kSkGroupK || g.Nw % tc::kM ||
      d.Nw % tc::kM || g.tiles != g.Nw / tc::kM || d.tiles != d.Nw / tc::kM || g.Nw != d.K || !f.ready ||
      !f.part_g || !f.part_d || !f.flag_g || !f.flag_d || f.ctas < 1)
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return launch_k(kfn, dim3(f.ctas), dim3(tc::kThreads), smem, st, f);
}

cudaError_t launch_tc_decode_fused(const TcFusedParams& f, bool fp4, int num_sms, cudaStream_t st) {
  return fp4 ? launch_fused<MIMO_TC_STF4, true>(f, num_sms, st) : launch_fused<MIMO_TC_STF, false>(f, num_sms, st);
}

cudaError_t launch_tc_pair(const TcParams& p, int kind, int num_sms, cudaStream_t st) {
  switch (kind) {
    case 2: return tc::launch_pair<2, MIMO_TC_PST2, 0, MIMO_TC_EPI_PREFILL>(p, num_sms, st);
    case 3: return tc::launch_pair<1, MIMO_TC_PST3, 2, MIMO_TC_EPI_PREFILL>(p, num_sms, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_tc_experts(const TcParams& p, int kind, int num_sms, cudaStream_t st) {
  switch (kind) {
    case 0: return tc::launch<2, kTcDecodeRoutes, tc::kStages[0], 0, 8>(p, num_sms, st);
    case 1: return tc::launch<1, kTcDecodeRoutes, tc::kStages[1], 1, 8>(p, num_sms, st);
    case 5: return tc::launch<2, kTcDecodeRoutes, tc::kStages[0], 3, 8>(p, num_sms, st);  // down, paired rows
    case 6:  // prefill down, paired rows
      return tc::launch<2, kTcPrefillRoutes, tc::kStages[2], 4, MIMO_TC_EPI_PREFILL>(p, num_sms, st);
    case 2: return tc::launch<2, kTcPrefillRoutes, tc::kStages[2], 0, MIMO_TC_EPI_PREFILL>(p, num_sms, st);
    case 3: return tc::launch<1, kTcPrefillRoutes, tc::kStages[3], 2, MIMO_TC_EPI_PREFILL>(p, num_sms, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace mimo
