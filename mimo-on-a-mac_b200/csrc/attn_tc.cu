// Attention on the 5th-generation tensor cores (tcgen05, TMEM accumulators, TMA) for query tiles of 128 rows:
// mimo_moe_layer_attention's kernel whenever the cache capacity is a multiple of 128 (semantics in layer.cu,
// whose mma.sync kernel takes the other caches).  Prefill runs one CTA per (query tile, kv head); decode
// (a tile of T * G <= 128 rows over a long cache) also splits the tile's key blocks over CTAs (grid z) and
// writes unnormalised partials that layer.cu's merge kernel folds with the sink.
//
// One CTA = 128 query rows of one kv head (the G = n_heads / n_kv_heads heads of 128 / G consecutive tokens,
// token-major, so one K/V block serves the whole GQA group), key blocks of 128, 10 warps:
//   warp 8 (one thread)  TMA producer: the Q tile once (head_dim / 64 boxes of [64 dims x G heads x 128/G
//                        tokens]), then K_j and V_j of every block through a ring of 3 shared-memory slots;
//   warp 9 (one thread)  MMA issuer: S_j = Q K_j^T (M 128, N 128, K 16 per instruction, kind::f16, f32
//                        accumulate) into one of two TMEM buffers; O += P_j V_j (V read as an MN-major
//                        operand) into the TMEM output; commits release ring slots and signal the softmax;
//   warps 0-7            softmax, two threads per query row (TMEM lane = row; warps 0-3 take columns 0-63,
//                        warps 4-7 columns 64-127, the row maximum exchanged through shared memory behind
//                        named barriers): S_j from TMEM, mask, running
//                        max in the exp2 domain, P_j = bf16(exp2(s - m)) into shared memory (128B-swizzled
//                        K-major rows, the layout the MMA reads), the row sum from the float32 P; the TMEM
//                        output is rescaled only when a row's maximum grows by more than 2^8 (the stale
//                        maximum bounds P by 256); at the end O / (l + sink term).  Per score: one FFMA, one
//                        ex2 and half a bf16x2 conversion, so the 128 scores of a row stay a short loop.
// Key blocks start at multiples of 128 positions and the cache capacity is a multiple of 128, so a block
// never wraps in the ring; keys outside a row's window are masked (P = 0).  Every wait is bounded and sets
// MIMO_ETIMEOUT in the status word; the producer drains its copies and the issuer its MMAs before exit.
#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace mimo {

namespace {

constexpr int kTcThreads = 320;  // warps 0-7 softmax (row, column half), 8 TMA producer, 9 MMA issuer
constexpr int kRing = 3;

__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  // MN-major, 128B swizzle: 64 contiguous values (128 B) along N per row of K, 8 K-rows per 1024-byte atom;
  // LBO = stride between 64-value groups along N, SBO = stride between 8-row groups along K.
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

// 2^x on the special-function unit (PTX ex2.approx.ftz.f32: 2^-inf = +0, results below 2^-126 flush to 0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
// Two float32 values rounded to nearest-even bf16 in one conversion: lo in bits 0-15, hi in bits 16-31.
__device__ __forceinline__ uint32_t pack_bf16x2_rn(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;\n" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};\n" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

template <int DQK, int DV>
struct TcShape {
  static constexpr int QCH = DQK / 64, VCH = DV / 64;
  static constexpr uint32_t QB = 128u * DQK * 2, KB = 128u * DQK * 2, VB = 128u * DV * 2;
  static constexpr uint32_t SLOT = KB > VB ? KB : VB;
  static constexpr uint32_t PB = 128u * 128 * 2;
  // barriers (1 KB), the row-maximum exchange (1 KB), alignment slack (1 KB), tiles
  static constexpr uint32_t SMEM = 3072 + QB + kRing * SLOT + PB;
};

template <int DQK, int DV>
__global__ void __launch_bounds__(kTcThreads, 1) attn_tc_kernel(const __grid_constant__ AttnTcParams p) {
  using S = TcShape<DQK, DV>;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint64_t* q_full = bars;
  uint64_t* ring_full = bars + 1;
  uint64_t* ring_empty = bars + 1 + kRing;
  uint64_t* s_full = bars + 1 + 2 * kRing;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* pv_done = p_full + 1;
  uint64_t* drain = pv_done + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 32);
  float* xchg = reinterpret_cast<float*>(smem + 1024);  // [2 halves][128 rows]
  uint8_t* base = reinterpret_cast<uint8_t*>(((uintptr_t)(smem + 2048) + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = base;
  uint8_t* sRing = base + S::QB;
  uint8_t* sP = sRing + kRing * S::SLOT;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = p.ntiles - 1 - (int)blockIdx.x;  // the longest key ranges start first
  const int hk = blockIdx.y;
  const int G = p.G, rows = p.T * G;
  const int r0 = tile * 128;
  const int t_first = r0 / G, t_last = min(rows - 1, r0 + 127) / G;
  const int qfirst = p.pos0 + t_first, qlast = p.pos0 + t_last;
  const int klo = p.window > 0 ? max(0, qfirst - p.window + 1) : 0;
  const int kbase = klo & ~127;
  // this split's key blocks [b_begin, b_begin + nblocks) of the tile's range (decode splits the keys)
  const int nball = (qlast - kbase) / 128 + 1;
  const int per = (nball + p.splits - 1) / p.splits;
  const int b_begin = min(nball, (int)blockIdx.z * per);
  const int nblocks = min(nball, b_begin + per) - b_begin;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&ring_full[i], 1);
      mbar_init(&ring_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 256);
    }
    mbar_init(p_full, 256);
    mbar_init(pv_done, 1);
    mbar_init(drain, 1);
    mbar_fence_init();
  }
  if (warp == 9) {
    tc::tmem_alloc(tslot, 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tslot;
  pdl_wait();  // q and the cache come from the preceding kernel (programmatic dependent launch)
  pdl_launch_dependents();
  const uint32_t tS[2] = {tbase, tbase + 128};
  const uint32_t tO = tbase + 256;
  bool ok = true;

  if (warp == 8) {
    if (lane == 0) {  // ---------------------------------------------------------------- TMA producer
      tma_prefetch_map(&p.qmap);
      tma_prefetch_map(&p.kmap);
      tma_prefetch_map(&p.vmap);
      const uint64_t pol = tc::l2_evict_normal_policy();
      mbar_arrive_expect_tx(q_full, S::QB);
#pragma unroll
      for (int c = 0; c < S::QCH; ++c) tma_load_3d(sQ + c * 16384, &p.qmap, c * 64, hk * G, t_first, q_full, pol);
      int issued = 0;
      for (int j = 0; j < nblocks && ok; ++j) {
        const int slot0 = (kbase + (b_begin + j) * 128) % p.cap;
        for (int half = 0; half < 2; ++half) {
          const int li = 2 * j + half, s = li % kRing;
          if (!mbar_wait(&ring_empty[s], (uint32_t)(((li / kRing) & 1) ^ 1))) {
            ok = false;
            break;
          }
          uint8_t* dst = sRing + s * S::SLOT;
          if (half == 0) {
            mbar_arrive_expect_tx(&ring_full[s], S::KB);
#pragma unroll
            for (int c = 0; c < S::QCH; ++c) tma_load_3d(dst + c * 16384, &p.kmap, c * 64, slot0, hk, &ring_full[s], pol);
          } else {
            mbar_arrive_expect_tx(&ring_full[s], S::VB);
#pragma unroll
            for (int c = 0; c < S::VCH; ++c) tma_load_3d(dst + c * 16384, &p.vmap, c * 64, slot0, hk, &ring_full[s], pol);
          }
          ++issued;
        }
      }
      // no copy may still be landing when the CTA exits: wait for the last copy of every slot and for Q
      for (int li = issued - 1; li >= 0 && li >= issued - kRing; --li)
        if (!mbar_wait(&ring_full[li % kRing], (uint32_t)((li / kRing) & 1))) ok = false;
      if (!mbar_wait(q_full, 0)) ok = false;
    }
  } else if (warp == 9) {
    if (lane == 0) {  // ----------------------------------------------------------------- MMA issuer
      const uint32_t idesc_s = tc::idesc_bf16(128, 128);
      const uint32_t idesc_o = tc::idesc_bf16(128, DV) | (1u << 16);  // B = V, MN-major
      const uint32_t aq = smem_u32(sQ), ap = smem_u32(sP);
      auto issue_pv = [&](int jj) -> bool {
        const int lv = 2 * jj + 1, sv = lv % kRing;
        if (!mbar_wait(p_full, (uint32_t)(jj & 1))) return false;
        if (!mbar_wait(&ring_full[sv], (uint32_t)((lv / kRing) & 1))) return false;
        tc::tc_fence_after();
        const uint32_t av = smem_u32(sRing + sv * S::SLOT);
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc::tc_mma_f16(tO, tc::desc_sw128(ap + c * 16384 + kk * 32),
                           desc_mn_sw128(av + (uint32_t)(c * 64 + kk * 16) * 128u, 16384u, 1024u), idesc_o,
                           (jj > 0 || (c | kk) != 0) ? 1u : 0u);
        tc::tc_commit(pv_done);
        tc::tc_commit(&ring_empty[sv]);
        return true;
      };
      if (!mbar_wait(q_full, 0)) ok = false;
      tc::tc_fence_after();
      for (int j = 0; j < nblocks && ok; ++j) {
        const int lk = 2 * j, sk = lk % kRing, sb = j & 1;
        if (!mbar_wait(&ring_full[sk], (uint32_t)((lk / kRing) & 1))) {
          ok = false;
          break;
        }
        if (j >= 2 && !mbar_wait(&s_free[sb], (uint32_t)(((j >> 1) - 1) & 1))) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t ak = smem_u32(sRing + sk * S::SLOT);
#pragma unroll
        for (int c = 0; c < S::QCH; ++c)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc::tc_mma_f16(tS[sb], tc::desc_sw128(aq + c * 16384 + kk * 32), tc::desc_sw128(ak + c * 16384 + kk * 32),
                           idesc_s, (c | kk) != 0 ? 1u : 0u);
        tc::tc_commit(&s_full[sb]);
        tc::tc_commit(&ring_empty[sk]);
        if (j >= 1 && !issue_pv(j - 1)) ok = false;
      }
      if (ok && nblocks > 0 && !issue_pv(nblocks - 1)) ok = false;
      tc::tc_commit(drain);  // every MMA issued above has completed once this arrives
      if (!mbar_wait(drain, 0)) ok = false;
    }
  } else {  // ---------------------------------------- softmax: thread = (row, column half), warpgroup = half
    const int h = warp >> 2;                 // columns [64 h, 64 h + 64) of S, P and O
    const int r = threadIdx.x & 127;         // query row = TMEM lane
    const int gr = r0 + r;
    const bool row_ok = gr < rows;
    const int t = row_ok ? gr / G : t_last;
    const int qpos = p.pos0 + t;
    const int lo = p.window > 0 ? qpos - p.window + 1 : 0;  // first visible key position (may be negative)
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const float sl2 = p.scale_log2;
    float m_ref = -INFINITY, l = 0.f;        // l: this half's share of the row sum
    const uint32_t prow = smem_u32(sP) + (uint32_t)h * 16384u + (uint32_t)r * 128u;
    // Both halves of a row must use one maximum: each writes its half's maximum, a named barrier over
    // the 256 softmax threads, each reads the other's.  A second barrier before the next write keeps
    // the single buffer free of races.  No thread leaves the loop early (the barriers count on all
    // 256); after a timed-out wait the loop runs on without waiting and the status records it.
    auto exchange = [&](float mine) -> float {
      asm volatile("bar.sync 1, 256;\n" ::: "memory");
      xchg[h * 128 + r] = mine;
      asm volatile("bar.sync 2, 256;\n" ::: "memory");
      return xchg[(h ^ 1) * 128 + r];
    };
    for (int j = 0; j < nblocks; ++j) {
      const int sb = j & 1;
      if (ok) ok = mbar_wait(&s_full[sb], (uint32_t)((j >> 1) & 1));
      ok = __all_sync(0xFFFFFFFFu, ok);
      tc::tc_fence_after();
      float s[4][16];
#pragma unroll
      for (int c = 0; c < 4; ++c) tc::tmem_ld<16>(tS[sb] + lane_off + h * 64 + c * 16, s[c]);
      tc::tmem_wait_ld();
      tc::tc_fence_before();
      mbar_arrive(&s_free[sb]);
      // The raw-score maximum (the scale is positive, so it orders the scaled scores alike); only blocks
      // that reach past a row's visible range mask by column.
      const int kp0 = kbase + (b_begin + j) * 128 + h * 64;
      const int c_lo = lo - kp0, c_hi = qpos - kp0;  // visible columns [c_lo, c_hi] of this half
      if (c_lo > 0 || c_hi < 63) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int col = c * 16 + e;
            if (col < c_lo || col > c_hi) s[c][e] = -INFINITY;
          }
      }
      float mxa[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float a = fmaxf(s[c][0], s[c][1]);
#pragma unroll
        for (int e = 2; e < 16; ++e) a = fmaxf(a, s[c][e]);
        mxa[c] = a;
      }
      const float mine = fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3]));
      const float mx = fmaxf(mine, exchange(mine)) * sl2;
      float alpha = 1.f;
      bool rescale = false;
      if (mx > -INFINITY) {
        if (m_ref == -INFINITY) {
          m_ref = mx;
        } else if (mx > m_ref + 8.f) {
          alpha = ex2_approx(m_ref - mx);
          m_ref = mx;
          rescale = true;
        }
      }
      // P = bf16(2^(s * scale * log2e - m)): one FFMA and one ex2 per score (2^-inf = 0 for masked
      // scores; a row with nothing visible yet uses m = 0), one conversion per pair; the half's row sum
      // takes the float32 values in four independent partial sums
      const float nm = (m_ref == -INFINITY) ? 0.f : -m_ref;
      uint32_t pk[32];
      float rsa[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float p0 = ex2_approx(fmaf(s[(2 * i) >> 4][(2 * i) & 15], sl2, nm));
        const float p1 = ex2_approx(fmaf(s[(2 * i + 1) >> 4][(2 * i + 1) & 15], sl2, nm));
        rsa[i & 3] += p0 + p1;
        pk[i] = pack_bf16x2_rn(p0, p1);
      }
      l = l * alpha + ((rsa[0] + rsa[1]) + (rsa[2] + rsa[3]));
      if (j > 0) {  // P_{j-1} V_{j-1} has completed: the P buffer is free and O is stable
        if (ok) ok = mbar_wait(pv_done, (uint32_t)((j - 1) & 1));
        ok = __all_sync(0xFFFFFFFFu, ok);
        tc::tc_fence_after();
      }
      if (__any_sync(0xFFFFFFFFu, rescale)) {  // warp-collective TMEM access; alpha = 1 for the other rows
#pragma unroll
        for (int c = 0; c < DV / 2; c += 16) {
          float o[16];
          tc::tmem_ld<16>(tO + lane_off + h * (DV / 2) + c, o);
          tc::tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) o[e] *= alpha;
          tmem_st16(tO + lane_off + h * (DV / 2) + c, o);
        }
        tmem_wait_st();
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint32_t addr = prow + (uint32_t)((u ^ (r & 7)) << 4);
        st_shared_v4(addr, pk[u * 4], pk[u * 4 + 1], pk[u * 4 + 2], pk[u * 4 + 3]);
      }
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      mbar_arrive(p_full);
    }
    if (nblocks > 0) {
      if (ok) ok = mbar_wait(pv_done, (uint32_t)((nblocks - 1) & 1));
      ok = __all_sync(0xFFFFFFFFu, ok);
    }
    const float l_row = l + exchange(l);  // both halves' sums (every softmax thread takes part)
    const int qh = hk * G + (row_ok ? gr % G : 0);
    tc::tc_fence_after();
    if (ok && p.splits > 1) {  // unnormalised partial (m in log2 units, l, O) for the merge kernel
      const size_t prow_g = (size_t)blockIdx.z * p.T * p.nq + (size_t)t * p.nq + qh;
      float* dst = p.part_o + prow_g * DV + h * (DV / 2);
#pragma unroll
      for (int c = 0; c < DV / 2; c += 16) {
        float o[16];
        tc::tmem_ld<16>(tO + lane_off + h * (DV / 2) + c, o);
        tc::tmem_wait_ld();
        if (row_ok) {
          float4* d4 = reinterpret_cast<float4*>(dst + c);
#pragma unroll
          for (int e = 0; e < 4; ++e)  // an empty split holds no P.V result: zeros
            d4[e] = nblocks > 0 ? make_float4(o[4 * e], o[4 * e + 1], o[4 * e + 2], o[4 * e + 3])
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      if (row_ok && h == 0) *reinterpret_cast<float2*>(p.part_ml + prow_g * 2) = make_float2(m_ref, l_row);
    } else if (ok) {
      float f;
      if (p.sinks) {
        const float sk = p.sinks[qh] * 1.4426950408889634f;
        const float Mn = fmaxf(m_ref, sk);
        const float sc = (m_ref == -INFINITY) ? 0.f : exp2f(m_ref - Mn);
        f = sc / (l_row * sc + exp2f(sk - Mn));
      } else {
        f = l_row > 0.f ? 1.f / l_row : 0.f;
      }
      uint16_t* dst = p.out + ((size_t)t * p.nq + qh) * DV + h * (DV / 2);
#pragma unroll
      for (int c = 0; c < DV / 2; c += 16) {
        float o[16];
        tc::tmem_ld<16>(tO + lane_off + h * (DV / 2) + c, o);
        tc::tmem_wait_ld();
        uint32_t w[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) w[e] = pack_bf16x2_rn(o[2 * e] * f, o[2 * e + 1] * f);
        if (row_ok) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c);
          d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
          d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
      }
    }
  }
  if (!ok && p.status) set_status(p.status, MIMO_ETIMEOUT);
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, 512);
  }
}

template <int DQK, int DV>
cudaError_t launch_tc(AttnTcParams& p, cudaStream_t st) {
  using S = TcShape<DQK, DV>;
  static bool attr_set[128] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 128 && !attr_set[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(attn_tc_kernel<DQK, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::SMEM);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  return launch_k(attn_tc_kernel<DQK, DV>, dim3(p.ntiles, p.nkv, p.splits), dim3(kTcThreads), S::SMEM, st, p);
}

}  // namespace

bool attn_tc_supported(const AttnParams& a) {
  return ((a.dqk == 192 && a.dv == 128) || (a.dqk == 128 && a.dv == 128)) && a.G >= 1 && a.G <= 128 &&
         128 % a.G == 0 && a.cap % 128 == 0;
}

cudaError_t launch_attention_tc(const AttnParams& a, int32_t* status, cudaStream_t st) {
  AttnTcParams p;
  std::memset(&p, 0, sizeof(p));
  cudaError_t e = bf16_map3(&p.qmap, a.q, (uint64_t)a.dqk, (uint64_t)a.nq, (uint64_t)a.T, a.G, 128 / a.G);
  if (e == cudaSuccess) e = bf16_map3(&p.kmap, a.k, (uint64_t)a.dqk, (uint64_t)a.cap, (uint64_t)a.nkv, 128, 1);
  if (e == cudaSuccess) e = bf16_map3(&p.vmap, a.v, (uint64_t)a.dv, (uint64_t)a.cap, (uint64_t)a.nkv, 128, 1);
  if (e != cudaSuccess) return e;
  p.sinks = a.sinks;
  p.out = a.out;
  p.status = status;
  p.T = a.T, p.nq = a.nq, p.nkv = a.nkv, p.G = a.G, p.cap = a.cap, p.window = a.window, p.pos0 = a.pos0;
  p.ntiles = (a.T * a.G + 127) / 128;
  p.splits = a.splits;
  p.part_o = a.part_o;
  p.part_ml = a.part_ml;
  p.scale_log2 = a.scale_log2;
  if (a.dqk == 192) return launch_tc<192, 128>(p, st);
  return launch_tc<128, 128>(p, st);
}

}  // namespace mimo
