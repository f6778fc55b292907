// The rest of the MiMo decoder layer around the MoE block (engine/mimo_stream/mimo_v2.py:66-162, 242-262;
// the engine's per-layer loop engine/mimo_stream/model.py:294-300):
//
//   r   = input_layernorm(x)                                  (rmsnorm_kernel, norm.cu)
//   qkv = r @ [Wq | Wk | Wv]^T                                (library GEMM, cuBLAS)
//   q,k = RoPE(q,k; offset) on the first rotary_dim dims,     rope_store_kernel
//   v   = v * attention_value_scale, k/v appended to the cache
//   o   = softmax_with_sinks(q k^T * scale, mask) v           attn_kernel (+ attn_merge_kernel)
//   h   = x + o @ Wo^T ;  r2 = post_attention_layernorm(h)    add_rmsnorm_kernel (after a library GEMM)
//   y   = MoE(r2)  or  down(swiglu(gate(r2), up(r2)))         MoE block / swiglu_kernel
//   out = h + y                                               add_kernel
//
// Semantics restated from the reference and the MLX operators it calls (mlx 0.32.2 / mlx-lm 0.31.3, not
// vendored in the reference project):
//  * RoPE (mlx_lm initialize_rope -> nn.RoPE(dims, traditional=False, base)): for i < dims/2 the pair
//    (x[i], x[i + dims/2]) is rotated by the angle pos * base^(-2i/dims); dims beyond rotary_dim pass through.
//    Here the angle and rotation are evaluated in float64 and rounded once to float32, then to bf16 (MLX
//    evaluates them in float32: ulp-level parity unpinned).
//  * v scale (mimo_v2.py:130-131): bf16 values times a Python float, i.e. bf16(v * bf16(scale)); the caller
//    passes the scale already rounded to bf16.
//  * attention (mlx fast.scaled_dot_product_attention with `sinks`): per query head h the softmax runs over
//    the scaled scores q.k * head_dim^-0.5 of the visible keys plus one extra logit sinks[h] that has no
//    value row; keys visible to a query at position p: kpos <= p (causal) and, for sliding-window layers,
//    kpos > p - window (mlx_lm create_attention_mask / RotatingKVCache(max_size=window)).  GQA: query head h
//    reads kv head h / (n_heads / n_kv_heads).
//
// KV cache layout in HBM: k [n_kv][cap][head_dim], v [n_kv][cap][v_head_dim] bf16, position p in slot
// p % cap (a ring for sliding-window layers; cap >= every position for full attention), so one kv head's
// keys are contiguous rows and a 64-key block is 64 row copies.
//
// attn_kernel is a flash-attention forward on the bf16 mma.sync tensor path (m16n8k16, float32 accumulate):
// one CTA = 64 query rows of one kv head (the G = n_heads / n_kv_heads query heads of consecutive tokens,
// token-major, so every K/V block loaded to shared memory serves all heads of the group), four warps of
// 16 rows, K/V blocks of 64 keys double-buffered by cp.async, online softmax in float32 (exp2 domain, the
// row sum from the float32 P), P rounded to bf16 for the P.V product.  Decode (few rows, many keys) splits the keys over CTAs
// (grid z); attn_merge_kernel folds the splits and the sink in a fixed split order.
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "kernels.h"

namespace mimo {

namespace {

constexpr int kAttnRows = 64;     // query rows per CTA
constexpr int kAttnKeys = 64;     // keys per block
constexpr int kAttnThreads = 128;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // src-size 0 fills the 16 bytes with zeros
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Two float32 values rounded to nearest-even bf16 in one conversion: lo in bits 0-15, hi in bits 16-31.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;\n" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// 2^x on the special-function unit (PTX ex2.approx.ftz.f32: 2^-inf = +0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

// Byte offset of 16-byte chunk c of row r in a tile whose rows hold CH chunks; the chunk index is XORed
// with the row's low 3 bits so the eight rows an ldmatrix reads fall in eight different bank groups.
template <int CH>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)(r * CH + (c ^ (r & 7))) * 16u;
}

template <int DQK, int DV>
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(AttnParams p) {
  static_assert(DQK % 64 == 0 && DV % 64 == 0, "head dims are multiples of 64");
  constexpr int QCH = DQK / 8, VCH = DV / 8;  // 16-byte chunks per row
  constexpr int KSTEPS = DQK / 16;            // k-steps of S = Q K^T
  constexpr int ONT = DV / 8;                 // n-tiles of O
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;
  uint8_t* sK[2] = {smem + kAttnRows * DQK * 2, smem + kAttnRows * DQK * 2 + kAttnKeys * (DQK + DV) * 2};
  uint8_t* sV[2] = {sK[0] + kAttnKeys * DQK * 2, sK[1] + kAttnKeys * DQK * 2};
  pdl_wait();  // inputs come from the preceding kernel (programmatic dependent launch)
  pdl_launch_dependents();

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hk = blockIdx.y, split = blockIdx.z;
  const int G = p.G, rows = p.T * G;
  const int r0 = blockIdx.x * kAttnRows;
  const int t_first = r0 / G, t_last = min(rows - 1, r0 + kAttnRows - 1) / G;
  const int qpos_first = p.pos0 + t_first, qpos_last = p.pos0 + t_last;
  const int klo = p.window > 0 ? max(0, qpos_first - p.window + 1) : 0;
  const int nkeys = qpos_last - klo + 1;
  const int nblocks = (nkeys + kAttnKeys - 1) / kAttnKeys;
  const int per = (nblocks + p.splits - 1) / p.splits;
  const int b_begin = min(nblocks, split * per), b_end = min(nblocks, b_begin + per);

  // ---- Q tile (rows beyond T*G are zero) and the first K/V block
  for (int i = tid; i < kAttnRows * QCH; i += kAttnThreads) {
    const int r = i / QCH, c = i % QCH, gr = r0 + r;
    const bool ok = gr < rows;
    const int t = ok ? gr / G : 0, qh = hk * G + (ok ? gr % G : 0);
    const uint16_t* src = p.q + ((size_t)t * p.nq + qh) * DQK + c * 8;
    cp_async16(smem_u32(sQ) + swz<QCH>(r, c), src, ok);
  }
  cp_async_commit();
  const uint16_t* kbase = p.k + (size_t)hk * p.cap * DQK;
  const uint16_t* vbase = p.v + (size_t)hk * p.cap * DV;
  auto load_kv = [&](int b, int stage) {
    const int kp0 = klo + b * kAttnKeys;
    for (int i = tid; i < kAttnKeys * QCH; i += kAttnThreads) {
      const int r = i / QCH, c = i % QCH, kp = kp0 + r;
      const bool ok = kp <= qpos_last;
      const uint16_t* src = kbase + (size_t)(ok ? kp % p.cap : 0) * DQK + c * 8;
      cp_async16(smem_u32(sK[stage]) + swz<QCH>(r, c), src, ok);
    }
    for (int i = tid; i < kAttnKeys * VCH; i += kAttnThreads) {
      const int r = i / VCH, c = i % VCH, kp = kp0 + r;
      const bool ok = kp <= qpos_last;
      const uint16_t* src = vbase + (size_t)(ok ? kp % p.cap : 0) * DV + c * 8;
      cp_async16(smem_u32(sV[stage]) + swz<VCH>(r, c), src, ok);
    }
    cp_async_commit();
  };
  if (b_begin < b_end) load_kv(b_begin, 0);

  // Rows of this thread: g and g + 8 of the warp's 16.
  const int g = lane >> 2, cq = lane & 3;
  int qpos_row[2];
  bool row_ok[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int gr = r0 + warp * 16 + g + h * 8;
    row_ok[h] = gr < rows;
    qpos_row[h] = p.pos0 + (row_ok[h] ? gr / G : t_last);
  }

  uint32_t qf[KSTEPS][4];
  float o[ONT][4];
#pragma unroll
  for (int j = 0; j < ONT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const float sl2 = p.scale_log2;

  for (int b = b_begin; b < b_end; ++b) {
    const int stage = (b - b_begin) & 1;
    if (b + 1 < b_end) {
      load_kv(b + 1, stage ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (b == b_begin) {
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
        const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = kk * 2 + (lane >> 4);
        ldsm_x4(smem_u32(sQ) + swz<QCH>(r, c), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    // ---- S = Q K^T for 16 rows x 64 keys
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    const uint32_t kb = smem_u32(sK[stage]);
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int r = np * 16 + (lane & 7) + (lane >> 4) * 8;
        const int c = kk * 2 + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb + swz<QCH>(r, c), b0, b1, b2, b3);
        mma_16816_bf16(s[2 * np], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1, s[2 * np]);
        mma_16816_bf16(s[2 * np + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b2, b3, s[2 * np + 1]);
      }
    }
    // ---- mask, online softmax (exp2 domain)
    const int kp0 = klo + b * kAttnKeys;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int qp = qpos_row[h];
      const int lo = p.window > 0 ? qp - p.window + 1 : 0;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int kp = kp0 + j * 8 + cq * 2 + e;
          float v = s[j][h * 2 + e] * sl2;
          if (kp > qp || kp < lo) v = -INFINITY;
          s[j][h * 2 + e] = v;
          mx = fmaxf(mx, v);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 2));
      const float m_new = fmaxf(m_run[h], mx);
      const float alpha = (m_new == -INFINITY) ? 1.f : exp2f(m_run[h] - m_new);
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float v = s[j][h * 2 + e];
          const float pv = ex2_approx(v - (m_new == -INFINITY ? 0.f : m_new));  // 2^-inf = 0
          s[j][h * 2 + e] = pv;
          rs += pv;
        }
      }
      l_run[h] = l_run[h] * alpha + rs;
      m_run[h] = m_new;
#pragma unroll
      for (int j = 0; j < ONT; ++j) {
        o[j][h * 2] *= alpha;
        o[j][h * 2 + 1] *= alpha;
      }
    }
    // ---- O += P V
    const uint32_t vb = smem_u32(sV[stage]);
#pragma unroll
    for (int kk = 0; kk < kAttnKeys / 16; ++kk) {
      const uint32_t a0 = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < ONT / 2; ++np) {
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = np * 2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vb + swz<VCH>(r, c), b0, b1, b2, b3);
        mma_16816_bf16(o[2 * np], a0, a1, a2, a3, b0, b1, o[2 * np]);
        mma_16816_bf16(o[2 * np + 1], a0, a1, a2, a3, b2, b3, o[2 * np + 1]);
      }
    }
    __syncthreads();  // this stage is refilled by the next iteration's load
  }
  if (b_begin >= b_end) cp_async_wait<0>();

  // ---- row sums over the quad, then either the final normalisation (with the sink) or a split partial
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_run[h] += __shfl_xor_sync(0xFFFFFFFFu, l_run[h], 1);
    l_run[h] += __shfl_xor_sync(0xFFFFFFFFu, l_run[h], 2);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (!row_ok[h]) continue;
    const int gr = r0 + warp * 16 + g + h * 8;
    const int t = gr / G, qh = hk * G + gr % G;
    const size_t row = (size_t)t * p.nq + qh;
    if (p.splits == 1) {
      float M = m_run[h], L = l_run[h];
      if (p.sinks) {
        const float sk = p.sinks[qh] * kLog2e;
        const float Mn = fmaxf(M, sk);
        L = (M == -INFINITY ? 0.f : L * exp2f(M - Mn)) + exp2f(sk - Mn);
        const float f = (M == -INFINITY ? 0.f : exp2f(M - Mn)) / L;
#pragma unroll
        for (int j = 0; j < ONT; ++j) {
          o[j][h * 2] *= f;
          o[j][h * 2 + 1] *= f;
        }
      } else {
        const float f = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
        for (int j = 0; j < ONT; ++j) {
          o[j][h * 2] *= f;
          o[j][h * 2 + 1] *= f;
        }
      }
      uint16_t* dst = p.out + row * DV;
#pragma unroll
      for (int j = 0; j < ONT; ++j)
        *reinterpret_cast<uint32_t*>(dst + j * 8 + cq * 2) = pack_bf16x2(o[j][h * 2], o[j][h * 2 + 1]);
    } else {
      const size_t prow = (size_t)split * p.T * p.nq + row;
      float* dst = p.part_o + prow * DV;
#pragma unroll
      for (int j = 0; j < ONT; ++j)
        *reinterpret_cast<float2*>(dst + j * 8 + cq * 2) = make_float2(o[j][h * 2], o[j][h * 2 + 1]);
      if (cq == 0) *reinterpret_cast<float2*>(p.part_ml + prow * 2) = make_float2(m_run[h], l_run[h]);
    }
  }
}

// One CTA of DV threads per (token, query head): folds the splits' (m, l, O) with the sink.  Warp 0 reads the
// splits' (m, l) in parallel (split s on lane s % 32) and takes their maximum and the sum of l * 2^(m - M) by
// butterflies (a fixed order); then every thread sums its output value over the splits in split order, the
// partial rows of consecutive threads contiguous (coalesced), several splits' loads in flight.
template <int DV>
__global__ void __launch_bounds__(DV) attn_merge_kernel(AttnParams p) {
  __shared__ float fs[64];
  __shared__ float inv_l;
  pdl_wait();  // inputs come from the preceding kernel (programmatic dependent launch)
  pdl_launch_dependents();
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  const size_t stride = (size_t)p.T * p.nq;
  if (tid < 32) {
    float2 ml[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int s = lane + 32 * k;
      ml[k] = s < p.splits ? *reinterpret_cast<const float2*>(p.part_ml + ((size_t)s * stride + row) * 2)
                           : make_float2(-INFINITY, 0.f);
    }
    float M = fmaxf(ml[0].x, ml[1].x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
    const float sk = p.sinks ? p.sinks[row % p.nq] * kLog2e : -INFINITY;
    M = fmaxf(M, sk);
    float L = 0.f;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float f = ml[k].x == -INFINITY ? 0.f : exp2f(ml[k].x - M);
      fs[lane + 32 * k] = f;
      L += ml[k].y * f;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xFFFFFFFFu, L, o);
    if (p.sinks) L += exp2f(sk - M);
    if (lane == 0) inv_l = L > 0.f ? 1.f / L : 0.f;
  }
  __syncthreads();
  const float* src = p.part_o + (size_t)row * DV + tid;
  float acc = 0.f;
#pragma unroll 8
  for (int s = 0; s < p.splits; ++s) acc = fmaf(src[(size_t)s * stride * DV], fs[s], acc);
  p.out[(size_t)row * DV + tid] = (uint16_t)f32_to_bf16(acc * inv_l);
}

// Grid (token slices, head groups): a CTA walks its tokens; per token it computes the cos/sin of every rotary
// pair once (float64: the angle pos * theta^(-2i/rot) and its sine and cosine), then its 16 warps take the
// heads (all of them, or the CTA's group of 16 when the grid has several) of the packed projection row
// [q heads | k heads | v heads]: RoPE on q and k (float64 rotation, rounded once to
// float32, then to bf16), v * v_scale, k/v into the cache slot; the value rows and the dims past the rotary
// ones move as bf16 pairs (every row offset is an even number of values).  (A float32 table moves
// near-cancelling rotations by a few bf16 ulps.)
__global__ void __launch_bounds__(512) rope_store_kernel(RopeParams p) {
  __shared__ double2 cs_tab[128];
  pdl_wait();  // inputs come from the preceding kernel (programmatic dependent launch)
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = p.rot / 2;
  const int heads = p.nq + p.nkv;
  const size_t rowlen = (size_t)p.nq * p.dqk + (size_t)p.nkv * (p.dqk + p.dv);
  for (int t = blockIdx.x; t < p.T; t += gridDim.x) {
    const int pos = p.pos0 + t;
    __syncthreads();  // the previous token's table is no longer read
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
      const double inv_freq = exp(-(double)(2 * i) / (double)p.rot * p.log_base);
      double sn, cs;
      sincos((double)pos * inv_freq, &sn, &cs);
      cs_tab[i] = make_double2(cs, sn);
    }
    __syncthreads();
    const uint16_t* row = p.qkv + (size_t)t * rowlen;
    const int slot = pos % p.cap;
    const int h_lo = gridDim.y > 1 ? blockIdx.y * 16 : 0, h_hi = gridDim.y > 1 ? min(heads, h_lo + 16) : heads;
    for (int hd = h_lo + warp; hd < h_hi; hd += blockDim.x / 32) {
      const uint16_t* src;
      uint16_t* dst;
      if (hd < p.nq) {
        src = row + (size_t)hd * p.dqk;
        dst = p.q + ((size_t)t * p.nq + hd) * p.dqk;
      } else {
        const int hk = hd - p.nq;
        src = row + (size_t)p.nq * p.dqk + (size_t)hk * p.dqk;
        dst = p.kc + ((size_t)hk * p.cap + slot) * p.dqk;
        const uint32_t* vs = reinterpret_cast<const uint32_t*>(row + (size_t)p.nq * p.dqk +
                                                               (size_t)p.nkv * p.dqk + (size_t)hk * p.dv);
        uint32_t* vd = reinterpret_cast<uint32_t*>(p.vc + ((size_t)hk * p.cap + slot) * p.dv);
#pragma unroll 4
        for (int i = lane; i < p.dv / 2; i += 32) {
          const uint32_t w = vs[i];
          vd[i] = p.has_vscale ? (f32_to_bf16(bf16_to_f32(w & 0xFFFFu) * p.v_scale) |
                                  (f32_to_bf16(bf16_to_f32(w >> 16) * p.v_scale) << 16))
                               : w;
        }
      }
      for (int i = lane; i < half; i += 32) {
        const double2 c = cs_tab[i];
        const double x1 = bf16_to_f32(src[i]), x2 = bf16_to_f32(src[i + half]);
        dst[i] = (uint16_t)f32_to_bf16(__double2float_rn(x1 * c.x - x2 * c.y));
        dst[i + half] = (uint16_t)f32_to_bf16(__double2float_rn(x1 * c.y + x2 * c.x));
      }
      const uint32_t* s2 = reinterpret_cast<const uint32_t*>(src + p.rot);
      uint32_t* d2 = reinterpret_cast<uint32_t*>(dst + p.rot);
#pragma unroll 4
      for (int i = lane; i < (p.dqk - p.rot) / 2; i += 32) d2[i] = s2[i];
    }
  }
}

// Decode-sized calls (T <= 16): one warp per (token, head) of the packed projection row [q heads | k heads |
// v heads].  Lane l evaluates the cos/sin of the rotary pairs l, l + 32, ... in float64 (the same angle and
// rotation as rope_store_kernel, so the results are bit-identical) before the grid dependency wait, so that
// work overlaps the preceding kernel's tail; then RoPE on q or k, v * v_scale, k/v into the cache slot.
// Value rows, and the dims past the rotary ones when rot is a multiple of 8, move as 16-byte vectors (every
// row offset is a multiple of 8 values); other pass-through dims move as bf16 pairs.  No shared memory and
// no block barrier.  About half the time of rope_store_kernel at 1 and 8 tokens; at 2048 tokens the
// token-walking kernel is faster.
constexpr int kRopeThreads = 256;

__device__ __forceinline__ uint32_t scale_bf16x2(uint32_t w, float s) {
  return f32_to_bf16(bf16_to_f32(w & 0xFFFFu) * s) | (f32_to_bf16(bf16_to_f32(w >> 16) * s) << 16);
}

template <int PAIRS>  // rotary pairs per lane: rot <= 64 * PAIRS
__global__ void __launch_bounds__(kRopeThreads) rope_store_decode_kernel(RopeParams p) {
  const int lane = threadIdx.x & 31;
  const long long item = (long long)blockIdx.x * (kRopeThreads / 32) + (threadIdx.x >> 5);
  const int heads = p.nq + p.nkv;
  const bool active = item < (long long)p.T * heads;
  const int t = active ? (int)(item / heads) : 0, hd = active ? (int)(item % heads) : 0;
  const int pos = p.pos0 + t, half = p.rot / 2;
  double cs[PAIRS], sn[PAIRS];
#pragma unroll
  for (int j = 0; j < PAIRS; ++j) {
    const int i = lane + 32 * j;
    cs[j] = 1.0, sn[j] = 0.0;
    if (i < half) {
      const double inv_freq = exp(-(double)(2 * i) / (double)p.rot * p.log_base);
      sincos((double)pos * inv_freq, &sn[j], &cs[j]);
    }
  }
  pdl_wait();  // the projection rows come from the preceding kernel (programmatic dependent launch)
  pdl_launch_dependents();
  if (!active) return;  // whole warps only: no barrier follows
  const int slot = pos % p.cap;
  const size_t rowlen = (size_t)p.nq * p.dqk + (size_t)p.nkv * (p.dqk + p.dv);
  const uint16_t* __restrict__ row = p.qkv + (size_t)t * rowlen;
  const bool vec_tail = (p.rot & 7) == 0;
  const uint16_t* __restrict__ src;
  uint16_t* __restrict__ dst;
  if (hd < p.nq) {
    src = row + (size_t)hd * p.dqk;
    dst = p.q + ((size_t)t * p.nq + hd) * p.dqk;
  } else {
    const int hk = hd - p.nq;
    src = row + (size_t)p.nq * p.dqk + (size_t)hk * p.dqk;
    dst = p.kc + ((size_t)hk * p.cap + slot) * p.dqk;
    const uint4* __restrict__ vs = reinterpret_cast<const uint4*>(row + (size_t)p.nq * p.dqk +
                                                                  (size_t)p.nkv * p.dqk + (size_t)hk * p.dv);
    uint4* __restrict__ vd = reinterpret_cast<uint4*>(p.vc + ((size_t)hk * p.cap + slot) * p.dv);
    for (int i = lane; i < p.dv / 8; i += 32) {
      uint4 w = vs[i];
      if (p.has_vscale) {
        w.x = scale_bf16x2(w.x, p.v_scale), w.y = scale_bf16x2(w.y, p.v_scale);
        w.z = scale_bf16x2(w.z, p.v_scale), w.w = scale_bf16x2(w.w, p.v_scale);
      }
      vd[i] = w;
    }
  }
#pragma unroll
  for (int j = 0; j < PAIRS; ++j) {
    const int i = lane + 32 * j;
    if (i < half) {
      const double x1 = bf16_to_f32(src[i]), x2 = bf16_to_f32(src[i + half]);
      dst[i] = (uint16_t)f32_to_bf16(__double2float_rn(x1 * cs[j] - x2 * sn[j]));
      dst[i + half] = (uint16_t)f32_to_bf16(__double2float_rn(x1 * sn[j] + x2 * cs[j]));
    }
  }
  if (vec_tail) {
    const uint4* __restrict__ s4 = reinterpret_cast<const uint4*>(src + p.rot);
    uint4* __restrict__ d4 = reinterpret_cast<uint4*>(dst + p.rot);
    for (int i = lane; i < (p.dqk - p.rot) / 8; i += 32) d4[i] = s4[i];
  } else {
    const uint32_t* __restrict__ s2 = reinterpret_cast<const uint32_t*>(src + p.rot);
    uint32_t* __restrict__ d2 = reinterpret_cast<uint32_t*>(dst + p.rot);
    for (int i = lane; i < (p.dqk - p.rot) / 2; i += 32) d2[i] = s2[i];
  }
}

constexpr int kNormThreads = 256;

// h = bf16(x + d); r = RMSNorm(h) with rmsnorm_kernel's reduction order (norm.cu), so r equals
// rmsnorm(h) bit for bit.
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(const uint16_t* __restrict__ x,
                                                                   const uint16_t* __restrict__ d,
                                                                   const uint16_t* __restrict__ weight, int H,
                                                                   float eps, uint16_t* __restrict__ hout,
                                                                   uint16_t* __restrict__ rout) {
  __shared__ float warp_ss[kNormThreads / 32];
  pdl_wait();  // inputs come from the preceding kernel (programmatic dependent launch)
  pdl_launch_dependents();
  const size_t row = (size_t)blockIdx.x * H;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row);
  const uint4* dr = reinterpret_cast<const uint4*>(d + row);
  uint4* hr = reinterpret_cast<uint4*>(hout + row);
  const int chunks = H / 8;
  float ss = 0.f;
  for (int c = threadIdx.x; c < chunks; c += kNormThreads) {
    const uint4 a = __ldg(xr + c), b = __ldg(dr + c);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
    uint32_t hw[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float lo = bf16_round(bf16_to_f32(aw[i] & 0xFFFFu) + bf16_to_f32(bw[i] & 0xFFFFu));
      const float hi = bf16_round(bf16_to_f32(aw[i] >> 16) + bf16_to_f32(bw[i] >> 16));
      ss = __fmaf_rn(lo, lo, ss);
      ss = __fmaf_rn(hi, hi, ss);
      hw[i] = f32_to_bf16(lo) | (f32_to_bf16(hi) << 16);
    }
    hr[c] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xFFFFFFFFu, ss, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) warp_ss[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot = __fadd_rn(tot, warp_ss[i]);
  const float inv = __frsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)H), eps));
  uint4* rr = reinterpret_cast<uint4*>(rout + row);
  const uint4* wr = reinterpret_cast<const uint4*>(weight);
  for (int c = threadIdx.x; c < chunks; c += kNormThreads) {
    const uint4 v = hr[c];  // this thread's own stores above
    const uint32_t hw[4] = {v.x, v.y, v.z, v.w};
    uint32_t ww[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};
    if (weight) {
      const uint4 gw = __ldg(wr + c);
      ww[0] = gw.x, ww[1] = gw.y, ww[2] = gw.z, ww[3] = gw.w;
    }
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float a = bf16_round(__fmul_rn(bf16_to_f32(hw[i] & 0xFFFFu), inv));
      float b = bf16_round(__fmul_rn(bf16_to_f32(hw[i] >> 16), inv));
      if (weight) {
        a = __fmul_rn(bf16_to_f32(ww[i] & 0xFFFFu), a);
        b = __fmul_rn(bf16_to_f32(ww[i] >> 16), b);
      }
      o[i] = f32_to_bf16(a) | (f32_to_bf16(b) << 16);
    }
    rr[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Dense MLP activation (mlx_lm swiglu: silu(gate) * up, each step rounded to bf16):
// out = bf16(bf16(g * bf16(sigmoid(g))) * u); gate_up rows are [gate (I) | up (I)].
__global__ void __launch_bounds__(256) swiglu_kernel(const uint16_t* __restrict__ gu, int T, int I,
                                                     uint16_t* __restrict__ out) {
  pdl_wait();  // inputs come from the preceding kernel (programmatic dependent launch)
  pdl_launch_dependents();
  const size_t n8 = (size_t)T * I / 8;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (size_t)gridDim.x * blockDim.x) {
    const size_t e = i * 8, t = e / I, c = e % I;
    const uint4 gv = __ldg(reinterpret_cast<const uint4*>(gu + t * 2 * I + c));
    const uint4 uv = __ldg(reinterpret_cast<const uint4*>(gu + t * 2 * I + I + c));
    const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float lo = swiglu_ref(bf16_to_f32(gw[k] & 0xFFFFu), bf16_to_f32(uw[k] & 0xFFFFu));
      const float hi = swiglu_ref(bf16_to_f32(gw[k] >> 16), bf16_to_f32(uw[k] >> 16));
      o[k] = f32_to_bf16(lo) | (f32_to_bf16(hi) << 16);
    }
    *reinterpret_cast<uint4*>(out + e) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// out = bf16(a + b) (the decoder layer's residual adds, mimo_v2.py:260-261).
__global__ void __launch_bounds__(256) add_kernel(const uint16_t* __restrict__ a, const uint16_t* __restrict__ b,
                                                  size_t n8, uint16_t* __restrict__ out) {
  pdl_wait();  // inputs come from the preceding kernel (programmatic dependent launch)
  pdl_launch_dependents();
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (size_t)gridDim.x * blockDim.x) {
    const uint4 x = __ldg(reinterpret_cast<const uint4*>(a) + i), y = __ldg(reinterpret_cast<const uint4*>(b) + i);
    const uint32_t xw[4] = {x.x, x.y, x.z, x.w}, yw[4] = {y.x, y.y, y.z, y.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float lo = bf16_to_f32(xw[k] & 0xFFFFu) + bf16_to_f32(yw[k] & 0xFFFFu);
      const float hi = bf16_to_f32(xw[k] >> 16) + bf16_to_f32(yw[k] >> 16);
      o[k] = f32_to_bf16(lo) | (f32_to_bf16(hi) << 16);
    }
    reinterpret_cast<uint4*>(out)[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <int DQK, int DV>
cudaError_t launch_attn_t(const AttnParams& p, cudaStream_t st) {
  const size_t smem = (size_t)kAttnRows * DQK * 2 + 2 * (size_t)kAttnKeys * (DQK + DV) * 2;
  static bool attr_set[128] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 128 && !attr_set[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(attn_kernel<DQK, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const dim3 grid((p.T * p.G + kAttnRows - 1) / kAttnRows, p.nkv, p.splits);
  cudaError_t e = launch_k(attn_kernel<DQK, DV>, grid, dim3(kAttnThreads), smem, st, p);
  if (e != cudaSuccess || p.splits == 1) return e;
  return launch_k(attn_merge_kernel<DV>, dim3(p.T * p.nq), dim3(DV), 0, st, p);
}

}  // namespace

bool attn_dims_supported(int dqk, int dv) {
  return (dqk == 192 && dv == 128) || (dqk == 128 && dv == 128) || (dqk == 64 && dv == 64);
}

// The tcgen05 kernel (attn_tc.cu) takes query tiles of 128 rows without a key split (prefill, chunked
// prefill); MIMO_MOE_ATTN=mma keeps every call on the mma.sync kernel (a comparison knob).
static bool attn_tc_enabled() {
  static const int on = [] {
    const char* v = std::getenv("MIMO_MOE_ATTN");
    return (v && std::strcmp(v, "mma") == 0) ? 0 : 1;
  }();
  return on != 0;
}

int attn_auto_splits(const AttnParams& p, int num_sms) {
  const bool tc = attn_tc_enabled() && attn_tc_supported(p);
  const int rows_tile = tc ? 128 : kAttnRows, keys_block = tc ? 128 : kAttnKeys;
  const int tiles = (p.T * p.G + rows_tile - 1) / rows_tile;
  const int last = p.pos0 + p.T - 1;
  const int first = p.window > 0 ? std::max(0, p.pos0 - p.window + 1) : 0;
  const int nblocks = (last - (tc ? (first & ~127) : first)) / keys_block + 1;
  // tcgen05: about one CTA per SM, at least two key blocks per split (fewer partials to merge);
  // mma.sync: two CTAs per SM
  const int want = tc ? (num_sms + tiles * p.nkv - 1) / (tiles * p.nkv)
                      : (2 * num_sms + tiles * p.nkv - 1) / (tiles * p.nkv);
  const int most = tc ? std::max(1, nblocks / 2) : nblocks;
  return std::max(1, std::min({want, most, 64}));
}

cudaError_t launch_attention(const AttnParams& p, cudaStream_t st) {
  if (attn_tc_enabled() && attn_tc_supported(p)) {
    const cudaError_t e = launch_attention_tc(p, p.status, st);
    if (e != cudaSuccess || p.splits == 1) return e;
    if (p.dv == 128) return launch_k(attn_merge_kernel<128>, dim3(p.T * p.nq), dim3(128), 0, st, p);
    return launch_k(attn_merge_kernel<64>, dim3(p.T * p.nq), dim3(64), 0, st, p);
  }
  if (p.dqk == 192 && p.dv == 128) return launch_attn_t<192, 128>(p, st);
  if (p.dqk == 128 && p.dv == 128) return launch_attn_t<128, 128>(p, st);
  if (p.dqk == 64 && p.dv == 64) return launch_attn_t<64, 64>(p, st);
  return cudaErrorInvalidValue;
}

cudaError_t launch_rope_store(const RopeParams& p, cudaStream_t st) {
  if (p.rot > 256) return cudaErrorInvalidValue;
  if (p.T <= 16) {
    const long long warps = (long long)p.T * (p.nq + p.nkv);
    const dim3 grid((unsigned)((warps + kRopeThreads / 32 - 1) / (kRopeThreads / 32)));
    if (p.rot <= 64) return launch_k(rope_store_decode_kernel<1>, grid, dim3(kRopeThreads), 0, st, p);
    if (p.rot <= 128) return launch_k(rope_store_decode_kernel<2>, grid, dim3(kRopeThreads), 0, st, p);
    return launch_k(rope_store_decode_kernel<4>, grid, dim3(kRopeThreads), 0, st, p);
  }
  // one CTA per (token, 16 heads) up to 148 tokens; beyond, up to 4 CTAs per SM walk the tokens, each taking
  // every head of its token
  const int groups = p.T <= 148 ? (p.nq + p.nkv + 15) / 16 : 1;
  return launch_k(rope_store_kernel, dim3(std::min(p.T, 148 * 4), groups), dim3(512), 0, st, p);
}

cudaError_t launch_add_rmsnorm(const uint16_t* x, const uint16_t* d, const uint16_t* weight, int T, int H, float eps,
                               uint16_t* h, uint16_t* r, cudaStream_t st) {
  return launch_k(add_rmsnorm_kernel, dim3(T), dim3(kNormThreads), 0, st, x, d, weight, H, eps, h, r);
}

cudaError_t launch_swiglu(const uint16_t* gu, int T, int I, uint16_t* out, cudaStream_t st) {
  const size_t n8 = (size_t)T * I / 8;
  const int blocks = (int)std::min<size_t>((n8 + 255) / 256, 148 * 8);
  return launch_k(swiglu_kernel, dim3(blocks), dim3(256), 0, st, gu, T, I, out);
}

cudaError_t launch_add(const uint16_t* a, const uint16_t* b, size_t n, uint16_t* out, cudaStream_t st) {
  const size_t n8 = n / 8;
  const int blocks = (int)std::min<size_t>((n8 + 255) / 256, 148 * 8);
  return launch_k(add_kernel, dim3(blocks), dim3(256), 0, st, a, b, n8, out);
}

}  // namespace mimo
