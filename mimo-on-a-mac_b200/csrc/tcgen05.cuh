// tcgen05 (5th-generation tensor core) building blocks for sm_100a: TMEM allocation, fences,
// commits, scale-factor copies, MMAs, TMEM loads and shared-memory matrix descriptors.  Forms follow
// the PTX ISA for tcgen05; descriptor bit positions are documented next to each builder.
#pragma once
#include "common.cuh"

namespace mimo {
namespace tc {

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}
// Arrives on `bar` once every tcgen05 operation this thread issued before has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;\n" ::"r"(taddr), "l"(sdesc) : "memory");
}
__device__ __forceinline__ void tc_mma_mx(uint32_t d_taddr, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t sfa_taddr, uint32_t sfb_taddr, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n}\n" ::"r"(
          d_taddr),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_taddr), "r"(sfb_taddr)
      : "memory");
}
// ---- CTA pairs (cta_group::2): a cluster of two CTAs whose tensor cores run one M = 256 MMA together.
// Both CTAs allocate (the same warp in each) and free; CTA 0 (the leader) issues the copies, MMAs and
// commits, which act on both CTAs' shared memory and TMEM at the same addresses.
__device__ __forceinline__ void tmem_alloc2(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}
// Arrives on the barrier at cluster address `bar` (this CTA's or the peer's) once the pair's tcgen05
// operations this thread issued before have completed.
__device__ __forceinline__ void tc_commit2(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
               : "memory");
}
// Scale-factor copy in both CTAs: each CTA's 512-byte block at `sdesc` into its own TMEM columns.
__device__ __forceinline__ void tc_cp_sf2(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;\n" ::"r"(taddr), "l"(sdesc) : "memory");
}
// M = 256 block-scaled MMA over the pair: each CTA's 128 A rows x all N columns (half of B from each
// CTA's shared memory) into its own TMEM.
__device__ __forceinline__ void tc_mma_mx2(uint32_t d_taddr, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t sfa_taddr, uint32_t sfb_taddr, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n}\n" ::"r"(
          d_taddr),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_taddr), "r"(sfb_taddr)
      : "memory");
}
template <int NC>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float (&v)[NC]);
template <>
__device__ __forceinline__ void tmem_ld<1>(uint32_t taddr, float (&v)[1]) {
  uint32_t r;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];\n" : "=r"(r) : "r"(taddr));
  v[0] = __uint_as_float(r);
}
template <>
__device__ __forceinline__ void tmem_ld<4>(uint32_t taddr, float (&v)[4]) {
  uint32_t r[4];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}
template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
      "[%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ uint64_t l2_evict_normal_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;\n" : "=l"(pol));
  return pol;
}

// Shared-memory matrix descriptors (sm_100 format: version 1 in bits 46-47).
//   K-major, 128B swizzle: 128-byte rows, 8-row groups 1024 B apart (stride byte offset); the
//   leading byte offset is unused for this layout.  Tiles start 1024-byte aligned (base offset 0).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
//   K-major, no swizzle: 8-row core matrices of 16-byte rows, 128 B apart (the scale blocks).
__device__ __forceinline__ uint64_t desc_sf(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(128 >> 4) << 16;
  d |= (uint64_t)(128 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}
//   K-major, 64B swizzle: 8-row groups of 64-byte rows (packed e2m1, 128 values per row), SBO = 512.
__device__ __forceinline__ uint64_t desc_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(512 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)4 << 61;
  return d;
}
// kind::mxf4 block-scaled MMA: A and B packed e2m1 (2 values per byte, low nibble first), one ue8m0
// scale per 32 values (scale_vec::2X: an MMA of K = 64 reads 2 scale bytes of each row's 32-bit TMEM
// cell, the pair picked by sf id 0 or 2).
__device__ __forceinline__ void tc_mma_mxf4(uint32_t d_taddr, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t sfa_taddr, uint32_t sfb_taddr, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.scale_vec::2X [%0], %1, %2, %3, [%5], [%6], p;\n}\n" ::"r"(
          d_taddr),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_taddr), "r"(sfb_taddr)
      : "memory");
}
// Instruction descriptor of kind::mxf4.block_scale: A and B e2m1 (format 1), ue8m0 scales (bit 23),
// both K-major, M = m, N = n, dense K = 64; sf id (0 or 2) for both operands at bits 4-5 and 29-30.
__device__ __forceinline__ uint32_t idesc_mxf4(int m, int n, uint32_t sfid) {
  return ((sfid & 3u) << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | (1u << 23) |
         ((uint32_t)(m >> 4) << 24) | ((sfid & 3u) << 29);
}

// kind::f16 MMA (bf16/f16 operands from shared memory, f32 accumulate), no disabled lanes.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_taddr, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_taddr),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
// Instruction descriptor of kind::f16: f32 accumulator (bits 4-5 = 1), A and B bf16 (bits 7-9 and
// 10-12 = 1), both K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28.
__device__ __forceinline__ uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// e4m3 two-term split helpers.
__device__ __forceinline__ uint32_t f32_to_e4m3(float v) {  // RNE, saturating
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;\n" : "=h"(r) : "f"(0.f), "f"(v));
  return (uint32_t)r & 0xFFu;
}
__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {  // exact (every e4m3 value is an f16)
  uint32_t h2;
  const uint16_t in = (uint16_t)b;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;\n" : "=r"(h2) : "h"(in));
  return __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFFu)));
}
// Two values at once: byte 0 = e4m3(lo), byte 1 = e4m3(hi) (RNE, saturating), and back (exact).
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;\n" : "=h"(r) : "f"(hi), "f"(lo));
  return (uint32_t)r;
}
__device__ __forceinline__ float2 e4m3x2_to_f32x2(uint32_t b2) {
  uint32_t h2;
  const uint16_t in = (uint16_t)b2;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;\n" : "=r"(h2) : "h"(in));
  return make_float2(__half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFFu))),
                     __half2float(__ushort_as_half((unsigned short)(h2 >> 16))));
}
// ue8m0 byte of a block whose largest magnitude is amax: 2^(e(amax) - 7), so |v| / s < 256 <= 448.
__device__ __forceinline__ uint32_t block_scale_byte(float amax) {
  if (!(amax > 0.f)) return 127u;
  const int e = (int)((__float_as_uint(amax) >> 23) & 0xFFu);
  const int b = e - 7;
  return (uint32_t)(b < 1 ? 1 : (b > 254 ? 254 : b));
}
__device__ __forceinline__ float exp2_byte(uint32_t b) { return __uint_as_float(b << 23); }  // 2^(b - 127)
__device__ __forceinline__ float inv_exp2_byte(uint32_t b) {                                  // 2^(127 - b)
  return __uint_as_float((254u - b) << 23);
}
// Splits 32 bf16 values (64 bytes at src, 16-byte aligned) into two e4m3 terms with one ue8m0 scale
// each: hi = e4m3(v / s1) with s1 = 2^(e(max|v|) - 7), lo = e4m3((v - hi * s1) / s2) with s2 from the
// residual's maximum.  Non-finite inputs set MIMO_ERANGE.
__device__ __forceinline__ void split_block32(const uint16_t* src, uint8_t* dh, uint8_t* dl, uint8_t* sh,
                                              uint8_t* sl, int32_t* status) {
  float v[32];
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 w = s4[i];
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[i * 8 + 2 * j] = __uint_as_float(ww[j] << 16);
      v[i * 8 + 2 * j + 1] = __uint_as_float(ww[j] & 0xFFFF0000u);
    }
  }
  float amax = 0.f;
  bool bad = false;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    amax = fmaxf(amax, fabsf(v[i]));
    bad |= !isfinite(v[i]);
  }
  if (bad) set_status(status, MIMO_ERANGE);
  const uint32_t b1 = block_scale_byte(amax);
  uint32_t hw[8] = {0, 0, 0, 0, 0, 0, 0, 0}, lw[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float r[32], rmax = 0.f;
  // Pairs of values per conversion (e4m3x2 / f16x2 forms): the same per-element roundings as one at a time.
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    const uint32_t e2 = f32x2_to_e4m3x2(v[i] * inv_exp2_byte(b1), v[i + 1] * inv_exp2_byte(b1));
    const float2 q = e4m3x2_to_f32x2(e2);
    r[i] = v[i] - q.x * exp2_byte(b1);
    r[i + 1] = v[i + 1] - q.y * exp2_byte(b1);
    rmax = fmaxf(rmax, fmaxf(fabsf(r[i]), fabsf(r[i + 1])));
    hw[i >> 2] |= e2 << (8 * (i & 3));
  }
  const uint32_t b2 = block_scale_byte(rmax);
#pragma unroll
  for (int i = 0; i < 32; i += 2)
    lw[i >> 2] |= f32x2_to_e4m3x2(r[i] * inv_exp2_byte(b2), r[i + 1] * inv_exp2_byte(b2)) << (8 * (i & 3));
  uint4* h4 = reinterpret_cast<uint4*>(dh);
  uint4* l4 = reinterpret_cast<uint4*>(dl);
  h4[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
  h4[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
  l4[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  l4[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
  *sh = (uint8_t)b1;
  *sl = (uint8_t)b2;
}

// split_block32 with one warp per block (lane = value): the same bytes (the maxima ignore NaN, as
// fmaxf does; every conversion is per element), in a few dependent steps instead of 32 serial values.
__device__ __forceinline__ void split_block32_warp(const uint16_t* src, uint8_t* dh, uint8_t* dl, uint8_t* sh,
                                                   uint8_t* sl, int32_t* status) {
  const int lane = threadIdx.x & 31;
  const float v = __uint_as_float((uint32_t)src[lane] << 16);
  if (__any_sync(0xFFFFFFFFu, !isfinite(v)) && lane == 0) set_status(status, MIMO_ERANGE);
  const float amax = __uint_as_float(__reduce_max_sync(0xFFFFFFFFu, isnan(v) ? 0u : __float_as_uint(fabsf(v))));
  const uint32_t b1 = block_scale_byte(amax);
  const uint32_t h = f32_to_e4m3(v * inv_exp2_byte(b1));
  const float r = v - e4m3_to_f32(h) * exp2_byte(b1);
  const float rmax = __uint_as_float(__reduce_max_sync(0xFFFFFFFFu, isnan(r) ? 0u : __float_as_uint(fabsf(r))));
  const uint32_t b2 = block_scale_byte(rmax);
  dh[lane] = (uint8_t)h;
  dl[lane] = (uint8_t)f32_to_e4m3(r * inv_exp2_byte(b2));
  if (lane == 0) {
    *sh = (uint8_t)b1;
    *sl = (uint8_t)b2;
  }
}

// ------------------------------------------------------------------ e2m1 multi-term activations
// A value block of 32 becomes kFp4Terms e2m1 terms, each with one ue8m0 scale: term t quantises the
// residual r_t (r_0 = v) with the scale s_t that puts max |r_t| / s_t in (3, 6], and
// r_{t+1} = r_t - q_t * s_t.  Each subtraction is exact (q_t * s_t is 0 or within a factor of 2 of
// r_t), and |r_{t+1}| <= s_t (half the widest e2m1 step), so the block's residual maximum falls at
// least 4x per term; on bf16 activations five terms leave dot products within ~1e-6 of exact.
constexpr int kFp4Terms = 5;
// Two floats -> one byte of two e2m1 codes (lo in bits 0-3), round to nearest even, saturating at 6.
__device__ __forceinline__ uint32_t f32x2_to_e2m1x2(float lo, float hi) {
  uint32_t r;
  asm("{\n.reg .b8 b0;\ncvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\nmov.b32 %0, {b0, b0, b0, b0};\n}\n"
      : "=r"(r)
      : "f"(lo), "f"(hi));
  return r & 0xFFu;
}
// One byte of two e2m1 codes -> their values (exact).
__device__ __forceinline__ float2 e2m1x2_to_f32x2(uint32_t byte) {
  uint32_t h2;
  asm("{\n.reg .b8 b0, b1, b2, b3;\nmov.b32 {b0, b1, b2, b3}, %1;\ncvt.rn.f16x2.e2m1x2 %0, b0;\n}\n"
      : "=r"(h2)
      : "r"(byte));
  return __half22float2(*reinterpret_cast<__half2*>(&h2));
}
// ue8m0 byte of the scale 2^e with the smallest e such that amax <= 6 * 2^e.
__device__ __forceinline__ uint32_t e2m1_scale_byte(float amax) {
  if (!(amax > 0.f)) return 127u;
  const uint32_t u = __float_as_uint(amax);
  const int b = (int)((u >> 23) & 0xFFu) - 2 + ((u & 0x7FFFFFu) > 0x400000u ? 1 : 0);
  return (uint32_t)(b < 1 ? 1 : (b > 254 ? 254 : b));
}
// Splits 32 bf16 values (src, 16-byte aligned) into kFp4Terms e2m1 terms: term t's 16 bytes go to
// dq + t * tstride, its scale byte to ds[t * sstride].  Non-finite inputs set MIMO_ERANGE.
__device__ __forceinline__ void split_block32_fp4(const uint16_t* src, uint8_t* dq, size_t tstride, uint8_t* ds,
                                                  size_t sstride, int32_t* status) {
  float v[32];
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 w = s4[i];
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[i * 8 + 2 * j] = __uint_as_float(ww[j] << 16);
      v[i * 8 + 2 * j + 1] = __uint_as_float(ww[j] & 0xFFFF0000u);
    }
  }
  bool bad = false;
#pragma unroll
  for (int i = 0; i < 32; ++i) bad |= !isfinite(v[i]);
  if (bad) set_status(status, MIMO_ERANGE);
#pragma unroll 1
  for (int t = 0; t < kFp4Terms; ++t) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const uint32_t b = e2m1_scale_byte(amax);
    const float inv = inv_exp2_byte(b), sc = exp2_byte(b);
    uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t q = f32x2_to_e2m1x2(v[2 * i] * inv, v[2 * i + 1] * inv);
      const float2 d = e2m1x2_to_f32x2(q);
      v[2 * i] -= d.x * sc;
      v[2 * i + 1] -= d.y * sc;
      w[i >> 2] |= q << (8 * (i & 3));
    }
    *reinterpret_cast<uint4*>(dq + (size_t)t * tstride) = make_uint4(w[0], w[1], w[2], w[3]);
    ds[(size_t)t * sstride] = (uint8_t)b;
  }
}

// Instruction descriptor of kind::mxf8f6f4.block_scale: A e2m1 (5), B e4m3 (0), ue8m0 scales,
// both K-major, M = 128, N = n, dense K = 32; the sf ids pick the byte (K block) of each 32-bit
// TMEM scale cell and equal the top two bits of the scale addresses.
__device__ __forceinline__ uint32_t idesc_mx(int n, uint32_t kb) {
  uint32_t d = 0;
  d |= (kb & 3u) << 4;   // B scale id
  d |= 5u << 7;          // A format E2M1
  d |= 0u << 10;         // B format E4M3
  d |= (uint32_t)(n >> 3) << 17;
  d |= 1u << 23;         // scale format UE8M0
  d |= (uint32_t)(128 >> 4) << 24;  // M = 128
  d |= (kb & 3u) << 29;  // A scale id
  return d;
}

}  // namespace tc
}  // namespace mimo
