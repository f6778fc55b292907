// CPU host for the reference's own MXFP4 expert kernels (TEST INFRASTRUCTURE ONLY).
//
// The reference ships its two expert kernels as Metal Shading Language bodies inside Python strings
// (engine/mimo_stream/kernels.py:19-30 HEADER, :33-85 kernel A, :88-123 kernel B).  oracle/ref_build.py
// extracts those strings at build time into oracle/_ref/*.inc (never committed) and compiles this file
// around them.  This file supplies the Metal vocabulary the bodies use (uint/uint3/uint4, vec<T,N>,
// bfloat16_t, half, as_type, simd_sum, thread_position_in_grid, thread_index_in_simdgroup) in plain
// C++, and runs each 32-lane SIMD-group on one host thread:
//   * bfloat16_t: float -> bf16 round-to-nearest-even, arithmetic in float then rounded (MLX's bf16
//     operator semantics);
//   * simd_sum: the only cross-lane operation in the bodies.  Lanes run one after another in two
//     passes: pass 0 records every lane's k-th simd_sum argument (returning 0), the sums are formed with
//     an xor butterfly (offsets 16, 8, 4, 2, 1), and pass 1 re-runs the lanes with simd_sum returning
//     those sums.  The bodies' control flow before each simd_sum does not depend on earlier sums, so
//     pass 1 reproduces the SIMD-group exactly; the Metal reduction order itself is unspecified
//     ("parity unpinned" at the last float32 ulp);
//   * compiled with -ffp-contract=off: each float multiply and add rounds separately.
// The bf16 sigmoid table the kernels read is passed in by the caller.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#define device
#define thread
#define constant

using uint = uint32_t;
using ushort = uint16_t;
using uchar = uint8_t;
typedef _Float16 half;

template <class T, class S>
inline T as_type(S s) {
  static_assert(sizeof(T) == sizeof(S), "as_type size");
  T t;
  std::memcpy(&t, &s, sizeof t);
  return t;
}

struct bfloat16_t {
  uint16_t bits;
  bfloat16_t() = default;
  bfloat16_t(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) {
      bits = 0x7FC0;
    } else {
      u += 0x7FFFu + ((u >> 16) & 1u);
      bits = (uint16_t)(u >> 16);
    }
  }
  operator float() const {
    const uint32_t u = (uint32_t)bits << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
  }
};
inline bfloat16_t operator*(bfloat16_t a, bfloat16_t b) { return bfloat16_t(float(a) * float(b)); }

struct uint3 {
  uint x, y, z;
};
struct uint4 {
  uint x, y, z, w;
  uint operator[](int i) const { return i == 0 ? x : i == 1 ? y : i == 2 ? z : w; }
};
template <class T, int N>
struct vec {
  T v[N];
  const T& operator[](int i) const { return v[i]; }
  T& operator[](int i) { return v[i]; }
};

// ------------------------------------------------------------------------- SIMD-group emulation
struct SimdCtx {
  int pass = 0, lane = 0, call = 0;
  std::vector<float> rec;   // [call][32]
  std::vector<float> sums;  // [call]
};
static thread_local SimdCtx* g_ctx = nullptr;

inline float simd_sum(float v) {
  SimdCtx& c = *g_ctx;
  const int k = c.call++;
  if (c.pass == 0) {
    if ((int)c.rec.size() < (k + 1) * 32) c.rec.resize((k + 1) * 32, 0.f);
    c.rec[k * 32 + c.lane] = v;
    return 0.f;
  }
  return c.sums[k];
}

static void finish_pass0(SimdCtx& c, int ncalls) {
  c.sums.assign(ncalls, 0.f);
  for (int k = 0; k < ncalls; ++k) {
    float v[32];
    for (int l = 0; l < 32; ++l) v[l] = c.rec[k * 32 + l];
    for (int o = 16; o > 0; o >>= 1) {
      float n[32];
      for (int l = 0; l < 32; ++l) n[l] = v[l] + v[l ^ o];
      std::memcpy(v, n, sizeof v);
    }
    c.sums[k] = v[0];
  }
}

#include "ref_header.inc"

template <int R, int KDIM, int NDIM>
static void mxs_gateup_lane(const bfloat16_t* x, const uint32_t* wg, const uint8_t* sg, const uint32_t* wu,
                            const uint8_t* su, const int32_t* uslot, const int32_t* urows, const int32_t* ucnt,
                            const bfloat16_t* sigtab, bfloat16_t* h, uint3 thread_position_in_grid,
                            uint thread_index_in_simdgroup) {
#include "gateup_body.inc"
}

template <int R, int KDIM, int HDIM>
static void mxs_down_lane(const bfloat16_t* h, const uint32_t* wd, const uint8_t* sd, const int32_t* uslot,
                          const int32_t* ucnt, const float* uw, float* part, uint3 thread_position_in_grid,
                          uint thread_index_in_simdgroup) {
#include "down_body.inc"
}

template <class F>
static void run_simdgroup(F&& lane_fn) {
  SimdCtx c;
  g_ctx = &c;
  c.pass = 0;
  for (int l = 0; l < 32; ++l) {
    c.lane = l;
    c.call = 0;
    lane_fn((uint)l);
  }
  const int ncalls = c.call;
  finish_pass0(c, ncalls);
  c.pass = 1;
  for (int l = 0; l < 32; ++l) {
    c.lane = l;
    c.call = 0;
    lane_fn((uint)l);
  }
  g_ctx = nullptr;
}

template <int R, int K, int N>
static void gateup_grid(const uint16_t* x, const uint32_t* wg, const uint8_t* sg, const uint32_t* wu,
                        const uint8_t* su, const int32_t* uslot, const int32_t* urows, const int32_t* ucnt,
                        const uint16_t* sigtab, uint16_t* h, int U) {
  const long total = (long)U * N;
#pragma omp parallel for schedule(dynamic, 16)
  for (long i = 0; i < total; ++i) {
    const uint u = (uint)(i / N), n = (uint)(i % N);
    run_simdgroup([&](uint lane) {
      mxs_gateup_lane<R, K, N>(reinterpret_cast<const bfloat16_t*>(x), wg, sg, wu, su, uslot, urows, ucnt,
                               reinterpret_cast<const bfloat16_t*>(sigtab), reinterpret_cast<bfloat16_t*>(h),
                               uint3{lane, n, u}, lane);
    });
  }
}

template <int R, int K, int H>
static void down_grid(const uint16_t* h, const uint32_t* wd, const uint8_t* sd, const int32_t* uslot,
                      const int32_t* ucnt, const float* uw, float* part, int U) {
  const long total = (long)U * H;
#pragma omp parallel for schedule(dynamic, 16)
  for (long i = 0; i < total; ++i) {
    const uint u = (uint)(i / H), m = (uint)(i % H);
    run_simdgroup([&](uint lane) {
      mxs_down_lane<R, K, H>(reinterpret_cast<const bfloat16_t*>(h), wd, sd, uslot, ucnt, uw, part,
                             uint3{lane, m, u}, lane);
    });
  }
}

extern "C" {

// Kernel A over grid (32, N, U) with K = hidden, N = intermediate; h is [U, R, N] bf16 bits.
// Supported (R, K, N): (8, 4096, 2048), (8, 512, 256).  Returns 0, or -1 for unsupported sizes.
int ref_gateup(int R, int K, int N, const uint16_t* x, const uint32_t* wg, const uint8_t* sg, const uint32_t* wu,
               const uint8_t* su, const int32_t* uslot, const int32_t* urows, const int32_t* ucnt,
               const uint16_t* sigtab, int U, uint16_t* h) {
  if (R == 8 && K == 4096 && N == 2048)
    gateup_grid<8, 4096, 2048>(x, wg, sg, wu, su, uslot, urows, ucnt, sigtab, h, U);
  else if (R == 8 && K == 512 && N == 256)
    gateup_grid<8, 512, 256>(x, wg, sg, wu, su, uslot, urows, ucnt, sigtab, h, U);
  else
    return -1;
  return 0;
}

// Kernel B over grid (32, H, U) with K = intermediate; part is [U, R, H] float32.
int ref_down(int R, int K, int H, const uint16_t* h, const uint32_t* wd, const uint8_t* sd, const int32_t* uslot,
             const int32_t* ucnt, const float* uw, int U, float* part) {
  if (R == 8 && K == 2048 && H == 4096)
    down_grid<8, 2048, 4096>(h, wd, sd, uslot, ucnt, uw, part, U);
  else if (R == 8 && K == 256 && H == 512)
    down_grid<8, 256, 512>(h, wd, sd, uslot, ucnt, uw, part, U);
  else
    return -1;
  return 0;
}

}  // extern "C"
