// C ABI of the MoE block (include/mimo_moe.h): argument checks, workspace carving, launches.
// No allocation, no host synchronisation, no device selection: everything is stream-ordered.
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/mimo_moe_layer.h"
#include "common.cuh"
#include "kernels.h"

using namespace mimo;

namespace {

thread_local int g_last_cuda_error = 0;

int cuda_fail(cudaError_t e) {
  g_last_cuda_error = (int)e;
  return MIMO_ECUDA;
}
#define MIMO_TRY(expr)                           \
  do {                                           \
    const cudaError_t _e = (expr);               \
    if (_e != cudaSuccess) return cuda_fail(_e); \
  } while (0)

int num_sms_current() {
  static int cache[128] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// ----------------------------------------------------------------- optional launch profiling
struct ProfRec {
  int kind;
  cudaEvent_t a, b;
};
std::mutex g_prof_mu;
std::vector<ProfRec> g_prof_pool;  // created once, reused
size_t g_prof_used = 0;
int g_prof_cap = 0;

// Runs `launch` between an event pair of the profiling pool when profiling is enabled.
template <class F>
cudaError_t profiled(int kind, cudaStream_t st, F&& launch) {
  ProfRec* rec = nullptr;
  if (g_prof_cap > 0) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    if (g_prof_used < (size_t)g_prof_cap && g_prof_used < g_prof_pool.size()) rec = &g_prof_pool[g_prof_used++];
  }
  if (rec) {
    rec->kind = kind;
    cudaEventRecord(rec->a, st);
  }
  const cudaError_t e = launch();
  if (rec) cudaEventRecord(rec->b, st);
  return e;
}

cudaError_t tiles(const ExpertParams& p, int kind, int sms, cudaStream_t st) {
  return profiled(kind, st, [&] { return launch_expert_tiles(p, kind, sms, st); });
}

// Bump allocator over the caller's workspace; with base == nullptr it only measures.
struct Carver {
  uint8_t* base;
  size_t off = 0;
  explicit Carver(void* b) : base(static_cast<uint8_t*>(b)) {}
  template <class T>
  T* take(size_t n) {
    off = (off + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += n * sizeof(T);
    return p;
  }
};

bool dims_ok(int H, int I) { return H > 0 && I > 0 && H % 2048 == 0 && I % 2048 == 0; }

bool pools_ok(const mimo_moe_pools* p) {
  return p && p->gate_w && p->gate_s && p->up_w && p->up_s && p->down_w && p->down_s &&
         p->num_slots > 0 && dims_ok(p->hidden, p->inter);
}

// ------------------------------------------------------------------- workspace layouts
// Term matrices of the tcgen05 path: per unit 2 * routes rows of e4m3 terms + ue8m0 block scales.
bool decode_fp4();

struct TermWs {
  uint8_t *bq, *bs, *hq, *hs;
  int32_t* ready;   // fused decodes: per-unit count of gate/up epilogue warps done, then (decode units)
                    // the stream-K hand-off flags; `nzero` words from `ready` on are zeroed per call
  int nzero;
  float *skg, *skd;  // stream-K decode: contributed gate/up and down group partials
  int32_t *flag_g, *flag_d;
  int32_t* done;     // decode: down tiles completed per output row tile (combine in the down kernel)
  int ctas;          // CTAs the stream-K scratch is sized for
};
// Activation terms of `units` units: e4m3 (2 terms, one byte a value) or, for decode units on the
// kind::mxf4 path, e2m1 (5 terms, half a byte a value).  Decode units also get the stream-K scratch.
TermWs carve_terms(Carver& c, int units, int routes, int H, int I) {
  const bool decode = routes == kTcDecodeRoutes;
  const bool fp4 = decode && decode_fp4();
  const size_t rows = (size_t)units * (fp4 ? kTcFp4Terms : 2) * routes;
  const int vb = fp4 ? 2 : 1;  // values per byte
  TermWs t;
  t.bq = c.take<uint8_t>(rows * H / vb);
  t.bs = c.take<uint8_t>(rows * (H / 32));
  t.hq = c.take<uint8_t>(rows * I / vb);
  t.hs = c.take<uint8_t>(rows * (I / 32));
  t.ctas = num_sms_current();
  const size_t nfg = decode ? sk_flag_count(t.ctas) : 0, nfd = nfg, ndone = decode ? (size_t)H / 128 : 0;
  t.ready = c.take<int32_t>((size_t)units + nfg + nfd + ndone);
  t.nzero = units + (int)(nfg + nfd + ndone);
  t.flag_g = decode ? t.ready + units : nullptr;
  t.flag_d = decode ? t.ready + units + nfg : nullptr;
  t.done = decode ? t.ready + units + nfg + nfd : nullptr;
  t.skg = decode ? c.take<float>(sk_part_g_floats(t.ctas)) : nullptr;
  t.skd = decode ? c.take<float>(sk_part_d_floats(t.ctas)) : nullptr;
  return t;
}

struct DecodeWs {
  __half* x16;
  __half* h16;
  float* part;
  TermWs t;
};
DecodeWs carve_decode(Carver& c, int M, int U, int R, int H, int I) {
  DecodeWs w;
  w.x16 = c.take<__half>((size_t)M * H);
  w.h16 = c.take<__half>((size_t)U * R * I);
  w.part = c.take<float>((size_t)U * R * H);
  w.t = carve_terms(c, U, kTcDecodeRoutes, H, I);
  return w;
}

struct PrefillWs {
  __half* x16;
  int32_t *offsets, *order, *inv, *unit_slot, *unit_p0, *unit_cnt, *unit_first, *unit_nsub, *num_units, *rtok;
  float* rw;
  void* dws;
  __half* h16;
  uint16_t* ypair;
  int ucap;
  TermWs t;
};
PrefillWs carve_prefill(Carver& c, int T, int topk, int H, int I, int E) {
  PrefillWs w;
  const int P = T * topk;
  w.ucap = P / std::min(kPrefillUnit, kTcPrefillRoutes) + E;
  w.x16 = c.take<__half>((size_t)T * H);
  w.offsets = c.take<int32_t>(E + 1);
  w.order = c.take<int32_t>(P);
  w.inv = c.take<int32_t>(P);
  w.dws = c.take<uint8_t>(dispatch_workspace_bytes(P, E));
  w.unit_slot = c.take<int32_t>(w.ucap);
  w.unit_p0 = c.take<int32_t>(w.ucap);
  w.unit_cnt = c.take<int32_t>(w.ucap);
  w.unit_first = c.take<int32_t>(w.ucap);
  w.unit_nsub = c.take<int32_t>(w.ucap);
  w.num_units = c.take<int32_t>(1);
  w.rtok = c.take<int32_t>(P);
  w.rw = c.take<float>(P);
  w.h16 = c.take<__half>((size_t)P * I);
  w.ypair = c.take<uint16_t>((size_t)P * H);
  w.t = carve_terms(c, w.ucap, kTcPrefillRoutes, H, I);
  return w;
}

// Expert-parallel per-route products: dispatch tables + units of up to 8 routes + term matrices.
struct RoutesWs {
  int32_t *offsets, *order, *inv, *unit_slot, *unit_p0, *unit_cnt, *num_units, *rtok;
  float* rw;
  void* dws;
  int ucap;
  TermWs t;
};
RoutesWs carve_routes(Carver& c, int P, int H, int I, int S) {
  RoutesWs w;
  w.ucap = P / kTcDecodeRoutes + S;
  w.offsets = c.take<int32_t>(S + 1);
  w.order = c.take<int32_t>(P);
  w.inv = c.take<int32_t>(P);
  w.dws = c.take<uint8_t>(dispatch_workspace_bytes(P, S));
  w.unit_slot = c.take<int32_t>(w.ucap);
  w.unit_p0 = c.take<int32_t>(w.ucap);
  w.unit_cnt = c.take<int32_t>(w.ucap);
  w.num_units = c.take<int32_t>(1);
  w.rtok = c.take<int32_t>(P);
  w.rw = c.take<float>(P);
  w.t = carve_terms(c, w.ucap, kTcDecodeRoutes, H, I);
  return w;
}

struct GroupWs {
  int32_t *uids, *urows, *ucnt, *gidx, *nu;
  float* uw;
  int ucap;
};
GroupWs carve_group(Carver& c, int M, int topk, int R, int E) {
  GroupWs g;
  g.ucap = std::min(E, M * topk);
  g.uids = c.take<int32_t>(g.ucap);
  g.urows = c.take<int32_t>((size_t)g.ucap * R);
  g.ucnt = c.take<int32_t>(g.ucap);
  g.uw = c.take<float>((size_t)g.ucap * R);
  g.gidx = c.take<int32_t>((size_t)M * topk);
  g.nu = c.take<int32_t>(1);
  return g;
}

ExpertParams gateup_params(const mimo_moe_pools* pools, int32_t* status) {
  ExpertParams p{};
  p.w[0] = reinterpret_cast<const uint8_t*>(pools->gate_w);
  p.s[0] = pools->gate_s;
  p.w[1] = reinterpret_cast<const uint8_t*>(pools->up_w);
  p.s[1] = pools->up_s;
  p.S = pools->num_slots;
  p.N = pools->inter;
  p.K = pools->hidden;
  p.tiles = pools->inter / 16;
  p.status = status;
  return p;
}

ExpertParams down_params(const ExpertParams& gu, const mimo_moe_pools* pools) {
  ExpertParams q = gu;
  q.w[0] = reinterpret_cast<const uint8_t*>(pools->down_w);
  q.s[0] = pools->down_s;
  q.w[1] = nullptr;
  q.s[1] = nullptr;
  q.N = pools->hidden;
  q.K = pools->inter;
  q.tiles = pools->hidden / 16;
  q.rtok = nullptr;
  q.bsrc = gu.h_out;
  q.brows = 0;
  q.h_out = nullptr;
  return q;
}

// The tcgen05 block-scaled path needs 32-byte aligned weight pools (TMA 16U4_ALIGN16B rule) and
// 16-byte aligned scale pools (TMA base rule); MIMO_MOE_EXPERT_PATH=cuda-core selects the mma.sync kernels instead
// (a comparison knob: both are complete CUDA implementations of the same products).
bool tc_path(const mimo_moe_pools* pools) {
  static const bool forced_off = [] {
    const char* e = getenv("MIMO_MOE_EXPERT_PATH");
    return e && std::string(e) == "cuda-core";
  }();
  auto al = [](const void* q, uintptr_t a) { return ((uintptr_t)q & (a - 1)) == 0; };
  return !forced_off && al(pools->gate_w, 32) && al(pools->up_w, 32) && al(pools->down_w, 32) &&
         al(pools->gate_s, 16) && al(pools->up_s, 16) && al(pools->down_s, 16);
}

// Decode expert kernels (MIMO_MOE_DECODE_KERNEL, a comparison knob; all measured on B200):
//   e4m3 (default)  two launches (gate/up, then down) over whole 128-row tiles dealt round-robin,
//                   kind::mxf8f6f4 with two e4m3 activation terms;
//   sk              one launch, stream-K: every CTA streams an equal share of 512-value K groups of the
//                   gate/up tiles, then of the down tiles; group partials folded in a fixed order
//                   (results independent of the split) and the combine fused; balanced, but its shared
//                   ring holds 5 stages (the gate/up kernel's holds 6) and it measured 18-24% slower;
//   e4m3-fused      the e4m3 arithmetic in one launch (bit-identical to e4m3), down tiles waiting on
//                   per-unit counters;
//   fp4             one launch, kind::mxf4: packed weights, five e2m1 activation terms.
enum DecodeKernel { kDecodeE4m3 = 0, kDecodeE4m3Fused = 1, kDecodeFp4 = 2, kDecodeSk = 3 };
int decode_kernel() {
  static const int mode = [] {
    const char* e = getenv("MIMO_MOE_DECODE_KERNEL");
    const std::string v = e ? e : "";
    return v == "fp4" ? kDecodeFp4 : v == "e4m3-fused" ? kDecodeE4m3Fused : v == "sk" ? kDecodeSk : kDecodeE4m3;
  }();
  return mode;
}
bool decode_fp4() { return decode_kernel() == kDecodeFp4; }

// Prefill expert kernels (MIMO_MOE_PREFILL_KERNEL, a comparison knob): "pair" runs each pass on SM
// pairs with M = 256 tcgen05.mma.cta_group::2; "single" (default) on one SM per 128-row tile.
bool prefill_pair() {
  static const bool on = [] {
    const char* e = getenv("MIMO_MOE_PREFILL_KERNEL");
    return e && std::string(e) == "pair";
  }();
  return on;
}


// Down kernel items, decode and prefill alike (MIMO_MOE_DOWN, a comparison knob): "pairs" (default)
// takes two 128-row tiles per item with one K chunk per stage (slot m = row tile m, the gate/up
// kernel's shape); "tiles" one 128-row tile per item with two K chunks per stage (the two slots hold
// the K halves, added in the epilogue).  The two differ in float32 summation order (within 1e-2 of
// each other); decode and prefill must use the same form, because expert-parallel and single-GPU
// paths compute a route's product through either.  Measured on B200 (graph-replayed decode steps):
// B = 8 161.2 against 163.2 us, B = 1 45.0 against 45.9; the forced-overlap B = 8 case (~22 units,
// half as many items to deal) 85.4 against 84.6.  Prefill: the paired form runs four 48 KiB stages
// where the one-tile form runs three of 64 KiB.
bool down_pairs() {
  static const bool on = [] {
    const char* e = getenv("MIMO_MOE_DOWN");
    return !(e && std::string(e) == "tiles");
  }();
  return on;
}

// Decode down launch waiting per unit for the gate/up launch's h instead of for the whole gate/up grid
// (MIMO_MOE_EARLY_DOWN=0 turns it off, a comparison knob; the outputs are the same either way): down
// items of units whose gate/up tiles are done run on the SMs the gate/up launch has already left.
bool early_down() {
  static const bool on = [] {
    const char* e = getenv("MIMO_MOE_EARLY_DOWN");
    return !(e && std::string(e) == "0");
  }();
  return on;
}

// Decode combine placement (MIMO_MOE_DECODE_COMBINE, a comparison knob; bit-identical outputs):
//   separate (default)  its own launch, M x H/1024 CTAs;
//   down                in the down kernel's epilogue, by the CTA completing each output row tile.  One
//                       launch fewer, but every tile pays a fence and three epilogue barriers and the
//                       last tiles' sums run serially at the end: on B200, B = 8 decode 181 us against
//                       167 us, B = 1 48.0 against 47.0.
bool combine_in_down() {
  static const bool on = [] {
    const char* e = getenv("MIMO_MOE_DECODE_COMBINE");
    return e && std::string(e) == "down";
  }();
  return on;
}

// The decode combine (kernels.py:194-199) of mimo_moe_experts, fused into the decode down kernel (or
// the stream-K expert kernel).
struct CombineArgs {
  uint16_t* y;
  const int32_t *gidx, *urows, *ucnt;
  int M, topk;
};

// Gate/up + SwiGLU and down over units of up to `routes` routes, on the tensor cores.
// Decode (routes 8): unit u's routes start at u * R, B rows come from rtok = urows, the down pass
// writes part = dot * weight.  Prefill (routes 32): units from build_units, down writes ypair.
int run_tc(const uint16_t* x, const mimo_moe_pools* pools, int routes, const int32_t* uslot,
           const int32_t* ucnt, const int32_t* up0, int p0_stride, const int32_t* ufirst,
           const int32_t* unsub, const int32_t* rtok, const float* rw,
           const int32_t* num_units, int ucap, int pairs_rounding, const TermWs& t, float* part,
           uint16_t* ypair, int32_t* status, cudaStream_t st, int by_token_rows = 0, bool terms_ready = false,
           bool ready_zeroed = false,
           const int32_t* out_row = nullptr, int x_ld = 0, float* const* peer_part = nullptr, int peer_rows = 0,
           int x_rows = 0, const CombineArgs* comb = nullptr, bool* combined = nullptr) {
  const int H = pools->hidden, I = pools->inter, S = pools->num_slots;
  const int sms = num_sms_current();
  const bool decode = routes == kTcDecodeRoutes;
  const bool fp4 = decode && decode_fp4();
  const int N = (fp4 ? kTcFp4Terms : 2) * routes;  // term rows per unit (MMA N)
  const bool pair = !decode && prefill_pair();     // prefill on SM pairs (256-row tiles)
  // by_token_rows = M > 0: B holds the M (<= 8) token rows once, shared by every unit (decode).
  if (!terms_ready) {
    if (fp4 && by_token_rows) MIMO_TRY(launch_tc_split_tokens_fp4(x, by_token_rows, H, t.bq, t.bs, status, st));
    else if (fp4) MIMO_TRY(launch_tc_split_fp4(x, H, ucnt, up0, p0_stride, rtok, num_units, ucap, t.bq, t.bs, status,
                                               st, x_ld, x_rows));
    else if (by_token_rows) MIMO_TRY(launch_tc_split_tokens(x, by_token_rows, H, t.bq, t.bs, status, st));
    else MIMO_TRY(launch_tc_split(x, H, ucnt, up0, p0_stride, rtok, num_units, ucap, routes, t.bq, t.bs, status, st,
                                  x_ld, x_rows));
  }
  const uint64_t brows = by_token_rows ? (uint64_t)N : (uint64_t)ucap * N;
  TcParams p{};
  if (fp4) {  // packed weights as stored, 64-byte (128-value) boxes
    MIMO_TRY(packed64_map(&p.amap[0], pools->gate_w, (uint64_t)S * I, H / 2, 128));
    MIMO_TRY(packed64_map(&p.amap[1], pools->up_w, (uint64_t)S * I, H / 2, 128));
    MIMO_TRY(packed64_map(&p.bmap, t.bq, brows, H / 2, N));
  } else {
    MIMO_TRY(fp4_weight_map(&p.amap[0], pools->gate_w, (uint64_t)S * I, H));
    MIMO_TRY(fp4_weight_map(&p.amap[1], pools->up_w, (uint64_t)S * I, H));
    MIMO_TRY(rows_map(&p.bmap, t.bq, brows, H, pair ? N / 2 : N));  // pairs: half the term rows per CTA
  }
  MIMO_TRY(sf_map(&p.smap[0], pools->gate_s, (uint64_t)S * I, H / 32, 128));
  MIMO_TRY(sf_map(&p.smap[1], pools->up_s, (uint64_t)S * I, H / 32, 128));
  MIMO_TRY(sf_map(&p.bsmap, t.bs, brows, H / 32, N));
  p.btok = by_token_rows ? rtok : nullptr;
  p.btok_rows = by_token_rows;
  p.S = S;
  p.Nw = I;
  p.K = H;
  p.tiles = I / (pair ? 256 : 128);
  p.unit_slot = uslot;
  p.unit_cnt = ucnt;
  p.unit_p0 = up0;
  p.p0_stride = p0_stride;
  p.unit_first = ufirst;
  p.unit_nsub = unsub;
  p.num_units = num_units;
  p.units_cap = ucap;
  p.weights_once = decode ? 1 : 0;
  p.hq = t.hq;
  p.hs = t.hs;
  p.status = status;
  const bool sk = decode && decode_kernel() == kDecodeSk;
  const bool fused = decode && (decode_kernel() == kDecodeE4m3Fused || decode_kernel() == kDecodeFp4);
  // decode, two launches: the down launch waits per unit for the gate/up epilogue's h (ready counters,
  // zeroed per call: by the route kernel when it made the terms, else here)
  const bool early = decode && !fused && !sk && down_pairs() && early_down();
  if (early) {
    if (!ready_zeroed) MIMO_TRY(cudaMemsetAsync(t.ready, 0, (size_t)ucap * sizeof(int32_t), st));
    p.ready = t.ready;
    p.ready_need = p.tiles * kTcDecodeEpiWarps;
  }
  if (pair) MIMO_TRY(profiled(2, st, [&] { return launch_tc_pair(p, 2, sms, st); }));
  else if (!fused && !sk)
    MIMO_TRY(profiled(decode ? 0 : 2, st, [&] { return launch_tc_experts(p, decode ? 0 : 2, sms, st); }));
  TcParams q = p;  // down: two K chunks per stage (3-D boxes, or two 2-D boxes when packed)
  if (fp4) {
    MIMO_TRY(packed64_map(&q.amap[0], pools->down_w, (uint64_t)S * H, I / 2, 128));
    MIMO_TRY(packed64_map(&q.bmap, t.hq, (uint64_t)ucap * N, I / 2, N));
  } else {
    MIMO_TRY(fp4_weight_map3(&q.amap[0], pools->down_w, (uint64_t)S * H, I, 2));
    MIMO_TRY(rows_map3(&q.bmap, t.hq, (uint64_t)ucap * N, I, pair ? N / 2 : N, 2));
  }
  q.amap[1] = q.amap[0];
  MIMO_TRY(sf_map(&q.smap[0], pools->down_s, (uint64_t)S * H, I / 32, 128));
  q.smap[1] = q.smap[0];
  MIMO_TRY(sf_map(&q.bsmap, t.hs, (uint64_t)ucap * N, I / 32, N));
  q.Nw = H;
  q.K = I;
  q.tiles = H / (pair ? 256 : 128);
  q.btok = nullptr;
  q.hq = nullptr;
  q.hs = nullptr;
  q.rw = rw;
  q.part = part;
  q.out_row = out_row;
  q.peer_part = peer_part;
  q.peer_rows = peer_rows;
  q.ypair = ypair;
  q.pairs_rounding = pairs_rounding;
  if (sk) {  // both passes in one launch, stream-K over K groups
    if (t.ctas != sms) return MIMO_EINVAL;  // workspace carved for another device
    if (!ready_zeroed) MIMO_TRY(cudaMemsetAsync(t.ready, 0, (size_t)t.nzero * sizeof(int32_t), st));
    TcSkParams f{};
    f.gu = p;
    f.dn = q;
    f.ready = t.ready;
    f.part_g = t.skg;
    f.part_d = t.skd;
    f.flag_g = t.flag_g;
    f.flag_d = t.flag_d;
    f.ctas = t.ctas;
    if (comb && part && !peer_part) {  // the combine runs in the expert kernel's epilogue
      f.y = comb->y;
      f.gidx = comb->gidx;
      f.urows = comb->urows;
      f.ucnt = comb->ucnt;
      f.done = t.done;
      f.M = comb->M;
      f.topk = comb->topk;
      f.R = p0_stride;
      if (combined) *combined = true;
    }
    MIMO_TRY(profiled(5, st, [&] { return launch_tc_decode_sk(f, st); }));
    return MIMO_OK;
  }
  if (fused) {  // both passes in one launch; the down tiles wait on per-unit counters
    if (!ready_zeroed) MIMO_TRY(cudaMemsetAsync(t.ready, 0, (size_t)ucap * sizeof(int32_t), st));
    const TcFusedParams f{p, q, t.ready};
    MIMO_TRY(profiled(4, st, [&] { return launch_tc_decode_fused(f, fp4, sms, st); }));
    return MIMO_OK;
  }
  if (!pair && down_pairs()) {
    // two row tiles per item, one K chunk per stage (2-D boxes)
    TcParams r = q;  // (q inherits ready / ready_need from p: set for the early decode down launch)
    MIMO_TRY(fp4_weight_map(&r.amap[0], pools->down_w, (uint64_t)S * H, I));
    r.amap[1] = r.amap[0];
    MIMO_TRY(rows_map(&r.bmap, t.hq, (uint64_t)ucap * N, I, N));
    r.tiles = H / 256;
    MIMO_TRY(profiled(decode ? 1 : 3, st, [&] { return launch_tc_experts(r, decode ? 5 : 6, sms, st); }));
    return MIMO_OK;
  }
  if (decode && comb && part && !peer_part && by_token_rows && combine_in_down()) {
    // the combine runs in the down kernel's epilogue: count the tiles of each output row tile
    if (!ready_zeroed) MIMO_TRY(cudaMemsetAsync(t.done, 0, (size_t)q.tiles * sizeof(int32_t), st));
    q.cy = comb->y;
    q.cgidx = comb->gidx;
    q.curows = comb->urows;
    q.cucnt = comb->ucnt;
    q.cdone = t.done;
    q.cM = comb->M;
    q.ctopk = comb->topk;
    if (combined) *combined = true;
  }
  if (pair) MIMO_TRY(profiled(3, st, [&] { return launch_tc_pair(q, 3, sms, st); }));
  else MIMO_TRY(profiled(decode ? 1 : 3, st, [&] { return launch_tc_experts(q, decode ? 1 : 3, sms, st); }));
  return MIMO_OK;
}

// Decode expert products through the TMA-fed kernels (H <= 4096, I <= 2048).
int run_experts_tma(const mimo_moe_pools* pools, const int32_t* uslot, const int32_t* urows,
                    const int32_t* ucnt, const float* uw, const int32_t* num_unique, int U, int R, int M,
                    int pairs_rounding, const DecodeWs& w, int32_t* status, cudaStream_t st) {
  const int H = pools->hidden, I = pools->inter, S = pools->num_slots;
  const int sms = num_sms_current();
  DecodeParams p{};
  WeightMap wm;
  MIMO_TRY(weight_map(&wm, pools->gate_w, (uint64_t)S * I, H / 2, 8));
  p.wmap[0] = wm.map;
  int per_panel = wm.per_panel;
  MIMO_TRY(weight_map(&wm, pools->up_w, (uint64_t)S * I, H / 2, 8));
  p.wmap[1] = wm.map;
  per_panel |= wm.per_panel;
  MIMO_TRY(scale_map(&p.smap[0], pools->gate_s, (uint64_t)S * I, H / 32, 64));
  MIMO_TRY(scale_map(&p.smap[1], pools->up_s, (uint64_t)S * I, H / 32, 64));
  if (per_panel) {  // keep both maps in the same (2-D) form
    MIMO_TRY(weight_map(&wm, pools->gate_w, (uint64_t)S * I, H / 2, 1));
    p.wmap[0] = wm.map;
    MIMO_TRY(weight_map(&wm, pools->up_w, (uint64_t)S * I, H / 2, 1));
    p.wmap[1] = wm.map;
  }
  p.per_panel = per_panel;
  p.S = S;
  p.N = I;
  p.K = H;
  p.tiles = I / 16;
  p.unit_slot = uslot;
  p.unit_cnt = ucnt;
  p.p0_stride = R;
  p.num_units = num_unique;
  p.units_cap = U;
  p.rtok = urows;
  p.bsrc = w.x16;
  p.brows = M;
  p.h_out = w.h16;
  p.status = status;
  MIMO_TRY(profiled(0, st, [&] { return launch_decode_tma(p, 0, sms, st); }));
  DecodeParams q{};
  MIMO_TRY(weight_map(&wm, pools->down_w, (uint64_t)S * H, I / 2, 8));
  q.wmap[0] = wm.map;
  if (wm.per_panel) {
    MIMO_TRY(weight_map(&wm, pools->down_w, (uint64_t)S * H, I / 2, 1));
    q.wmap[0] = wm.map;
  }
  q.per_panel = wm.per_panel;
  MIMO_TRY(scale_map(&q.smap[0], pools->down_s, (uint64_t)S * H, I / 32, 64));
  q.S = S;
  q.N = H;
  q.K = I;
  q.tiles = H / 16;
  q.unit_slot = uslot;
  q.unit_cnt = ucnt;
  q.p0_stride = R;
  q.num_units = num_unique;
  q.units_cap = U;
  q.rtok = nullptr;
  q.bsrc = w.h16;
  q.rw = uw;
  q.part_out = w.part;
  q.pairs_rounding = pairs_rounding;
  q.status = status;
  MIMO_TRY(profiled(1, st, [&] { return launch_decode_tma(q, 1, sms, st); }));
  return MIMO_OK;
}

int run_experts(const uint16_t* x, const mimo_moe_pools* pools, const int32_t* uslot,
                const int32_t* urows, const int32_t* ucnt, const float* uw, const int32_t* num_unique,
                int U, int R, const int32_t* gidx, int topk, int M, int pairs_rounding, uint16_t* y,
                const DecodeWs& w, int32_t* status, cudaStream_t st, bool x16_ready = false,
                bool terms_ready = false) {
  const int H = pools->hidden;
  const int sms = num_sms_current();
  if (R <= kTcDecodeRoutes && tc_path(pools)) {
    const CombineArgs comb{y, gidx, urows, ucnt, M, topk};
    bool combined = false;
    const int rc = run_tc(x, pools, kTcDecodeRoutes, uslot, ucnt, nullptr, R, nullptr, nullptr, urows, uw,
                          num_unique, U, pairs_rounding, w.t, w.part, nullptr, status, st,
                          M <= kTcDecodeRoutes ? M : 0, terms_ready && M <= kTcDecodeRoutes,
                          /*ready_zeroed=*/terms_ready, nullptr, 0, nullptr, 0, /*x_rows=*/M, &comb, &combined);
    if (rc != MIMO_OK) return rc;
    if (!combined)
      MIMO_TRY(profiled(7, st, [&] {
        return launch_combine_decode(w.part, gidx, urows, ucnt, num_unique, U, R, M, topk, H, y, status, st);
      }));
    return MIMO_OK;
  }
  if (!x16_ready) MIMO_TRY(launch_to_f16(x, w.x16, (size_t)M * H, status, st));
  if (pools->hidden <= 4096 && pools->inter <= 2048) {
    const int rc = run_experts_tma(pools, uslot, urows, ucnt, uw, num_unique, U, R, M, pairs_rounding, w, status, st);
    if (rc != MIMO_OK) return rc;
    MIMO_TRY(profiled(7, st, [&] {
      return launch_combine_decode(w.part, gidx, urows, ucnt, num_unique, U, R, M, topk, H, y, status, st);
    }));
    return MIMO_OK;
  }
  ExpertParams p = gateup_params(pools, status);
  p.unit_slot = uslot;
  p.unit_p0 = nullptr;
  p.p0_stride = R;
  p.unit_cnt = ucnt;
  p.num_units = num_unique;
  p.units_cap = U;
  p.rtok = urows;
  p.bsrc = w.x16;
  p.brows = M;
  p.h_out = w.h16;
  MIMO_TRY(tiles(p, 0, sms, st));
  ExpertParams q = down_params(p, pools);
  q.rw = uw;
  q.part_out = w.part;
  q.pairs_rounding = pairs_rounding;
  MIMO_TRY(tiles(q, 1, sms, st));
  MIMO_TRY(profiled(7, st, [&] {
    return launch_combine_decode(w.part, gidx, urows, ucnt, num_unique, U, R, M, topk, H, y, status, st);
  }));
  return MIMO_OK;
}

// x_rows rows of x (route_row null: x_rows = T and route p reads row p / topk; else row route_row[p],
// with x_rows <= T so the f16 copy fits the workspace); weight null: 1.
int run_prefill(const uint16_t* x, const mimo_moe_pools* pools, const int32_t* slot_of,
                const int32_t* idx, const float* weight, int T, int topk, int E, uint16_t* y,
                const PrefillWs& w, int32_t* status, cudaStream_t st, int x_rows,
                const int32_t* route_row = nullptr) {
  const int H = pools->hidden;
  const int P = T * topk;
  const int sms = num_sms_current();
  if (tc_path(pools)) {
    MIMO_TRY(launch_dispatch(idx, P, E, w.offsets, w.order, w.inv, w.dws, status, st));
    MIMO_TRY(launch_build_units(w.offsets, slot_of, E, pools->num_slots, kTcPrefillRoutes, w.ucap,
                                w.unit_slot, w.unit_p0, w.unit_cnt, w.unit_first, w.unit_nsub, w.num_units,
                                w.order, weight, P, topk, w.rtok, w.rw, status, st, route_row));
    const int rc = run_tc(x, pools, kTcPrefillRoutes, w.unit_slot, w.unit_cnt, w.unit_p0, 0, w.unit_first,
                          w.unit_nsub, w.rtok, nullptr, w.num_units, w.ucap, 0, w.t, nullptr, w.ypair, status, st,
                          0, false, false, nullptr, 0, nullptr, 0, x_rows);
    if (rc != MIMO_OK) return rc;
    MIMO_TRY(launch_combine_prefill(w.ypair, w.inv, weight, T, topk, H, y, st));
    return MIMO_OK;
  }
  MIMO_TRY(launch_to_f16(x, w.x16, (size_t)x_rows * H, status, st));
  MIMO_TRY(launch_dispatch(idx, P, E, w.offsets, w.order, w.inv, w.dws, status, st));
  MIMO_TRY(launch_build_units(w.offsets, slot_of, E, pools->num_slots, kPrefillUnit, w.ucap,
                              w.unit_slot, w.unit_p0, w.unit_cnt, nullptr, nullptr, w.num_units, w.order,
                              weight, P, topk, w.rtok, w.rw, status, st, route_row));
  ExpertParams p = gateup_params(pools, status);
  p.unit_slot = w.unit_slot;
  p.unit_p0 = w.unit_p0;
  p.unit_cnt = w.unit_cnt;
  p.num_units = w.num_units;
  p.units_cap = w.ucap;
  p.rtok = w.rtok;
  p.bsrc = w.x16;
  p.brows = x_rows;
  p.h_out = w.h16;
  MIMO_TRY(tiles(p, 2, sms, st));
  ExpertParams q = down_params(p, pools);
  q.ypair_out = w.ypair;
  MIMO_TRY(tiles(q, 3, sms, st));
  MIMO_TRY(launch_combine_prefill(w.ypair, w.inv, weight, T, topk, H, y, st));
  return MIMO_OK;
}

}  // namespace

extern "C" {

int mimo_moe_version(void) { return MIMO_MOE_VERSION; }

const char* mimo_moe_strerror(int code) {
  switch (code) {
    case MIMO_OK: return "ok";
    case MIMO_EINVAL: return "invalid argument (shape, null pointer or workspace too small)";
    case MIMO_ERANGE: return "value out of range (expert id, rows per expert, or activation beyond f16)";
    case MIMO_ETIMEOUT: return "bounded device wait expired";
    case MIMO_ECUDA: return "CUDA error";
    case MIMO_EIO: return "file open or read failed (or the file is shorter than the spans)";
    default: return "unknown error";
  }
}

int mimo_moe_last_cuda_error(void) { return g_last_cuda_error; }

int mimo_moe_router(const uint16_t* x, const uint16_t* w, const float* bias, int32_t T, int32_t H,
                    int32_t E, int32_t topk, float* logits, int32_t* idx, float* weight, void* stream) {
  if (!x || !w || !logits || !idx || !weight || T < 1 || H < 256 || H % 256 || E < 32 || E > 256 ||
      E % 32 || topk < 1 || topk > 8 || topk > E)
    return MIMO_EINVAL;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  MIMO_TRY(launch_router_logits(x, w, logits, T, H, E, st));
  MIMO_TRY(launch_router_topk(logits, bias, T, E, topk, idx, weight, st));
  return MIMO_OK;
}

int mimo_moe_topk(const float* logits, const float* bias, int32_t T, int32_t E, int32_t topk,
                  int32_t* idx, float* weight, void* stream) {
  if (!logits || !idx || !weight || T < 1 || E < 32 || E > 256 || E % 32 || topk < 1 || topk > 8 ||
      topk > E)
    return MIMO_EINVAL;
  MIMO_TRY(launch_router_topk(logits, bias, T, E, topk, idx, weight, static_cast<cudaStream_t>(stream)));
  return MIMO_OK;
}

int mimo_moe_group_routes(const int32_t* idx, const float* weight, int32_t M, int32_t topk, int32_t R,
                          int32_t E, int32_t* uids, int32_t* urows, int32_t* ucnt, float* uw,
                          int32_t* gather_idx, int32_t* num_unique, int32_t* status, void* stream) {
  if (!idx || !weight || !uids || !urows || !ucnt || !uw || !gather_idx || !num_unique || M < 1 ||
      topk < 1 || R < 1 || E < 1 || E > 1024 || (int64_t)M * topk > 1024)
    return MIMO_EINVAL;
  MIMO_TRY(launch_group_routes(idx, weight, M, topk, R, E, uids, urows, ucnt, uw, gather_idx, num_unique,
                               status, static_cast<cudaStream_t>(stream)));
  return MIMO_OK;
}

size_t mimo_moe_dispatch_workspace_bytes(int32_t T, int32_t topk, int32_t E) {
  if (T < 1 || topk < 1 || E < 1) return 0;
  return dispatch_workspace_bytes(T * topk, E);
}

int mimo_moe_dispatch(const int32_t* idx, int32_t T, int32_t topk, int32_t E, int32_t* offsets,
                      int32_t* order, int32_t* inv, void* workspace, size_t workspace_bytes,
                      int32_t* status, void* stream) {
  if (!idx || !offsets || !order || !inv || !workspace || T < 1 || topk < 1 || E < 1 || E > 1024 ||
      (int64_t)T * topk > (1 << 30))
    return MIMO_EINVAL;
  if (workspace_bytes < dispatch_workspace_bytes(T * topk, E)) return MIMO_EINVAL;
  MIMO_TRY(launch_dispatch(idx, T * topk, E, offsets, order, inv, workspace, status,
                           static_cast<cudaStream_t>(stream)));
  return MIMO_OK;
}

size_t mimo_moe_ep_plan_workspace_bytes(int32_t T, int32_t world) {
  if (T < 1 || world < 1 || world > 8) return 0;
  return ep_plan_workspace_bytes(T, world);
}

int mimo_moe_ep_plan(const int32_t* idx, int32_t T, int32_t topk, int32_t per_rank, int32_t world,
                     int64_t* counts, int32_t* order, int32_t* inv, int32_t* send_tok, int32_t* send_tag,
                     void* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  if (!idx || !counts || !order || !inv || !send_tok || !send_tag || !workspace || T < 1 || topk < 1 ||
      topk > 16 || world < 1 || world > 8 || per_rank < 1 || (int64_t)T * topk > (1 << 30))
    return MIMO_EINVAL;
  if (workspace_bytes < ep_plan_workspace_bytes(T, world)) return MIMO_EINVAL;
  MIMO_TRY(launch_ep_plan(idx, T, topk, per_rank, world, counts, order, inv, send_tok, send_tag, workspace,
                          status, static_cast<cudaStream_t>(stream)));
  return MIMO_OK;
}

int mimo_moe_gather_rows(const uint16_t* x, int64_t x_rows, int32_t H, const int32_t* rows, int64_t n,
                         uint16_t* out, int32_t* status, void* stream) {
  if ((n > 0 && (!x || !rows || !out)) || H < 8 || H % 8 || n < 0 || n > 0x7FFFFFFF || x_rows < 0)
    return MIMO_EINVAL;
  MIMO_TRY(launch_gather_rows(x, x_rows, H, rows, n, out, status, static_cast<cudaStream_t>(stream)));
  return MIMO_OK;
}

int mimo_moe_ep_recv_index(const int32_t* recv_tag, const int64_t* recv_counts, int32_t world, int64_t n_recv,
                           int32_t* route_row, int32_t* eid, int32_t* status, void* stream) {
  if ((n_recv > 0 && (!recv_tag || !recv_counts || !route_row || !eid)) || world < 1 || world > 8 || n_recv < 0 ||
      n_recv > 0x7FFFFFFF)
    return MIMO_EINVAL;
  MIMO_TRY(launch_ep_recv_index(recv_tag, recv_counts, world, n_recv, route_row, eid, status,
                                static_cast<cudaStream_t>(stream)));
  return MIMO_OK;
}

size_t mimo_moe_experts_workspace_bytes(int32_t M, int32_t U, int32_t R, int32_t H, int32_t I) {
  if (M < 1 || U < 1 || R < 1) return 0;
  Carver c(nullptr);
  carve_decode(c, M, U, R, H, I);
  return c.off;
}

int mimo_moe_experts(const uint16_t* x, const mimo_moe_pools* pools, const int32_t* uslot,
                     const int32_t* urows, const int32_t* ucnt, const float* uw,
                     const int32_t* num_unique, int32_t U, int32_t R, const int32_t* gather_idx,
                     int32_t topk, int32_t M, int32_t pairs_rounding, uint16_t* y, void* workspace,
                     size_t workspace_bytes, int32_t* status, void* stream) {
  if (!x || !pools_ok(pools) || !uslot || !urows || !ucnt || !uw || !y || !workspace || U < 1 ||
      R < 1 || R > 8 || M < 1 || M > 128 || (gather_idx && (topk < 1 || topk > 64)))
    return MIMO_EINVAL;
  Carver c(workspace);
  const DecodeWs w = carve_decode(c, M, U, R, pools->hidden, pools->inter);
  if (c.off > workspace_bytes) return MIMO_EINVAL;
  return run_experts(x, pools, uslot, urows, ucnt, uw, num_unique, U, R, gather_idx, topk, M,
                     pairs_rounding, y, w, status, static_cast<cudaStream_t>(stream));
}

size_t mimo_moe_prefill_workspace_bytes(int32_t T, int32_t topk, int32_t H, int32_t I, int32_t E) {
  if (T < 1 || topk < 1 || E < 1) return 0;
  Carver c(nullptr);
  carve_prefill(c, T, topk, H, I, E);
  return c.off;
}

int mimo_moe_prefill(const uint16_t* x, const mimo_moe_pools* pools, const int32_t* slot_of, int32_t E,
                     const int32_t* idx, const float* weight, int32_t T, int32_t topk, uint16_t* y,
                     void* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  if (!x || !pools_ok(pools) || !idx || !weight || !y || !workspace || T < 1 || topk < 1 || topk > 64 ||
      (int64_t)T * topk > (1 << 26) || E < 1 || E > 1024 || (!slot_of && E != pools->num_slots))
    return MIMO_EINVAL;
  Carver c(workspace);
  const PrefillWs w = carve_prefill(c, T, topk, pools->hidden, pools->inter, E);
  if (c.off > workspace_bytes) return MIMO_EINVAL;
  return run_prefill(x, pools, slot_of, idx, weight, T, topk, E, y, w, status,
                     static_cast<cudaStream_t>(stream), T);
}

int mimo_moe_prefill_routes(const uint16_t* x, int32_t x_rows, const mimo_moe_pools* pools,
                            const int32_t* slot_of, int32_t E, const int32_t* route_row, const int32_t* idx,
                            int32_t P, uint16_t* y, void* workspace, size_t workspace_bytes, int32_t* status,
                            void* stream) {
  if (!x || !pools_ok(pools) || !route_row || !idx || !y || !workspace || P < 1 || P > (1 << 26) ||
      x_rows < 1 || x_rows > P || E < 1 || E > 1024 || (!slot_of && E != pools->num_slots))
    return MIMO_EINVAL;
  Carver c(workspace);
  const PrefillWs w = carve_prefill(c, P, 1, pools->hidden, pools->inter, E);
  if (c.off > workspace_bytes) return MIMO_EINVAL;
  return run_prefill(x, pools, slot_of, idx, nullptr, P, 1, E, y, w, status, static_cast<cudaStream_t>(stream),
                     x_rows, route_row);
}

size_t mimo_moe_block_workspace_bytes(int32_t T, int32_t H, int32_t I, int32_t E, int32_t topk) {
  if (T < 1 || topk < 1 || E < 1) return 0;
  Carver c(nullptr);
  c.take<float>((size_t)T * E);
  c.take<int32_t>((size_t)T * topk);
  c.take<float>((size_t)T * topk);
  if (T <= 8) {
    c.take<float>((size_t)T * E);  // router scores
    const GroupWs g = carve_group(c, T, topk, 8, E);
    carve_decode(c, T, g.ucap, 8, H, I);
  } else {
    carve_prefill(c, T, topk, H, I, E);
  }
  return c.off;
}

int mimo_moe_block(const uint16_t* x, const uint16_t* router_w, const float* bias,
                   const mimo_moe_pools* pools, int32_t T, int32_t topk, uint16_t* y, int32_t* idx_out,
                   float* w_out, void* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  if (!x || !router_w || !pools_ok(pools) || !y || !workspace || T < 1 || topk < 1 || topk > 8 ||
      (int64_t)T * topk > (1 << 26))
    return MIMO_EINVAL;
  const int E = pools->num_slots, H = pools->hidden, I = pools->inter;
  if (E < 32 || E > 256 || E % 32 || topk > E) return MIMO_EINVAL;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver c(workspace);
  float* logits = c.take<float>((size_t)T * E);
  int32_t* idx = c.take<int32_t>((size_t)T * topk);
  float* wts = c.take<float>((size_t)T * topk);
  if (idx_out) idx = idx_out;
  if (w_out) wts = w_out;
  if (T <= 8) {
    float* score = c.take<float>((size_t)T * E);  // router scores (sigmoid of the logits)
    const GroupWs g = carve_group(c, T, topk, 8, E);
    const DecodeWs dw = carve_decode(c, T, g.ucap, 8, H, I);
    if (c.off > workspace_bytes) return MIMO_EINVAL;
    // one launch: logits, top-k, grouping and the expert kernels' copy of x (e4m3 terms for the
    // tensor-core path, f16 for the mma.sync path)
    const bool tc = tc_path(pools);
    MIMO_TRY(profiled(6, st, [&] {
      return launch_route_decode(x, router_w, bias, T, H, E, topk, 8, logits, idx, wts, g.uids,
                                 g.urows, g.ucnt, g.uw, g.gidx, g.nu, tc ? nullptr : dw.x16,
                                 tc ? dw.t.bq : nullptr, tc ? dw.t.bs : nullptr, score, status, st,
                                 tc && decode_fp4() ? 1 : 0, tc ? dw.t.ready : nullptr, dw.t.nzero);
    }));
    return run_experts(x, pools, g.uids, g.urows, g.ucnt, g.uw, g.nu, g.ucap, 8, g.gidx, topk, T,
                       T == 1 ? 1 : 0, y, dw, status, st, /*x16_ready=*/!tc, /*terms_ready=*/tc);
  }
  const PrefillWs pw = carve_prefill(c, T, topk, H, I, E);
  if (c.off > workspace_bytes) return MIMO_EINVAL;
  MIMO_TRY(launch_router_logits(x, router_w, logits, T, H, E, st, status));
  MIMO_TRY(launch_router_topk(logits, bias, T, E, topk, idx, wts, st));
  return run_prefill(x, pools, nullptr, idx, wts, T, topk, E, y, pw, status, st, T);
}

size_t mimo_moe_experts_routes_workspace_bytes(int32_t rows, int32_t topk, int32_t H, int32_t I, int32_t S) {
  if (rows < 1 || topk < 1 || S < 1 || !dims_ok(H, I)) return 0;
  Carver c(nullptr);
  carve_routes(c, rows * topk, H, I, S);
  return c.off;
}

int mimo_moe_experts_routes(const uint16_t* x, int32_t x_ld, int32_t rows, const mimo_moe_pools* pools,
                            int32_t expert_base, const int32_t* idx, const float* weight, int32_t route_ld,
                            int32_t topk, int32_t pairs_rounding, float* part, float* const* peer_part,
                            int32_t rows_per_rank, void* workspace, size_t workspace_bytes, int32_t* status,
                            void* stream) {
  if (!x || !pools_ok(pools) || !idx || !weight || !workspace || !status || rows < 1 || topk < 1 ||
      topk > 8 || expert_base < 0 || (int64_t)rows * topk > (1 << 24) || pools->num_slots > 1024 ||
      (!part && !peer_part) || (peer_part && (rows_per_rank < 1 || (rows * topk) % rows_per_rank)))
    return MIMO_EINVAL;
  const int P = rows * topk, S = pools->num_slots, H = pools->hidden, I = pools->inter;
  if (x_ld <= 0) x_ld = H;
  if (route_ld <= 0) route_ld = topk;
  if (x_ld < H || x_ld % 8 || route_ld < topk) return MIMO_EINVAL;
  Carver c(workspace);
  const RoutesWs w = carve_routes(c, P, H, I, S);
  if (c.off > workspace_bytes) return MIMO_EINVAL;
  if (!tc_path(pools)) return MIMO_EINVAL;  // needs the TMA alignment of the tensor-core path
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!peer_part) MIMO_TRY(cudaMemsetAsync(part, 0, (size_t)P * H * sizeof(float), st));
  if (P <= 1024 && S <= 256) {  // decode sizes: one CTA builds the units
    MIMO_TRY(launch_routes_prep(idx, weight, route_ld, rows, topk, expert_base, S, kTcDecodeRoutes, w.ucap, w.order,
                                w.rtok, w.rw, w.unit_slot, w.unit_p0, w.unit_cnt, w.num_units, st));
  } else {
    if (route_ld != topk) return MIMO_EINVAL;  // the general dispatch reads packed routes
    MIMO_TRY(launch_dispatch(idx, P, S, w.offsets, w.order, w.inv, w.dws, status, st, expert_base, 1));
    MIMO_TRY(launch_build_units(w.offsets, nullptr, S, S, kTcDecodeRoutes, w.ucap, w.unit_slot, w.unit_p0,
                                w.unit_cnt, nullptr, nullptr, w.num_units, w.order, weight, P, topk, w.rtok,
                                w.rw, status, st));
  }
  return run_tc(x, pools, kTcDecodeRoutes, w.unit_slot, w.unit_cnt, w.unit_p0, 0, nullptr, nullptr, w.rtok,
                w.rw, w.num_units, w.ucap, pairs_rounding, w.t, part, nullptr, status, st, 0, false, false, w.order,
                x_ld, peer_part, rows_per_rank, /*x_rows=*/rows);
}

// ------------------------------------------------------------------- peer-memory exchange
int mimo_moe_peer_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return MIMO_EINVAL;
  MIMO_TRY(cudaMalloc(ptr, bytes));
  MIMO_TRY(cudaMemset(*ptr, 0, bytes));
  cudaIpcMemHandle_t h;
  MIMO_TRY(cudaIpcGetMemHandle(&h, *ptr));
  std::memcpy(handle, &h, sizeof(h));
  return MIMO_OK;
}

int mimo_moe_peer_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return MIMO_EINVAL;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  MIMO_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return MIMO_OK;
}

int mimo_moe_peer_close(void* ptr) {
  if (!ptr) return MIMO_EINVAL;
  MIMO_TRY(cudaIpcCloseMemHandle(ptr));
  return MIMO_OK;
}

int mimo_moe_peer_free(void* ptr) {
  if (!ptr) return MIMO_EINVAL;
  MIMO_TRY(cudaFree(ptr));
  return MIMO_OK;
}

int mimo_moe_peer_barrier(int32_t* const* signals, int32_t* my_signals, int32_t rank, int32_t world,
                          int32_t* epoch, int32_t timeout_us, int32_t* status, void* stream) {
  if (!signals || !my_signals || !epoch || !status || world < 1 || world > 32 || rank < 0 || rank >= world ||
      timeout_us < 0)
    return MIMO_EINVAL;
  const uint64_t limit_ns = timeout_us ? (uint64_t)timeout_us * 1000ull : 2000000000ull;
  MIMO_TRY(launch_peer_barrier(signals, my_signals, rank, world, epoch, limit_ns, status,
                               static_cast<cudaStream_t>(stream)));
  return MIMO_OK;
}

int mimo_moe_route_scatter(const uint16_t* x, int32_t T, int32_t H, const uint16_t* router_w, const float* bias,
                           int32_t E, int32_t topk, int32_t* const* rows, int32_t ld, int32_t rank, int32_t world,
                           float* logits, void* stream) {
  if (!x || !router_w || !rows || !logits || T < 1 || T > 8 || H < 256 || H % 256 || E < 32 || E > 256 ||
      E % 32 || topk < 1 || topk > 8 || topk > E || world < 1 || world > 16 || rank < 0 || rank >= world ||
      ld < H / 2 + 2 * topk)
    return MIMO_EINVAL;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  MIMO_TRY(launch_router_logits(x, router_w, logits, T, H, E, st));
  MIMO_TRY(launch_route_scatter(x, logits, bias, T, H, E, topk, rows, ld, rank, world, st));
  return MIMO_OK;
}

int mimo_moe_combine(const float* part, int64_t part_rows, const int32_t* gather_idx, int32_t M, int32_t topk,
                     int32_t H, uint16_t* y, int32_t* status, void* stream) {
  if (!part || !y || M < 1 || topk < 1 || topk > 8 || H < 4 || H % 4) return MIMO_EINVAL;
  if (part_rows <= 0) part_rows = (int64_t)M * topk;
  if (!gather_idx && part_rows < (int64_t)M * topk) return MIMO_EINVAL;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  MIMO_TRY(launch_combine_rows(part, gather_idx, M, topk, H, part_rows, y, status, st));
  return MIMO_OK;
}

int mimo_moe_combine_pairs(const uint16_t* ypair, const int32_t* inv, const float* weight, int32_t T, int32_t topk,
                           int32_t H, uint16_t* y, void* stream) {
  if (!ypair || !inv || !weight || !y || T < 1 || topk < 1 || topk > 8 || H < 8 || H % 8) return MIMO_EINVAL;
  MIMO_TRY(launch_combine_prefill(ypair, inv, weight, T, topk, H, y, static_cast<cudaStream_t>(stream)));
  return MIMO_OK;
}

int mimo_moe_rmsnorm(const uint16_t* x, const uint16_t* weight, int32_t T, int32_t H, float eps, uint16_t* y,
                     void* stream) {
  const auto a16 = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  if (!x || !y || T < 1 || H < 8 || H % 8 || !(eps >= 0.f) || !a16(x) || !a16(y) || (weight && !a16(weight)))
    return MIMO_EINVAL;
  MIMO_TRY(launch_rmsnorm(x, weight, T, H, eps, y, static_cast<cudaStream_t>(stream)));
  return MIMO_OK;
}

int mimo_moe_profile_enable(int32_t capacity) {
  if (capacity < 0) return MIMO_EINVAL;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  while (g_prof_pool.size() < (size_t)capacity) {
    ProfRec r{0, nullptr, nullptr};
    MIMO_TRY(cudaEventCreate(&r.a));
    MIMO_TRY(cudaEventCreate(&r.b));
    g_prof_pool.push_back(r);
  }
  g_prof_cap = capacity;
  g_prof_used = 0;
  return MIMO_OK;
}


int mimo_moe_profile_read(int32_t* launches, float* milliseconds) {
  if (!launches || !milliseconds) return MIMO_EINVAL;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  for (int k = 0; k < MIMO_MOE_PROFILE_KINDS; ++k) {
    launches[k] = 0;
    milliseconds[k] = 0.f;
  }
  for (size_t i = 0; i < g_prof_used; ++i) {
    const ProfRec& r = g_prof_pool[i];
    MIMO_TRY(cudaEventSynchronize(r.b));
    float ms = 0.f;
    MIMO_TRY(cudaEventElapsedTime(&ms, r.a, r.b));
    launches[r.kind] += 1;
    milliseconds[r.kind] += ms;
  }
  g_prof_used = 0;
  return MIMO_OK;
}

// ------------------------------------------------------------- decoder layer (include/mimo_moe_layer.h)
namespace {
bool a16(const void* p) { return ((uintptr_t)p & 15) == 0; }
size_t attn_split_bytes(int32_t T, int32_t nq, int32_t dv) { return (size_t)T * nq * ((size_t)dv + 2) * 4; }
}  // namespace

int mimo_moe_layer_rope_store(const uint16_t* qkv, int32_t T, int32_t n_heads, int32_t n_kv_heads,
                              int32_t head_dim, int32_t v_head_dim, int32_t rotary_dim, float rope_theta,
                              float v_scale, int32_t pos0, int32_t cap, uint16_t* q, uint16_t* k_cache,
                              uint16_t* v_cache, void* stream) {
  if (!qkv || !q || !k_cache || !v_cache || T < 1 || n_heads < 1 || n_kv_heads < 1 || head_dim < 8 ||
      v_head_dim < 8 || head_dim % 8 || v_head_dim % 8 || rotary_dim < 0 || rotary_dim % 2 || rotary_dim > head_dim ||
      rotary_dim > 256 ||
      !(rope_theta > 0.f) || !(v_scale >= 0.f) || pos0 < 0 || cap < T || (int64_t)pos0 + T > INT32_MAX ||
      !a16(qkv) || !a16(q) || !a16(k_cache) || !a16(v_cache))
    return MIMO_EINVAL;
  RopeParams p{};
  p.qkv = qkv, p.q = q, p.kc = k_cache, p.vc = v_cache;
  p.T = T, p.nq = n_heads, p.nkv = n_kv_heads, p.dqk = head_dim, p.dv = v_head_dim, p.rot = rotary_dim;
  p.pos0 = pos0, p.cap = cap, p.has_vscale = v_scale > 0.f ? 1 : 0, p.v_scale = v_scale;
  p.log_base = std::log((double)rope_theta);
  MIMO_TRY(launch_rope_store(p, static_cast<cudaStream_t>(stream)));
  return MIMO_OK;
}

size_t mimo_moe_layer_attention_workspace_bytes(int32_t T, int32_t n_heads, int32_t v_head_dim, int32_t splits) {
  if (T < 1 || n_heads < 1 || v_head_dim < 1 || splits <= 1) return 0;
  return (size_t)splits * attn_split_bytes(T, n_heads, v_head_dim);
}

int mimo_moe_layer_attention(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                             const float* sinks, int32_t T, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                             int32_t v_head_dim, float scale, int32_t window, int32_t pos0, int32_t cap,
                             int32_t splits, uint16_t* out, void* workspace, size_t workspace_bytes, int32_t* status,
                             void* stream) {
  if (!q || !k_cache || !v_cache || !out || T < 1 || n_heads < 1 || n_kv_heads < 1 || n_heads % n_kv_heads ||
      !attn_dims_supported(head_dim, v_head_dim) || !(scale > 0.f) || window < 0 || pos0 < 0 || cap < 1 ||
      (int64_t)pos0 + T > INT32_MAX || !a16(q) || !a16(k_cache) || !a16(v_cache) || !a16(out))
    return MIMO_EINVAL;
  const int last = pos0 + T - 1;
  const int first_visible = window > 0 ? std::max(0, pos0 - window + 1) : 0;
  if (last - first_visible + 1 > cap) return MIMO_EINVAL;  // a visible key would have been overwritten
  const int G = n_heads / n_kv_heads;
  const size_t per_split = attn_split_bytes(T, n_heads, v_head_dim);
  AttnParams p{};
  p.T = T, p.nq = n_heads, p.nkv = n_kv_heads, p.G = G, p.dqk = head_dim, p.dv = v_head_dim, p.cap = cap;
  p.window = window, p.pos0 = pos0;
  if (splits <= 0) {
    splits = attn_auto_splits(p, num_sms_current());
    if (splits > 1 && (!workspace || workspace_bytes < (size_t)splits * per_split))
      splits = workspace ? (int)std::min<size_t>(splits, workspace_bytes / per_split) : 1;
    splits = std::max(splits, 1);
  }
  if (splits > 64 || (splits > 1 && (!workspace || !a16(workspace) || workspace_bytes < (size_t)splits * per_split)))
    return MIMO_EINVAL;
  p.q = q, p.k = k_cache, p.v = v_cache, p.sinks = sinks, p.out = out;
  p.part_o = splits > 1 ? static_cast<float*>(workspace) : nullptr;
  p.part_ml = splits > 1 ? static_cast<float*>(workspace) + (size_t)splits * T * n_heads * v_head_dim : nullptr;
  p.T = T, p.nq = n_heads, p.nkv = n_kv_heads, p.G = G, p.dqk = head_dim, p.dv = v_head_dim, p.cap = cap;
  p.window = window, p.pos0 = pos0, p.splits = splits;
  p.scale_log2 = (float)((double)scale * 1.4426950408889634);
  p.status = status;
  MIMO_TRY(launch_attention(p, static_cast<cudaStream_t>(stream)));
  return MIMO_OK;
}

size_t mimo_moe_layer_linear_workspace_bytes(int32_t T, int32_t N, int32_t K) {
  if (T < 1 || T > 16 || N < 8 || N % 8 || K < 256 || K % 64) return 0;
  const int S = linear_decode_splits(N, K, num_sms_current());
  return S > 1 ? (size_t)S * T * N * 4 : 0;
}

int mimo_moe_layer_linear(const uint16_t* x, const uint16_t* w, int32_t T, int32_t N, int32_t K, uint16_t* y,
                          void* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  if (!x || !w || !y || T < 1 || T > 16 || N < 8 || N % 8 || K < 256 || K % 64 || !a16(x) || !a16(w) || !a16(y) ||
      (workspace && !a16(workspace)))
    return MIMO_EINVAL;
  const int sms = num_sms_current();
  int S = linear_decode_splits(N, K, sms);
  while (S > 1 && (!workspace || workspace_bytes < (size_t)S * T * N * 4)) S /= 2;  // what the workspace holds
  MIMO_TRY(launch_linear_decode(x, w, T, N, K, S, y, S > 1 ? static_cast<float*>(workspace) : nullptr, status, sms,
                                static_cast<cudaStream_t>(stream)));
  return MIMO_OK;
}

int mimo_moe_layer_add_rmsnorm(const uint16_t* x, const uint16_t* delta, const uint16_t* weight, int32_t T,
                               int32_t H, float eps, uint16_t* h, uint16_t* r, void* stream) {
  if (!x || !delta || !h || !r || T < 1 || H < 8 || H % 8 || !(eps >= 0.f) || !a16(x) || !a16(delta) || !a16(h) ||
      !a16(r) || (weight && !a16(weight)))
    return MIMO_EINVAL;
  MIMO_TRY(launch_add_rmsnorm(x, delta, weight, T, H, eps, h, r, static_cast<cudaStream_t>(stream)));
  return MIMO_OK;
}

int mimo_moe_layer_swiglu(const uint16_t* gate_up, int32_t T, int32_t I, uint16_t* out, void* stream) {
  if (!gate_up || !out || T < 1 || I < 8 || I % 8 || !a16(gate_up) || !a16(out)) return MIMO_EINVAL;
  MIMO_TRY(launch_swiglu(gate_up, T, I, out, static_cast<cudaStream_t>(stream)));
  return MIMO_OK;
}

int mimo_moe_layer_add(const uint16_t* a, const uint16_t* b, int64_t n, uint16_t* out, void* stream) {
  if (!a || !b || !out || n < 8 || n % 8 || !a16(a) || !a16(b) || !a16(out)) return MIMO_EINVAL;
  MIMO_TRY(launch_add(a, b, (size_t)n, out, static_cast<cudaStream_t>(stream)));
  return MIMO_OK;
}

}  // extern "C"
