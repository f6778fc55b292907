// Internal launch interface between the C ABI (api.cu) and the kernels.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>
#include <cstdint>

#include "tma.h"

namespace mimo {

// Kernel launch with programmatic stream serialization: the kernel may start while the preceding
// kernel on the stream finishes; it calls pdl_wait() before touching that kernel's results.
// MIMO_MOE_PDL=0 launches plainly (a comparison knob).
bool pdl_enabled();
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Parameters of the expert tile kernel (see experts.cu).
struct ExpertParams {
  const uint8_t* w[2];  // packed e2m1 bytes of matrix m: [S][N][K/2]
  const uint8_t* s[2];  // e8m0 scales of matrix m: [S][N][K/32]
  int S, N, K, tiles;   // tiles = N / 16
  // work units: (pool slot, first route position p0, route count)
  const int32_t* unit_slot;
  const int32_t* unit_p0;  // null: p0 = unit * p0_stride
  const int32_t* unit_cnt;
  int p0_stride;
  const int32_t* num_units;  // device count, null: units_cap
  int units_cap;
  // B operand: row(route p) = rtok ? rtok[p] : p; values bsrc[row * K + k] (f16)
  const int32_t* rtok;
  const __half* bsrc;
  int brows;        // rows of bsrc (> 0: route rows outside [0, brows) set MIMO_ERANGE, read row 0)
  const float* rw;  // route weights (down, decode)
  // outputs (one per mode)
  __half* h_out;        // gate/up: SwiGLU output [P][N] (f16 copy of the bf16 value)
  float* part_out;      // down, decode: [P][N] float32 = dot * weight
  uint16_t* ypair_out;  // down, prefill: [P][N] bf16(dot)
  int pairs_rounding;
  int32_t* status;
};

// Parameters of the TMA-fed decode kernel (see experts.cu).  Passed as a __grid_constant__ so the
// tensor maps stay in parameter space.
struct DecodeParams {
  CUtensorMap wmap[2];  // weight maps of matrix m (gate/up or down), see tma.h
  CUtensorMap smap[2];  // scale maps
  int per_panel;        // weight maps are 2-D (one TMA box per 128-byte panel)
  int S, N, K, tiles;
  const int32_t* unit_slot;
  const int32_t* unit_cnt;
  int p0_stride;             // unit u's routes start at u * p0_stride
  const int32_t* num_units;  // device count, null: units_cap
  int units_cap;
  const int32_t* rtok;  // B row of route p (null: row p)
  const __half* bsrc;   // B rows [*, K] f16
  int brows;            // rows of bsrc (> 0: route rows outside [0, brows) set MIMO_ERANGE, read row 0)
  const float* rw;
  __half* h_out;
  float* part_out;
  int pairs_rounding;
  int32_t* status;
};
// kind 0: gate/up + SwiGLU (K <= 4096); kind 1: down x weight (K <= 2048)
cudaError_t launch_decode_tma(const DecodeParams& p, int kind, int num_sms, cudaStream_t st);

// Parameters of the tcgen05 block-scaled expert kernel (see tc_experts.cu).  Unit u's activation
// terms are rows [u * 2 * ntok, (u + 1) * 2 * ntok) of the term matrix: rows q < ntok hold the first
// e4m3 term of route q, rows ntok + q the second.
struct TcParams {
  CUtensorMap amap[2];   // weights of matrix m, 16U4_ALIGN16B, 128B swizzle: gate/up 2-D boxes
                         // [128 values, 128 rows]; down one 3-D view [chunk][row][128 values], box 2 chunks
  CUtensorMap smap[2];   // e8m0 scales of matrix m [S * Nw][K / 32], box [16 B, 128 rows]
  CUtensorMap bmap;      // activation terms [units * 2 * ntok][K] e4m3: box [128 B, 2 * ntok rows]
                         // (gate/up), or the 3-D view [chunk][row][128 B] with 2 chunks per box (down)
  CUtensorMap bsmap;     // their ue8m0 scales [units * 2 * ntok][K / 32], box [16 B, 2 * ntok rows]
  int S, Nw, K, tiles;   // Nw: weight rows (output features) per expert; tiles = Nw / 128 (Nw / 256 when an
                         // item takes two row tiles, decode down kind 1)
  const int32_t* unit_slot;
  const int32_t* unit_cnt;
  const int32_t* unit_p0;     // null: p0 = unit * p0_stride
  int p0_stride;
  const int32_t* btok;        // non-null: B rows are token rows (hi t, lo ntok + t) shared by every unit,
                              // and route q of a unit reads column btok[p0 + q]; null: B rows per route
  int btok_rows;              // token rows behind btok (a btok entry outside [0, btok_rows) sets MIMO_ERANGE)
  const int32_t* unit_first;  // first unit of the unit's expert group (null: one unit per group)
  const int32_t* unit_nsub;   // units in that group
  const int32_t* num_units;   // device count, null: units_cap
  int units_cap;
  int weights_once;           // weights are read once per call: stream them with L2 evict-first
  const float* rw;            // route weights (down, decode)
  uint8_t* hq;                // gate/up: h terms [units * 2 * ntok][Nw] e4m3
  uint8_t* hs;                // gate/up: h term scales [units * 2 * ntok][Nw / 32]
  float* part;                // down, decode: [P][Nw] = dot * weight
  uint16_t* ypair;            // down, prefill: [P][Nw] bf16(dot)
  const int32_t* out_row;     // down, decode kinds: partial of sorted route i goes to row out_row[i]
  float* const* peer_part;    // non-null: row r goes to rank r / peer_rows's buffer, row r % peer_rows
  int peer_rows;
  int pairs_rounding;
  int32_t* status;
  // Decode, per-unit readiness instead of the grid dependency wait: the gate/up launch (kind 0) adds 1 to
  // ready[unit] per epilogue warp and item after its h stores; the paired-tile down launch (kind 1,
  // MODE 3) skips the wait for the whole gate/up grid and loads a unit's h once ready[unit] reaches
  // ready_need, so down items of finished units run on SMs the gate/up launch has already left.
  int32_t* ready;
  int ready_need;
  // Down, decode, fused combine (cy non-null, partials in `part`): the CTA storing the last unit's
  // partials of output rows [128 r, 128 r + 128) (cdone[r] counts them, zeroed per call) forms
  // cy[m] = bf16(sum over k in order of part[cgidx[m * ctopk + k]]) for those rows (cgidx null: the
  // (u, r) scatter order over curows / cucnt with p0_stride route slots per unit).
  uint16_t* cy;
  const int32_t* cgidx;
  const int32_t* curows;
  const int32_t* cucnt;
  int32_t* cdone;
  int cM, ctopk;
};
// Both decode passes in one launch (tc_experts.cu): gate/up params (kind 0 layout) and down params
// (kind 1 layout) over the same units; ready: [units_cap] zeroed counters.
struct TcFusedParams {
  TcParams gu, dn;
  int32_t* ready;
};
// fp4: kind::mxf4 with packed weight maps and five e2m1 activation terms (maps from packed64_map,
// term rows unit * 40 + t * 8 + q); else kind::mxf8f6f4 with the kind 0 / kind 1 maps.
cudaError_t launch_tc_decode_fused(const TcFusedParams& f, bool fp4, int num_sms, cudaStream_t st);

// Stream-K decode (tc_experts.cu, tc_decode_sk_kernel): both passes in one launch of `ctas` CTAs, each
// streaming an equal contiguous range of 512-value K groups of the gate/up tiles, then of the down
// tiles.  A tile's groups are added in a fixed order (a right fold); a CTA whose range starts inside a
// tile publishes its partial fold of that tile in part_g / part_d behind per-warp flags for the CTA
// before it.  Scratch sizes: sk_part_*_floats / sk_flag_count; flags and ready zeroed per call.
struct TcSkParams {
  TcParams gu, dn;
  int32_t* ready;   // [units_cap] h readiness counters (8 epilogue warps per gate/up tile)
  float* part_g;    // [ctas][4 quads][2 matrices][8 columns][32 lanes]
  float* part_d;    // [ctas][4 quads][8 columns][32 lanes]
  int32_t* flag_g;  // [ctas][8 epilogue warps]
  int32_t* flag_d;  // [ctas][8 epilogue warps]
  int ctas;
  // Fused combine (y non-null; the down pass then writes dn.part, not peers): the CTA that completes
  // the last down tile of output rows [128 r, 128 r + 128) (done[r] counts the tiles, zeroed per call)
  // forms y[m] = bf16(sum over k in order of part[gidx[m * topk + k]]) for those rows (gidx null: the
  // (u, r) scatter order over urows / ucnt with R route slots per unit), like combine_decode_kernel.
  uint16_t* y;
  const int32_t* gidx;
  const int32_t* urows;
  const int32_t* ucnt;
  int32_t* done;  // [H / 128]
  int M, topk, R;
};
constexpr int kSkGroupK = 512;  // K values per stream-K group (4 chunks of 128)
inline size_t sk_part_g_floats(int ctas) { return (size_t)ctas * 4 * 2 * 8 * 32; }
inline size_t sk_part_d_floats(int ctas) { return (size_t)ctas * 4 * 8 * 32; }
inline size_t sk_flag_count(int ctas) { return (size_t)ctas * 8; }  // per phase
cudaError_t launch_tc_decode_sk(const TcSkParams& f, cudaStream_t st);
// kind 0: decode gate/up (8 routes per unit), 1: decode down, 2: prefill gate/up (64 routes per
// unit), 3: prefill down.
cudaError_t launch_tc_experts(const TcParams& p, int kind, int num_sms, cudaStream_t st);
// Dense block-scaled tensor peak probe: num_sms CTAs, each iters x (M 128, N 256, K 128) MMAs of
// kind::mxf8f6f4 (e2m1 x e4m3, fp4 = 0) or kind::mxf4 (e2m1 x e2m1, fp4 = 1).
// Prefill kinds 2 / 3 on SM pairs (clusters of two CTAs, tcgen05 cta_group::2): 256-row weight tiles
// (tiles = Nw / 256) and term maps whose boxes hold half a unit's term rows (64).
cudaError_t launch_tc_pair(const TcParams& p, int kind, int num_sms, cudaStream_t st);
// Same splits into five e2m1 terms (kind::mxf4 decode): by-token rows (token t's term j at row
// j * 8 + t), or per-unit rows (unit u, route q, term j at row u * 40 + j * 8 + q); K / 2 bytes a row.
cudaError_t launch_tc_split_tokens_fp4(const uint16_t* x, int T, int K, uint8_t* bq, uint8_t* bs, int32_t* status,
                                       cudaStream_t st);
cudaError_t launch_tc_split_fp4(const uint16_t* x, int K, const int32_t* unit_cnt, const int32_t* unit_p0,
                                int p0_stride, const int32_t* rtok, const int32_t* num_units, int units_cap,
                                uint8_t* bq, uint8_t* bs, int32_t* status, cudaStream_t st, int x_ld = 0,
                                int x_rows = 0);
// Splits bf16 activation rows into the two e4m3 terms + ue8m0 scales of each unit's routes.
// x rows are x_ld elements apart; x_rows > 0 bounds the route rows (outside: MIMO_ERANGE, row 0 read).
cudaError_t launch_tc_split(const uint16_t* x, int K, const int32_t* unit_cnt, const int32_t* unit_p0,
                            int p0_stride, const int32_t* rtok, const int32_t* num_units, int units_cap,
                            int ntok, uint8_t* bq, uint8_t* bs, int32_t* status, cudaStream_t st, int x_ld = 0,
                            int x_rows = 0);
// Expert-parallel exchange over peer memory (peer.cu).
cudaError_t launch_peer_barrier(int32_t* const* signals, int32_t* my_signals, int rank, int world, int32_t* epoch,
                                uint64_t limit_ns, int32_t* status, cudaStream_t st);
cudaError_t launch_route_scatter(const uint16_t* x, const float* logits, const float* bias, int T, int H, int E,
                                 int topk, int32_t* const* rows, int ld, int rank, int world, cudaStream_t st);
cudaError_t launch_routes_prep(const int32_t* idx, const float* w, int route_ld, int rows, int topk, int base, int S,
                               int unit_max, int ucap, int32_t* order, int32_t* rtok, float* rw, int32_t* unit_slot,
                               int32_t* unit_p0, int32_t* unit_cnt, int32_t* num_units, cudaStream_t st);
// Splits token rows x[t] (t < T <= 8) into terms at rows t (hi) and 8 + t (lo) of bq/bs.
cudaError_t launch_tc_split_tokens(const uint16_t* x, int T, int K, uint8_t* bq, uint8_t* bs, int32_t* status,
                                   cudaStream_t st);
constexpr int kTcDecodeRoutes = 8;   // routes per decode unit on the tcgen05 path
constexpr int kTcDecodeEpiWarps = 8;  // epilogue warps of the decode tcgen05 kernels
constexpr int kTcFp4Terms = 5;  // e2m1 activation terms of the kind::mxf4 decode path
constexpr int kTcPrefillRoutes = 64; // routes per prefill unit on the tcgen05 path

// T > 8: tcgen05 GEMM (128 x 64 tiles; an expired wait sets MIMO_ETIMEOUT in `status` when given);
// T <= 8 or unaligned operands: one warp per expert row.
cudaError_t launch_router_logits(const uint16_t* x, const uint16_t* w, float* logits, int T, int H,
                                 int E, cudaStream_t st, int32_t* status = nullptr);
cudaError_t launch_router_topk(const float* logits, const float* bias, int T, int E, int topk,
                               int32_t* idx, float* weight, cudaStream_t st);
// Decode routing (T <= 8), two launches: logits + scores (+ the expert kernels' x terms, and zeroing of
// ready_n words at `ready`), then top-k and grouping in one CTA.
cudaError_t launch_route_decode(const uint16_t* x, const uint16_t* w, const float* bias, int T, int H,
                                int E, int topk, int R, float* logits, int32_t* idx, float* wts,
                                int32_t* uids, int32_t* urows, int32_t* ucnt, float* uw,
                                int32_t* gidx, int32_t* num_unique, __half* x16, uint8_t* xq, uint8_t* xs,
                                float* score, int32_t* status, cudaStream_t st, int fp4 = 0,
                                int32_t* ready = nullptr, int ready_n = 0);
cudaError_t launch_group_routes(const int32_t* idx, const float* weight, int M, int topk, int R,
                                int E, int32_t* uids, int32_t* urows, int32_t* ucnt, float* uw,
                                int32_t* gidx, int32_t* num_unique, int32_t* status, cudaStream_t st);
size_t dispatch_workspace_bytes(int P, int E);
// Expert-parallel prefill exchange plan and row gathers (ep_plan.cu).
size_t ep_plan_workspace_bytes(int T, int world);
cudaError_t launch_ep_plan(const int32_t* idx, int T, int topk, int per_rank, int world, int64_t* counts,
                           int32_t* order, int32_t* inv, int32_t* send_tok, int32_t* send_tag, void* ws,
                           int32_t* status, cudaStream_t st);
cudaError_t launch_gather_rows(const uint16_t* x, long long x_rows, int H, const int32_t* rows, long long n,
                               uint16_t* out, int32_t* status, cudaStream_t st);
cudaError_t launch_ep_recv_index(const int32_t* tag, const int64_t* recv_counts, int world, long long n_recv,
                                 int32_t* route_row, int32_t* eid, int32_t* status, cudaStream_t st);
// Routes with expert id - id_base outside [0, E) are dropped (inv = -1); they set MIMO_ERANGE unless
// skip_outside (expert parallelism: routes to other ranks' experts).
cudaError_t launch_dispatch(const int32_t* idx, int P, int E, int32_t* offsets, int32_t* order,
                            int32_t* inv, void* ws, int32_t* status, cudaStream_t st, int id_base = 0,
                            int skip_outside = 0);
cudaError_t launch_build_units(const int32_t* offsets, const int32_t* slot_of, int E, int S,
                               int unit_max, int ucap, int32_t* unit_slot, int32_t* unit_p0,
                               int32_t* unit_cnt, int32_t* unit_first, int32_t* unit_nsub,
                               int32_t* num_units, const int32_t* order,
                               const float* weight, int P, int topk, int32_t* rtok, float* rw,
                               int32_t* status, cudaStream_t st, const int32_t* route_row = nullptr);
cudaError_t launch_to_f16(const uint16_t* x, __half* y, size_t n, int32_t* status, cudaStream_t st);
// kind: 0 decode gate/up, 1 decode down, 2 prefill gate/up, 3 prefill down
cudaError_t launch_expert_tiles(const ExpertParams& p, int kind, int num_sms, cudaStream_t st);
// part_rows: rows of part (gidx entries at or beyond it set MIMO_ERANGE in status and are skipped).
cudaError_t launch_combine_rows(const float* part, const int32_t* gidx, int M, int topk, int H, long long part_rows,
                                uint16_t* y, int32_t* status, cudaStream_t st);
cudaError_t launch_combine_decode(const float* part, const int32_t* gidx, const int32_t* urows,
                                  const int32_t* ucnt, const int32_t* num_unique, int ucap, int R,
                                  int M, int topk, int H, uint16_t* y, int32_t* status, cudaStream_t st);
cudaError_t launch_rmsnorm(const uint16_t* x, const uint16_t* weight, int T, int H, float eps, uint16_t* y,
                           cudaStream_t st);
cudaError_t launch_combine_prefill(const uint16_t* ypair, const int32_t* inv, const float* w, int T,
                                   int topk, int H, uint16_t* y, cudaStream_t st);
cudaError_t launch_fill_synthetic(uint32_t* gw, uint8_t* gs, uint32_t* uw, uint8_t* us, uint32_t* dw,
                                  uint8_t* ds, int S, int H, int I, uint64_t seed, int layer,
                                  int first_expert, cudaStream_t st);

constexpr int kPrefillUnit = 64;  // routes per prefill work unit (8 token blocks of 8)

// ---- decoder layer around the MoE block (layer.cu)
struct AttnParams {
  const uint16_t* q;   // [T][nq][dqk] bf16, RoPE applied
  const uint16_t* k;   // [nkv][cap][dqk] bf16 cache, position p in slot p % cap
  const uint16_t* v;   // [nkv][cap][dv]
  const float* sinks;  // [nq] sink logits, or null
  uint16_t* out;       // [T][nq][dv] bf16
  float* part_o;       // splits > 1: [splits][T*nq][dv] unnormalised partial outputs
  float* part_ml;      // splits > 1: [splits][T*nq] (running max in log2 units, row sum)
  int T, nq, nkv, G, dqk, dv, cap, window, pos0, splits;
  float scale_log2;    // head_dim^-0.5 * log2(e)
  int32_t* status;     // optional device word: MIMO_ETIMEOUT when a bounded wait of the tcgen05 kernel expires
};
// Parameters of the tcgen05 attention kernel (attn_tc.cu): TMA maps of q [T][nq][dqk] (box 64 x G x 128/G),
// the K cache [nkv][cap][dqk] and the V cache [nkv][cap][dv] (boxes 64 x 128 x 1), 128B swizzle.
struct AttnTcParams {
  CUtensorMap qmap, kmap, vmap;
  const float* sinks;
  uint16_t* out;
  int32_t* status;
  float* part_o;   // splits > 1: unnormalised partials (the AttnParams layout)
  float* part_ml;
  int T, nq, nkv, G, cap, window, pos0, ntiles, splits;
  float scale_log2;
};
struct RopeParams {
  const uint16_t* qkv;  // [T][nq*dqk + nkv*dqk + nkv*dv] projection rows
  uint16_t* q;          // [T][nq][dqk]
  uint16_t* kc;         // [nkv][cap][dqk]
  uint16_t* vc;         // [nkv][cap][dv]
  int T, nq, nkv, dqk, dv, rot, pos0, cap, has_vscale;
  float v_scale;        // already a bf16 value
  double log_base;      // ln(rope_theta)
};
// Decode-size projection y[T, N] = bf16(x[T, K] . W[N, K]^T) on tcgen05 (linear.cu): TMA maps of W (box
// 64 x 128 rows) and x (box 64 x 16 rows), S K segments (partials [S][T][N] float32 when S > 1).
struct LinearParams {
  CUtensorMap wmap, xmap;
  uint16_t* y;
  float* part;
  int32_t* status;
  int T, N, K, S, tiles;
};
int linear_decode_splits(int N, int K, int num_sms);
cudaError_t launch_linear_decode(const uint16_t* x, const uint16_t* w, int T, int N, int K, int S, uint16_t* y,
                                 float* part, int32_t* status, int num_sms, cudaStream_t st);
bool attn_dims_supported(int dqk, int dv);
cudaError_t launch_attention(const AttnParams& p, cudaStream_t st);
bool attn_tc_supported(const AttnParams& p);
int attn_auto_splits(const AttnParams& p, int num_sms);  // split count for the kernel launch_attention picks
cudaError_t launch_attention_tc(const AttnParams& p, int32_t* status, cudaStream_t st);
cudaError_t launch_rope_store(const RopeParams& p, cudaStream_t st);
cudaError_t launch_add_rmsnorm(const uint16_t* x, const uint16_t* d, const uint16_t* weight, int T, int H, float eps,
                               uint16_t* h, uint16_t* r, cudaStream_t st);
cudaError_t launch_swiglu(const uint16_t* gu, int T, int I, uint16_t* out, cudaStream_t st);
cudaError_t launch_add(const uint16_t* a, const uint16_t* b, size_t n, uint16_t* out, cudaStream_t st);

}  // namespace mimo
