/*
 * mimo_moe.h — C ABI of the B200 (sm_100a) MiMo MoE block:
 *   router -> dispatch -> MXFP4 expert products -> fixed-order combine.
 *
 * Every pointer argument is a DEVICE pointer except `pools`, which is a host pointer to a struct of
 * device pointers; `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 * The entry points below do not allocate memory, synchronise the host or change the current device:
 * outputs and workspaces are caller-owned, and every launch is stream-ordered.  Return value: MIMO_OK
 * or an error code below (host-side argument checks and launch errors).  Errors found while the kernels
 * run (a route table that overflows R, an activation outside the f16 range, a bounded device wait that
 * expired) are written to the optional device word `status` (caller-zeroed int32; first error wins) and
 * are visible after the stream is synchronised.
 *
 * Tensor contract (the reference's expert pool layout, engine/mimo_stream/model.py:28-45 and
 * scripts/convert-mimo-v26-mlx.py:8-12): per MoE layer and slot s,
 *   gate_w, up_w  uint32 [S, I, H/8]   e2m1 nibbles, 8 per word, element k = nibble k%8 of word k/8
 *   gate_s, up_s  uint8  [S, I, H/32]  e8m0 scale per 32 consecutive K elements (s=0 -> 2^-127, 255 -> NaN)
 *   down_w        uint32 [S, H, I/8]
 *   down_s        uint8  [S, H, I/32]
 * Activations are bf16 (passed as uint16_t bit patterns); router logits and weights are float32.
 */
#ifndef MIMO_MOE_H
#define MIMO_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MIMO_MOE_VERSION 1

enum mimo_moe_error {
  MIMO_OK = 0,
  MIMO_EINVAL = 1,    /* bad shape, null pointer, unsupported size, workspace too small */
  MIMO_ERANGE = 2,    /* expert id outside [0,E), more than R rows on one expert, activation overflow */
  MIMO_ETIMEOUT = 3,  /* a bounded device-side wait expired; the kernel returned without the result */
  MIMO_ECUDA = 4,     /* CUDA launch / runtime error (see mimo_moe_last_cuda_error) */
  MIMO_EIO = 5,       /* file open / read failure or short read (expert-file loader) */
};

/* Expert pool of one MoE layer (device pointers, reference layout above). */
typedef struct mimo_moe_pools {
  const uint32_t* gate_w;
  const uint8_t* gate_s;
  const uint32_t* up_w;
  const uint8_t* up_s;
  const uint32_t* down_w;
  const uint8_t* down_s;
  int32_t num_slots; /* S */
  int32_t hidden;    /* H, multiple of 2048 (4096 for MiMo) */
  int32_t inter;     /* I, multiple of 2048 (2048 for MiMo) */
} mimo_moe_pools;

/* Library version and error text. */
int mimo_moe_version(void);
const char* mimo_moe_strerror(int code);
/* Last CUDA error code seen by a failing call on this host thread (0 if none). */
int mimo_moe_last_cuda_error(void);

/*
 * Router — replaces Router.__call__ (engine/mimo_stream/model.py:58-65).
 *   logits[T,E] = fp32(x[T,H]) . fp32(w[E,H])^T         (float32 accumulation)
 *   s = sigmoid(logits); sel = s + bias; idx = top-k of sel (descending sel, ties by ascending id)
 *   weight[t,j] = s[t,idx[t,j]] / (sum_j s[t,idx[t,j]] + 1e-20)   (float32 sum in j order)
 * E multiple of 32 and <= 256; 1 <= topk <= 8; H multiple of 256.  `logits` is a caller buffer [T,E].
 */
int mimo_moe_router(const uint16_t* x, const uint16_t* w, const float* bias, int32_t T, int32_t H,
                    int32_t E, int32_t topk, float* logits, int32_t* idx, float* weight, void* stream);

/* The selection half of the router, from given logits — model.py:60-64.  bias may be NULL (zeros). */
int mimo_moe_topk(const float* logits, const float* bias, int32_t T, int32_t E, int32_t topk,
                  int32_t* idx, float* weight, void* stream);

/*
 * Decode route grouping — replaces group_routes (engine/mimo_stream/kernels.py:149-173).
 * idx/weight [M,topk] (expert or slot ids in [0,E)) -> per distinct id u (ascending):
 *   uids[u], urows[u,R] (row per route, 0-padded), ucnt[u], uw[u,R] (weight, 0-padded),
 *   gather_idx[M*topk] = u*R + c, num_unique[0] = U.
 * Output arrays are sized for U_max = min(E, M*topk).  M*topk <= 1024.  More than R routes on one id
 * sets MIMO_ERANGE in `status` (the reference raises ValueError, kernels.py:167-168).
 */
int mimo_moe_group_routes(const int32_t* idx, const float* weight, int32_t M, int32_t topk, int32_t R,
                          int32_t E, int32_t* uids, int32_t* urows, int32_t* ucnt, float* uw,
                          int32_t* gather_idx, int32_t* num_unique, int32_t* status, void* stream);

/*
 * Prefill dispatch — replaces the pair permutation of Engine._moe_prefill
 * (engine/mimo_stream/model.py:235-244, 266-268): pairs p = t*topk + j in flat order, stable-sorted by
 * idx; order[i] = pair at sorted position i, inv[p] = sorted position of pair p, offsets[E+1] = bucket
 * starts.  Workspace: mimo_moe_dispatch_workspace_bytes(T, topk, E).
 */
size_t mimo_moe_dispatch_workspace_bytes(int32_t T, int32_t topk, int32_t E);
int mimo_moe_dispatch(const int32_t* idx, int32_t T, int32_t topk, int32_t E, int32_t* offsets,
                      int32_t* order, int32_t* inv, void* workspace, size_t workspace_bytes,
                      int32_t* status, void* stream);

/*
 * Expert-parallel prefill exchange plan (no reference counterpart: the reference keeps every expert
 * on one device; this moves each pair of model.py:235-244 to the rank owning its expert).  Rank d owns
 * experts [d*per_rank, (d+1)*per_rank); routes p = t*topk + j are stable-sorted by destination rank:
 *   counts   int64 [world][2]  (routes, token rows) sent to each rank
 *   order    int32 [P]         route at send position s;   inv [P] = send position of route p
 *                              (-1 and MIMO_ERANGE for an expert id outside [0, world*per_rank))
 *   send_tok int32 [P]         token of send row r, the rows of rank 0 first (sum counts[:,1] used):
 *                              each token row travels once to each rank owning any of its experts
 *   send_tag int32 [P][2]      (row within the destination's rows, local expert id) per send position
 * topk <= 16, world <= 8.  Workspace: mimo_moe_ep_plan_workspace_bytes(T, world).
 * mimo_moe_gather_rows: out[r] = x[rows[r]] for r < n (bf16 rows of H; a row outside [0, x_rows) sets
 * MIMO_ERANGE and gives zeros).  mimo_moe_ep_recv_index, on the receiving rank: route i of the
 * received routes (recv_counts = the senders' counts rows, device int64 [world][2]) names row tag[i][0]
 * of the rows received from its sender; route_row[i] = that row's index in the received rows (-1 and
 * MIMO_ERANGE outside them), eid[i] = tag[i][1].  The routes then run through mimo_moe_prefill_routes.
 */
size_t mimo_moe_ep_plan_workspace_bytes(int32_t T, int32_t world);
int mimo_moe_ep_plan(const int32_t* idx, int32_t T, int32_t topk, int32_t per_rank, int32_t world,
                     int64_t* counts, int32_t* order, int32_t* inv, int32_t* send_tok, int32_t* send_tag,
                     void* workspace, size_t workspace_bytes, int32_t* status, void* stream);
int mimo_moe_gather_rows(const uint16_t* x, int64_t x_rows, int32_t H, const int32_t* rows, int64_t n,
                         uint16_t* out, int32_t* status, void* stream);
int mimo_moe_ep_recv_index(const int32_t* recv_tag, const int64_t* recv_counts, int32_t world, int64_t n_recv,
                           int32_t* route_row, int32_t* eid, int32_t* status, void* stream);

/*
 * Small-batch expert products over distinct experts — replaces moe_experts
 * (engine/mimo_stream/kernels.py:176-199: kernel A gate/up+SwiGLU, kernel B down*weight, combine).
 *   x [M,H] bf16; uslot/urows/ucnt/uw/gather_idx from mimo_moe_group_routes (uslot = pool slot per
 *   distinct expert); U = capacity of those arrays; num_unique (device, may be NULL -> U) = live count;
 *   topk = routes per row in gather_idx [M*topk].
 *   y [M,H] bf16 = sum over each row's routes, in gather_idx order, of w * expert(x_row)   (float32 sum)
 *   gather_idx NULL -> per-row sum in (u, r) order (the reference's scatter-add, kernels.py:196-197).
 *   pairs_rounding != 0 rounds each expert's down output to bf16 before weighting, as the reference's
 *   stock gather_qmm path does at M == 1 (model.py:173-182).
 * 1 <= R <= 8, M <= 128.  Workspace: mimo_moe_experts_workspace_bytes(M, U, R, H, I).
 */
size_t mimo_moe_experts_workspace_bytes(int32_t M, int32_t U, int32_t R, int32_t H, int32_t I);
int mimo_moe_experts(const uint16_t* x, const mimo_moe_pools* pools, const int32_t* uslot,
                     const int32_t* urows, const int32_t* ucnt, const float* uw,
                     const int32_t* num_unique, int32_t U, int32_t R, const int32_t* gather_idx,
                     int32_t topk, int32_t M, int32_t pairs_rounding, uint16_t* y, void* workspace,
                     size_t workspace_bytes, int32_t* status, void* stream);

/*
 * Prefill expert products — replaces Engine._pair_outputs + the combine of Engine._moe_prefill
 * (engine/mimo_stream/model.py:221-271): per (token, k) pair, bf16 gate/up, bf16 SwiGLU, bf16 down
 * output; y[t] = bf16(sum_k fp32(out[t,k]) * w[t,k]) in k order.
 *   idx/weight [T,topk] expert ids in [0,E); slot_of [E] (may be NULL: slot = expert id, E = S) maps
 *   expert id -> pool slot.  Workspace: mimo_moe_prefill_workspace_bytes(T, topk, H, I, E).
 */
size_t mimo_moe_prefill_workspace_bytes(int32_t T, int32_t topk, int32_t H, int32_t I, int32_t E);
int mimo_moe_prefill(const uint16_t* x, const mimo_moe_pools* pools, const int32_t* slot_of, int32_t E,
                     const int32_t* idx, const float* weight, int32_t T, int32_t topk, uint16_t* y,
                     void* workspace, size_t workspace_bytes, int32_t* status, void* stream);
/*
 * Per-route prefill products (the expert side of expert-parallel prefill): route p applies expert idx[p]
 * to row route_row[p] of x [x_rows,H] (x_rows <= P); y[p] = the route's bf16 pair output
 * (model.py:221-228), the same bits mimo_moe_prefill combines.  Workspace:
 * mimo_moe_prefill_workspace_bytes(P, 1, H, I, E).
 */
int mimo_moe_prefill_routes(const uint16_t* x, int32_t x_rows, const mimo_moe_pools* pools,
                            const int32_t* slot_of, int32_t E, const int32_t* route_row, const int32_t* idx,
                            int32_t P, uint16_t* y, void* workspace, size_t workspace_bytes, int32_t* status,
                            void* stream);

/*
 * The whole block — replaces one MoE layer of Engine.forward (engine/mimo_stream/model.py:303-336)
 * with all experts resident (E = S): router, then the reference's dispatch rule (T == 1: stock-path
 * rounding; 2 <= T <= 8: distinct-expert kernels; T > 8: prefill path).  idx_out/w_out (may be NULL)
 * receive the routes.  Workspace: mimo_moe_block_workspace_bytes(T, H, I, E, topk).
 */
size_t mimo_moe_block_workspace_bytes(int32_t T, int32_t H, int32_t I, int32_t E, int32_t topk);
int mimo_moe_block(const uint16_t* x, const uint16_t* router_w, const float* bias,
                   const mimo_moe_pools* pools, int32_t T, int32_t topk, uint16_t* y, int32_t* idx_out,
                   float* w_out, void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/*
 * Expert parallelism building blocks (the reference runs on one device; these follow the multi-GPU
 * design of the B200 build: experts [expert_base, expert_base + S) live on this GPU).
 *
 * mimo_moe_experts_routes: per-route products of every route whose expert is local.  x holds `rows`
 * token rows (bf16, row r at x + r * x_ld; x_ld = 0 means H); idx/weight hold row r's topk global
 * expert ids and router weights at idx + r * route_ld (route_ld = 0 means topk).  Route
 * p = r * topk + k gets fp32(down . SwiGLU(gate . x_r, up . x_r)) * weight[r, k] (bf16-rounded before
 * the weight when pairs_rounding != 0, the M = 1 stock path), exactly the per-route partial of
 * mimo_moe_experts (kernels.py:120; model.py:173-182).  Output: with part (float32 [rows * topk, H]),
 * part is zeroed and row p receives the partials of local routes, so the partials of all ranks add
 * exactly (one nonzero term per element); with peer_part (a device array of world pointers), row p
 * is stored straight into peer_part[p / rows_per_rank] at row p % rows_per_rank (each route on
 * exactly one rank: no zeroing, no reduction).  Workspace:
 * mimo_moe_experts_routes_workspace_bytes(rows, topk, H, I, S).
 *
 * mimo_moe_combine: y[m] = bf16(sum over k in order of part[gather_idx[m * topk + k]]) with
 * gather_idx = NULL meaning row m * topk + k (kernels.py:194-199).  part holds part_rows rows
 * (<= 0: M * topk); a gather_idx entry at or beyond part_rows sets MIMO_ERANGE in *status (may be
 * NULL) and is skipped, as negative entries are.
 *
 * Peer-memory exchange (one process per GPU on one node): mimo_moe_peer_alloc allocates `bytes` of
 * zeroed device memory and writes its 64-byte CUDA IPC handle; mimo_moe_peer_open maps another
 * process's handle (mimo_moe_peer_close unmaps, mimo_moe_peer_free frees).  mimo_moe_peer_barrier
 * orders everything issued before it on every rank before everything issued after it on every rank:
 * signals[r] points at rank r's int32[world] signal array, my_signals at this rank's, epoch at a
 * device counter that starts at 0; a wait longer than timeout_us microseconds (0: 2 s) sets
 * MIMO_ETIMEOUT in *status and the barrier kernel returns (a rank that never arrives is reported, the
 * GPU does not hang).
 * mimo_moe_route_scatter routes T <= 8 tokens (router logits into `logits`, float32 [T, E]) and stores
 * each token's packed row [x as H/2 int32 words | topk ids | topk weights] into rows[r] at row
 * rank * T + t for every rank r (ld int32 words per row).
 */
size_t mimo_moe_experts_routes_workspace_bytes(int32_t rows, int32_t topk, int32_t H, int32_t I, int32_t S);
int mimo_moe_experts_routes(const uint16_t* x, int32_t x_ld, int32_t rows, const mimo_moe_pools* pools,
                            int32_t expert_base, const int32_t* idx, const float* weight, int32_t route_ld,
                            int32_t topk, int32_t pairs_rounding, float* part, float* const* peer_part,
                            int32_t rows_per_rank, void* workspace, size_t workspace_bytes, int32_t* status,
                            void* stream);
int mimo_moe_combine(const float* part, int64_t part_rows, const int32_t* gather_idx, int32_t M, int32_t topk,
                     int32_t H, uint16_t* y, int32_t* status, void* stream);
/* Prefill combine (model.py:266-271): y[t] = bf16(sum over k in order of fp32(ypair[inv[t*topk+k]]) *
 * weight[t*topk+k]), skipping inv < 0.  ypair bf16 [*, H] (per-route expert outputs). */
int mimo_moe_combine_pairs(const uint16_t* ypair, const int32_t* inv, const float* weight, int32_t T, int32_t topk,
                           int32_t H, uint16_t* y, void* stream);
/* RMSNorm of each row before an MoE layer (model.py:75 `post_attention_layernorm`, MLX
 * fast.rms_norm): y = bf16(x * rsqrt(mean(x^2) + eps)), times weight (bf16 [H]) when weight is not
 * null.  x, y bf16 [T, H], 16-byte aligned, H a multiple of 8; x == y is allowed. */
int mimo_moe_rmsnorm(const uint16_t* x, const uint16_t* weight, int32_t T, int32_t H, float eps, uint16_t* y,
                     void* stream);
/* Expert-file loader.  One contiguous byte range of a file and where it goes. */
typedef struct mimo_moe_file_span {
  int64_t file_offset;
  int64_t nbytes;
  void* dst; /* device memory (dst_host == 0) or host memory */
} mimo_moe_file_span;

/* Copies the spans of one file (a converted experts-LNN.safetensors: expert e of a projection at
 * base + e * stride, 16 KiB aligned; scripts/convert-mimo-v26-mlx.py:92-131) to their destinations.
 * Replaces the reference's SSD streaming (engine/mimo_stream/store.py:14-82: ExpertStore.jobs +
 * IOPool.run, a preadv thread pool into GPU-visible slot memory).  `threads` reader threads pread in
 * chunks of `chunk_bytes` (a multiple of 4096) into pinned staging buffers and copy them on their own
 * streams, ordered after the work already queued on `stream`; O_DIRECT for 4 KiB-aligned chunks when
 * `direct` is set.  With dst_host the reads go straight into host memory (no CUDA calls).  Blocks
 * until every byte has landed.  Returns MIMO_EIO when the file cannot be opened or is too short. */
int mimo_moe_read_file_spans(const char* path, const mimo_moe_file_span* spans, int32_t n, int32_t threads,
                             int64_t chunk_bytes, int32_t direct, int32_t dst_host, void* stream);
int mimo_moe_peer_alloc(size_t bytes, void** ptr, void* handle);
int mimo_moe_peer_open(const void* handle, void** ptr);
int mimo_moe_peer_close(void* ptr);
int mimo_moe_peer_free(void* ptr);
int mimo_moe_peer_barrier(int32_t* const* signals, int32_t* my_signals, int32_t rank, int32_t world,
                          int32_t* epoch, int32_t timeout_us, int32_t* status, void* stream);
int mimo_moe_route_scatter(const uint16_t* x, int32_t T, int32_t H, const uint16_t* router_w, const float* bias,
                           int32_t E, int32_t topk, int32_t* const* rows, int32_t ld, int32_t rank, int32_t world,
                           float* logits, void* stream);

/*
 * mimo_moe_experts with no workspace argument (no counterpart in the reference).  For callers that
 * cannot allocate device memory when they run the block - a runtime that passes only activations and
 * weights, a fixed preallocated arena, a process barred from cudaMalloc - the scratch lives in a
 * fixed device array inside the library, held on every GPU that loads it until exit
 * (mimo_moe_experts_static_scratch_bytes(), about 10 MiB).  Limits: M <= 8, U*R <= 512, H <= 4096,
 * I <= 2048; larger sizes return MIMO_ERANGE without launching.  The first call on a device (and
 * again in a new CUDA context of it) looks up the array's device address, so make it before any
 * stream capture.  All calls share the array: calls that overlap on the GPU race, so issue them on
 * one stream.  Arguments as mimo_moe_experts.  It runs the mma.sync decode kernels (f16 tensor-core
 * products of CUDA-core-decoded e2m1 weights), not the tcgen05 kernels mimo_moe_experts takes for
 * TMA-aligned pools, so its results match mimo_moe_experts within the output tolerance (rel_err
 * <= 1e-2 against the reference path's restatement), not bit for bit, and it is slower at M = 8.
 */
size_t mimo_moe_experts_static_scratch_bytes(void);
int mimo_moe_experts_static(const uint16_t* x, const mimo_moe_pools* pools, const int32_t* uslot,
                            const int32_t* urows, const int32_t* ucnt, const float* uw,
                            const int32_t* num_unique, int32_t U, int32_t R, const int32_t* gather_idx,
                            int32_t topk, int32_t M, int32_t pairs_rounding, uint16_t* y, int32_t* status,
                            void* stream);

/*
 * Expert residency table (host) — replaces engine/mimo_stream/cache.py:13-65 (SlotCache): which experts
 * of one layer occupy its S device slots, with the reference's decayed-LFU eviction.  For a model or a
 * device where a layer's experts do not all fit in HBM; the caller copies each returned (expert, slot)
 * load into the slot and hands the kernels the slot map (mimo_moe_prefill's slot_of, or per-slot ids
 * to mimo_moe_group_routes / mimo_moe_experts).
 *   create(S, E): S slots (1 <= S <= E) for experts [0, E); NULL on bad sizes.  destroy frees it.
 *   preload(experts, n): experts[i] into slot i for i < min(n, S) (cache.py:24-28); loads written to
 *     load_expert/load_slot, *n_loads = min(n, S).
 *   resolve(needed, n, count, stats): one tick; needed = the step's distinct expert ids; counts them
 *     (count != 0), stamps their last use, assigns the missing ones the lowest-scoring slots
 *     (count * 1e12 + last use; empty slots -1; slots of needed experts never taken; ties and victim
 *     order by ascending slot), and adds to the hit / miss counters (stats != 0) (cache.py:30-62).
 *     The loads are written in `needed` order.  MIMO_ERANGE, with nothing changed, when n > S;
 *     MIMO_EINVAL for repeated or out-of-range ids.
 *   decay(): halves every count (cache.py:64-65; the engine calls it every 16 decode tokens).
 *   state(): copies slot_of [E] (expert -> slot or -1), expert_in [S] (slot -> expert or -1) and the
 *     hit / miss counters (any pointer may be NULL).
 * Host-only calls (no CUDA); one table per layer, not thread-safe.
 */
void* mimo_moe_slot_cache_create(int32_t n_slots, int32_t n_experts);
void mimo_moe_slot_cache_destroy(void* cache);
int mimo_moe_slot_cache_preload(void* cache, const int32_t* experts, int32_t n, int32_t* load_expert,
                                int32_t* load_slot, int32_t* n_loads);
int mimo_moe_slot_cache_resolve(void* cache, const int32_t* needed, int32_t n, int32_t count, int32_t stats,
                                int32_t* load_expert, int32_t* load_slot, int32_t* n_loads);
int mimo_moe_slot_cache_decay(void* cache);
int mimo_moe_slot_cache_state(void* cache, int32_t* slot_of, int32_t* expert_in, int64_t* hits, int64_t* misses);

/*
 * Benchmark support (no counterpart in the reference).  mimo_moe_profile_enable(n) with n > 0 makes
 * the library record a CUDA event pair around each of the next n expert-path kernel launches on the
 * launching stream (the events are created here, once); n = 0 turns it off.  mimo_moe_profile_read()
 * synchronises those events and returns, per kernel kind (0 decode gate/up, 1 decode down, 2 prefill
 * gate/up, 3 prefill down, 4 decode gate/up + down in one launch, 5 the same as one stream-K launch,
 * 6 the decode route kernel of mimo_moe_block, 7 the decode combine; MIMO_MOE_PROFILE_KINDS entries in
 * each array), the launch count and the summed device milliseconds, then resets.
 * Off by default; do not enable it while a stream is being captured.
 */
#define MIMO_MOE_PROFILE_KINDS 8
int mimo_moe_profile_enable(int32_t capacity);
int mimo_moe_profile_read(int32_t* launches, float* milliseconds);

#ifdef __cplusplus
}
#endif
#endif /* MIMO_MOE_H */
