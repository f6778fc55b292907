/*
 * mimo_moe_layer.h — C ABI of the rest of the MiMo decoder layer around the MoE block (same library,
 * libmimo_moe.so; error codes and conventions of mimo_moe.h).
 *
 * The decoder layer (engine/mimo_stream/mimo_v2.py:242-262, the engine's loop engine/mimo_stream/model.py:294-300):
 *   r   = input_layernorm(x)                          mimo_moe_rmsnorm (mimo_moe.h)
 *   qkv = r @ [Wq | Wk | Wv]^T                        mimo_moe_layer_linear (decode) / caller's GEMM     :117-128
 *   q,k = RoPE, v *= value scale, k/v -> cache        mimo_moe_layer_rope_store       mimo_v2.py:130-139
 *   o   = attention with sinks over the cache         mimo_moe_layer_attention        mimo_v2.py:141-148
 *   h   = x + o @ Wo^T; r2 = post_attention_layernorm(h)
 *                                                     caller's GEMM + mimo_moe_layer_add_rmsnorm
 *   y   = MoE block (mimo_moe_block) or dense MLP: down(swiglu(gate(r2), up(r2)))
 *                                                     caller's GEMMs + mimo_moe_layer_swiglu  mimo_v2.py:151-160
 *   out = h + y                                       mimo_moe_layer_add                mimo_v2.py:261
 *
 * Every pointer is a device pointer, 16-byte aligned; bf16 values are passed as uint16_t bit patterns;
 * nothing here allocates, synchronises the host or changes the current device.
 *
 * KV cache layout: k_cache bf16 [n_kv_heads][cap][head_dim], v_cache bf16 [n_kv_heads][cap][v_head_dim];
 * the token at absolute position p lives in slot p % cap.  A full-attention layer uses cap >= the longest
 * sequence (slot = position); a sliding-window layer uses a ring with cap >= window + T - 1 for every call
 * of T tokens (the window of the chunk's first query and the chunk itself must both be resident).
 */
#ifndef MIMO_MOE_LAYER_H
#define MIMO_MOE_LAYER_H

#include "mimo_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

/* RoPE + value scale + cache append (mimo_v2.py:130-139; mlx_lm nn.RoPE(rotary_dim, traditional=False,
 * base=rope_theta) with offset = pos0).  qkv: bf16 [T][n_heads*head_dim + n_kv_heads*head_dim +
 * n_kv_heads*v_head_dim], the q | k | v projection rows of T consecutive tokens at positions pos0..pos0+T-1.
 * For i < rotary_dim/2 the pair (x[i], x[i + rotary_dim/2]) of every q and k head is rotated by
 * (pos * rope_theta^(-2i/rotary_dim)); the other dims pass through.  v is multiplied by v_scale (a value
 * representable in bf16, as MLX casts the Python scale to the array's type) when v_scale > 0, else copied.
 * Outputs: q bf16 [T][n_heads][head_dim]; k and v of each token written to slot (pos % cap) of each kv head.
 * Needs T <= cap and rotary_dim <= 256. */
int mimo_moe_layer_rope_store(const uint16_t* qkv, int32_t T, int32_t n_heads, int32_t n_kv_heads,
                              int32_t head_dim, int32_t v_head_dim, int32_t rotary_dim, float rope_theta,
                              float v_scale, int32_t pos0, int32_t cap, uint16_t* q, uint16_t* k_cache,
                              uint16_t* v_cache, void* stream);

/* Workspace for mimo_moe_layer_attention with `splits` key splits (0 when splits <= 1). */
size_t mimo_moe_layer_attention_workspace_bytes(int32_t T, int32_t n_heads, int32_t v_head_dim, int32_t splits);

/* Attention of T query tokens at positions pos0..pos0+T-1 over the cache (mlx fast.scaled_dot_product_attention
 * with `sinks`, mimo_v2.py:141-148).  For query head h (kv head h / (n_heads / n_kv_heads)) at position p:
 *   out = sum_j softmax_j v_j,  softmax over { scale * q.k_j : keys j visible to p } plus, when sinks is not
 *   null, one extra logit sinks[h] with no value row;
 * key position j is visible when j <= p and, for window > 0, j > p - window.  q bf16 [T][n_heads][head_dim]
 * (after RoPE), out bf16 [T][n_heads][v_head_dim], sinks float32 [n_heads] or null.  (head_dim, v_head_dim)
 * in {(192,128), (128,128), (64,64)}.  splits: the number of key ranges each query tile is divided into
 * (decode: many keys, few queries; at most 64); 0 picks a split count that fills the GPU within the workspace given;
 * splits > 1 need mimo_moe_layer_attention_workspace_bytes(T, n_heads, v_head_dim, splits).  Needs every
 * visible position resident: (pos0 + T - 1) - first visible position + 1 <= cap.  Query tiles of 128 rows
 * (T * n_heads / n_kv_heads >= 256, no key split) run on the tcgen05 tensor cores when cap is a multiple of
 * 128 and 128 is a multiple of n_heads / n_kv_heads; cache slots a key block reads beyond the visible
 * positions must then hold finite values (a zero-initialised cache does).  status: optional caller-zeroed
 * device word, set to MIMO_ETIMEOUT if a bounded wait of that kernel expires. */
int mimo_moe_layer_attention(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                             const float* sinks, int32_t T, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                             int32_t v_head_dim, float scale, int32_t window, int32_t pos0, int32_t cap,
                             int32_t splits, uint16_t* out, void* workspace, size_t workspace_bytes, int32_t* status,
                             void* stream);

/* Decode-size projection (nn.Linear without bias on a few token rows: the q|k|v and o projections,
 * mimo_v2.py:117-149, and the dense MLP's, :151-160): y[T, N] = bf16(x[T, K] . W[N, K]^T), float32
 * accumulation.  x bf16 [T][K] with 1 <= T <= 16, W bf16 [N][K] (nn.Linear layout), y bf16 [T][N]; N a
 * multiple of 8, K a multiple of 64 and at least 256.  The weights stream once through the tcgen05 tensor
 * cores; the K dimension may be split over CTAs for balance, with float32 partials in the workspace
 * (mimo_moe_layer_linear_workspace_bytes; a smaller or null workspace splits less) added in a fixed order.
 * status: optional caller-zeroed device word (MIMO_ETIMEOUT if a bounded wait expires).  Prefill-sized
 * projections are plain GEMMs the caller runs on its library (cuBLAS). */
size_t mimo_moe_layer_linear_workspace_bytes(int32_t T, int32_t N, int32_t K);
int mimo_moe_layer_linear(const uint16_t* x, const uint16_t* w, int32_t T, int32_t N, int32_t K, uint16_t* y,
                          void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/* Residual add and the next RMSNorm in one pass (mimo_v2.py:260 then post_attention_layernorm):
 * h = bf16(x + delta); r = RMSNorm(h) * weight exactly as mimo_moe_rmsnorm computes it.  [T, H] bf16,
 * H a multiple of 8; weight bf16 [H] or null (unit weight). */
int mimo_moe_layer_add_rmsnorm(const uint16_t* x, const uint16_t* delta, const uint16_t* weight, int32_t T,
                               int32_t H, float eps, uint16_t* h, uint16_t* r, void* stream);

/* Dense MLP activation (mlx_lm swiglu, mimo_v2.py:160): gate_up bf16 [T][2*I] holding [gate | up] per row,
 * out bf16 [T][I] = bf16(bf16(g * bf16(sigmoid(g))) * u).  I a multiple of 8. */
int mimo_moe_layer_swiglu(const uint16_t* gate_up, int32_t T, int32_t I, uint16_t* out, void* stream);

/* out = bf16(a + b) over n bf16 values (n a multiple of 8); the decoder layer's residual adds. */
int mimo_moe_layer_add(const uint16_t* a, const uint16_t* b, int64_t n, uint16_t* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* MIMO_MOE_LAYER_H */
