/*
 * mimo_moe_testkit.h - C ABI of libmimo_moe_testkit.so, the test and benchmark kit that ships beside
 * the MoE block library (include/mimo_moe.h; error codes as there).  Not part of the block's path.
 */
#ifndef MIMO_MOE_TESTKIT_H
#define MIMO_MOE_TESTKIT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/*
 * Synthetic pool fill (benchmarks and tests): counter-based splitmix64 stream per (seed, layer, tensor);
 * experts [first_expert, first_expert + S) of the layer are written to slots [0, S).  Nibbles uniform
 * over the 16 e2m1 codes; scale bytes 120 with p = 0.6875, else 119.
 */
int mimo_moe_fill_synthetic_pool(uint32_t* gate_w, uint8_t* gate_s, uint32_t* up_w, uint8_t* up_s,
                                 uint32_t* down_w, uint8_t* down_s, int32_t S, int32_t H, int32_t I,
                                 uint64_t seed, int32_t layer, int32_t first_expert, void* stream);

/*
 * Benchmark support (no counterpart in the reference).  Measures this GPU's dense block-scaled tensor
 * peak for an MMA form the expert kernels use: kind 0 = tcgen05.mma.kind::mxf8f6f4 (e2m1 weights x
 * e4m3 activations, the expert kernels' form), kind 1 = kind::mxf4 (e2m1 x e2m1, the FP4 rate).  One
 * CTA per SM issues `iters` x (M 128, N 256, K 128) MMAs on operands held in shared memory; the launch
 * is timed with CUDA events on `stream` and synchronised.  *tflops receives 2*M*N*K*iters*SMs / time.
 * status: device int32 word (MIMO_ETIMEOUT if the final wait expired).
 */
int mimo_moe_tensor_peak(int32_t kind, int32_t iters, float* tflops, int32_t* status, void* stream);

#ifdef __cplusplus
}
#endif
#endif  /* MIMO_MOE_TESTKIT_H */
