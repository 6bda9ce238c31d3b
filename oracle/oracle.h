/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the jax4j B200 engine.
 *
 * A plain-C restatement of the reference's jax4j-core CPU path (Java). Only tests/, the
 * smoke() check and bench.py's cpu_baseline / --impl reference legs may load it, and only as a
 * checker or as the timed CPU baseline; the engine never calls it.
 *
 * Java float semantics are kept: every float op rounds to binary32, no FMA contraction (build
 * with -ffp-contract=off), transcendentals are evaluated in double and cast to float, and full
 * and axis sums accumulate in double exactly as CpuBackend does.
 *
 * Parity status:
 *   - PRNG, Q4_0, Q2_0, halfToFloat, elementwise/reduction/matmul primitives and Adam are
 *     restatements of reference source (file:line cited per function) and are pinned by the
 *     reference's JAX fixtures (jax-parity.properties) and known-answer tests.
 *   - Q8_0 and Q4_K have no implementation in the reference (QuantType.java:8-9 holds only
 *     their geometry). Their codecs follow the public GGUF block layouts; parity for them is
 *     "unpinned" against the reference and defined by this oracle.
 */
#ifndef JAX4J_ORACLE_H
#define JAX4J_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- PRNG: ComputeBackend.java:51-76, 282-295; PrngKey.java:44-56 ---- */
uint64_t j4o_mix64(uint64_t v);
void j4o_random_uniform(int64_t seed, int64_t counter, int64_t n, float* out);
void j4o_random_normal(int64_t seed, int64_t counter, int64_t n, float* out);
/* PrngKey.split(count): writes count (seed, counter=0) keys as seeds. */
void j4o_prng_split(int64_t seed, int64_t counter, int count, int64_t* seeds_out);

/* ---- half precision: CpuQ4Gemm.java:58-77 (decode); RNE encode (ours) ---- */
float j4o_half_to_float(uint32_t bits);
uint16_t j4o_float_to_half(float f);

/* ---- GGUF block codecs. type ids follow QuantType.java:4-13 ---- */
enum { J4O_Q4_0 = 2, J4O_Q8_0 = 8, J4O_Q4_K = 12, J4O_Q6_K = 14, J4O_Q2_0 = 42 };
int64_t j4o_quant_row_bytes(int type, int64_t cols);
/* Encode rows x cols f32 (row-major) into GGUF blocks. Returns 0 or -1 on bad geometry. */
int j4o_quantize(int type, const float* w, int64_t rows, int64_t cols, uint8_t* out);
/* quantGatherRow: CpuBackend.java:738-755 / CpuQ4Gemm.gather. Bit-exact dequantised row. */
int j4o_gather_row(int type, const uint8_t* blob, int64_t rows, int64_t cols, int64_t row,
                   float* out);
/* quantMatvec: CpuBackend.java:707-725, float-sequential accumulation per row, batch rows of
 * x processed one after the other (each is the reference's rank-1 call). y is [batch, rows]. */
int j4o_quant_matvec(int type, const uint8_t* blob, int64_t rows, int64_t cols,
                     const float* x, int64_t batch, float* y);
/* Same product evaluated in double from the dequantised weights (the exact answer used for
 * tolerance checks of the GPU tensor-core path). */
int j4o_quant_matvec_f64(int type, const uint8_t* blob, int64_t rows, int64_t cols,
                         const float* x, int64_t batch, double* y);

/* ---- CpuBackend primitives (CpuBackend.java:61-686) ---- */
/* op codes follow Op.java:19-23 ordinal order */
enum {
  J4O_ADD = 0, J4O_SUB, J4O_MUL, J4O_DIV, J4O_MAX, J4O_MIN,
  J4O_NEG, J4O_EXP, J4O_LOG, J4O_SQRT, J4O_RSQRT, J4O_TANH, J4O_SIGMOID, J4O_RELU,
  J4O_ABS, J4O_SIGN
};
float j4o_apply_binary(int op, float x, float y);
float j4o_apply_unary(int op, float x);
void j4o_binary(int op, const float* a, const float* b, int64_t n, float* out);
void j4o_scalar(int op, const float* a, double value, int64_t n, float* out);
void j4o_unary(int op, const float* a, int64_t n, float* out);
void j4o_transpose(const float* a, int64_t rows, int64_t cols, float* out);
void j4o_matmul(const float* a, const float* b, int64_t m, int64_t k, int64_t n, float* out);
void j4o_batched_matmul(const float* a, const float* b, int64_t batch, int64_t m, int64_t k,
                        int64_t n, float* out);
float j4o_reduce_sum(const float* a, int64_t n);
float j4o_reduce_max(const float* a, int64_t n);
void j4o_sum_axis(const float* a, int64_t outer, int64_t axis, int64_t inner, float* out);
void j4o_max_axis(const float* a, int64_t outer, int64_t axis, int64_t inner, float* out);
void j4o_argmax_axis(const float* a, int64_t outer, int64_t axis, int64_t inner, float* out);
void j4o_max_axis_backward(const float* up, const float* in, int64_t outer, int64_t axis,
                           int64_t inner, float* out);
/* broadcastTo (CpuBackend.java:401-447): src dims right-aligned against target dims. */
void j4o_broadcast_to(const float* a, const int64_t* src_dims, int src_rank,
                      const int64_t* dst_dims, int dst_rank, float* out);
/* reindex / scatterAdd (ComputeBackend.java:247-274); -1 means zero / discard. */
int j4o_reindex(const float* a, int64_t n_src, const int32_t* map, int64_t n_dst, float* out);
int j4o_scatter_add(const float* a, int64_t n_src, const int32_t* map, int64_t n_dst,
                    float* out);
void j4o_relu_backward(const float* up, const float* in, int64_t n, float* out);

/* fused(Expr): CpuBackend.java:628-682. The expression is a postfix program of int32 words:
 *   [0, input_index] | [1, op] (unary, pops 1) | [2, op] (binary, pops 2) |
 *   [3, op, lo32, hi32] (scalar with a double immediate, pops 1).
 * Evaluation follows the reference: unary/binary/scalar applied per element in float. */
int j4o_fused(const int32_t* prog, int prog_len, const float* const* inputs, int n_inputs,
              int64_t n, float* out);

/* Scalar-AAD Monte-Carlo replay (core/engine/cpu/ScalarReplay.java:145-232, Philox.java:30-94):
 * paths [path_from, path_from + count) of a tape of n nodes (op codes = AadOp ordinals; RANDN /
 * RANDU: arg_a = ordinal, arg_b = stream). Fills per output o: value[o] = sum of y, sumsq[o] =
 * sum of y^2, grad[o * n_in + j] = sum of dy/d input j (when adjoints). Returns 0 on success. */
int j4o_aad_replay(int n, const int32_t* op, const int32_t* arg_a, const int32_t* arg_b,
                   const double* constant, const double* inputs, int n_in, const int32_t* in_nodes,
                   int n_out, const int32_t* out_nodes, int n_streams, int adjoints, int64_t path_from,
                   int64_t count, int64_t seed, double* value, double* sumsq, double* grad);
void j4o_philox2x32_10(uint32_t c0, uint32_t c1, uint32_t key, uint32_t* out0, uint32_t* out1);

/* conv2d / conv2dGradInput / conv2dGradWeight (CpuBackend.java:479-609); ConvSpec as ints.
 * Return -1 for a spec ConvSpec rejects. */
int j4o_conv2d(const float* x, const float* w, int64_t batch, int in_c, int in_h, int in_w, int out_c, int kernel,
               int stride, int pad, float* out);
int j4o_conv2d_grad_input(const float* up, const float* w, int64_t batch, int in_c, int in_h, int in_w, int out_c,
                          int kernel, int stride, int pad, float* dx);
int j4o_conv2d_grad_weight(const float* x, const float* up, int64_t batch, int in_c, int in_h, int in_w, int out_c,
                           int kernel, int stride, int pad, float* dw);

#ifdef __cplusplus
}
#endif
#endif
