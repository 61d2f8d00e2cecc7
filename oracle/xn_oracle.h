/*
 * xn_oracle.h - CPU restatement of the reference CPU backend for the fused
 * layer-op path (mimi-rs/src/cpu_backend.rs of LaurentMazare/random-things).
 *
 * TEST INFRASTRUCTURE ONLY. This is the parity checker and the timed CPU
 * baseline. Nothing in the product library links, loads or calls it; only
 * tests/, __graft_entry__.smoke() and bench.py (cpu_baseline and
 * --impl reference) use it.
 *
 * Pinning: the restatement is checked against every known-answer test the
 * reference holds for these ops (mimi-rs/tests/cuda_tests.rs and
 * tests/tensor_tests.rs; fixtures in tests/golden/known_answers.json).
 *
 * dtype codes follow xn_fused.h: 0 = f16, 1 = bf16, 2 = f32. Every op is
 * written once per dtype; "T arithmetic" means each +,-,*,/,exp of two T
 * values is done in f32 and rounded to T (round-to-nearest-even), which is
 * what the `half` 2.7.1 crate does for bf16/f16 arithmetic.
 */
#ifndef XN_ORACLE_H
#define XN_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

void xo_set_num_threads(int n);
int xo_get_num_threads(void);

/* Scalar conversions exposed for the tests. */
uint16_t xo_f32_to_bf16(float f);
float xo_bf16_to_f32(uint16_t h);
uint16_t xo_f32_to_f16(float f);
float xo_f16_to_f32(uint16_t h);

/* cpu_backend.rs:691-709 */
void xo_rms_norm(int dtype, void *dst, const void *src, const void *alpha,
                 int64_t dim_m1, int64_t d, float eps);
/* cpu_backend.rs:711-750 */
void xo_layer_norm(int dtype, void *dst, const void *src, const void *weight,
                   const void *bias, int64_t dim_m1, int64_t d, float eps,
                   int remove_mean);
/* Batched matmul (cpu_backend.rs:45-88, 425-540, the gemm crate): lhs
 * [batch, m, k] times rhs [batch, k, n] (trans_rhs = 0) or the transpose of
 * rhs [batch, n, k] (trans_rhs = 1, matmul_t); f32 accumulation, sequential
 * in k with FMA, result rounded to T. */
void xo_matmul(int dtype, void *dst, const void *lhs, const void *rhs, int64_t batch,
               int64_t m, int64_t n, int64_t k, int trans_rhs);
/* cpu_backend.rs:667-689 */
void xo_softmax(int dtype, void *dst, const void *src, int64_t dim_m1, int64_t d);
/* cpu_backend.rs:647-665 */
void xo_apply_causality_mask(int dtype, void *dst, int64_t bh, int64_t t1,
                             int64_t t2, int64_t offset);
/* cpu_backend.rs:359-392 */
void xo_rope(int dtype, void *dst, const void *src, const void *cos,
             const void *sin, int64_t b, int64_t h, int64_t t, int64_t d,
             int64_t pos);
/* cpu_backend.rs:394-422 */
void xo_rope_i(int dtype, void *dst, const void *src, const void *cos,
               const void *sin, int64_t b, int64_t h, int64_t t, int64_t d,
               int64_t pos);
/* cpu_backend.rs:184-222; op 0 = Silu, 1 = GeluErf, 2 = T(exp(x)) (the softmax step, :681) */
void xo_unary(int dtype, void *dst, const void *src, int64_t len, int op);
/* cpu_backend.rs:224-258; op 0 = Add, 1 = Sub, 2 = Mul, 3 = Div */
void xo_binary(int dtype, void *dst, const void *lhs, const void *rhs,
               int64_t len, int op);
/* cpu_backend.rs:1379-1387 (broadcast_binary with rhs_strides == [0, 1]);
 * op codes as xo_binary. */
void xo_broadcast_binary_rows(int dtype, void *dst, const void *lhs,
                              const void *rhs, int64_t rows, int64_t cols,
                              int op);
/* cpu_backend.rs:624-645; a byte copy, so any element size works. */
void xo_index_select(int64_t elem_bytes, void *dst, const void *src,
                     const uint32_t *ids, int64_t n_ids, int64_t left,
                     int64_t src_dim, int64_t right);
/* mimi-rs/src/models/mimi.rs:1162-1185 (variant 0) and
 * mimi-rs/src/models/llama.rs:406-434 (variant 1): cos/sin [max_pos, d/2]. */
void xo_rope_tables(int dtype, void *cos, void *sin, int64_t head_dim,
                    int64_t max_pos, float theta, int variant);

#ifdef __cplusplus
}
#endif

#endif /* XN_ORACLE_H */
