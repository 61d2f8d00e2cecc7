/*
 * xn_oracle.c - CPU restatement of mimi-rs/src/cpu_backend.rs (the `xn`
 * reference CPU backend) for the fused layer-op path.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline.
 * The product library never links or calls this file.
 *
 * Fidelity rules (each one mirrors how the reference Rust code evaluates):
 *   - Per-row reductions are sequential left folds in f32 starting at -0.0,
 *     as `Iterator::sum::<f32>()` is (no reassociation, no vectorised sum).
 *   - No fused multiply-add: the file is compiled with -ffp-contract=off,
 *     as rustc never contracts a*b+c.
 *   - T arithmetic (bf16/f16) is f32 arithmetic rounded to T after each op,
 *     which is how the `half` 2.7.1 crate implements Add/Sub/Mul/Div and
 *     num_traits::Float::exp for bf16 and f16.
 *   - Row-parallel ops (rayon `par_chunks` in the reference) are OpenMP
 *     parallel over rows; unary/binary ops are single-threaded loops, as
 *     `apply_unary` / `apply_binary` are (cpu_backend.rs:1088-1106).
 *   - expf/sinf/cosf/powf/sqrtf come from the C library, like Rust's f32
 *     methods on Linux. `libm` 0.2.16's erff (a port of musl's erff, the
 *     Sun/FreeBSD rational approximation) is not available here; glibc's
 *     erff stands in for it. Both are accurate to about 1 ulp of f32.
 */
#include "xn_oracle.h"

#include <math.h>
#include <string.h>
#include <omp.h>

/* ---------------------------------------------------------------------------
 * Scalar conversions.
 * bf16 from f32 is round-to-nearest-even on the bit pattern; NaN keeps its
 * sign and top payload bits and is made quiet (half 2.7.1 bf16::from_f32).
 * ------------------------------------------------------------------------- */
uint16_t xo_f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
  uint32_t lsb = (u >> 16) & 1u;
  return (uint16_t)((u + 0x7fffu + lsb) >> 16);
}

float xo_bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

uint16_t xo_f32_to_f16(float f) {
  _Float16 x = (_Float16)f; /* IEEE conversion, round to nearest even */
  uint16_t h;
  memcpy(&h, &x, 2);
  return h;
}

float xo_f16_to_f32(uint16_t h) {
  _Float16 x;
  memcpy(&x, &h, 2);
  return (float)x;
}

void xo_set_num_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}

int xo_get_num_threads(void) { return omp_get_max_threads(); }

#define F32_TO(x) (x)
#define F32_FROM(x) (x)
#define BF16_TO(x) xo_bf16_to_f32(x)
#define BF16_FROM(x) xo_f32_to_bf16(x)
#define F16_TO(x) xo_f16_to_f32(x)
#define F16_FROM(x) xo_f32_to_f16(x)

/* FRAC_1_SQRT_2 as f32 (std::f32::consts::FRAC_1_SQRT_2). */
static const float kFrac1Sqrt2 = (float)0.707106781186547524400844362104849039;

/*
 * One instantiation of every op for storage type ST with conversions TO/FROM.
 * `TB(expr)` rounds an f32 value to T and back, i.e. one T-typed result.
 */
#define XO_DEFINE(SUF, ST, TO, FROM)                                                   \
  static inline float tb_##SUF(float v) { return TO(FROM(v)); }                        \
                                                                                       \
  /* cpu_backend.rs:691-709 */                                                         \
  static void rms_norm_##SUF(ST *dst, const ST *src, const ST *alpha, int64_t dim_m1,  \
                             int64_t d, float eps) {                                   \
    _Pragma("omp parallel for schedule(static)") for (int64_t r = 0; r < d; r++) {     \
      const ST *s = src + r * dim_m1;                                                  \
      ST *o = dst + r * dim_m1;                                                        \
      float sum2 = -0.0f;                                                              \
      for (int64_t i = 0; i < dim_m1; i++) {                                           \
        float v = TO(s[i]);                                                            \
        sum2 = sum2 + v * v;                                                           \
      }                                                                                \
      float m = sqrtf(sum2 / (float)dim_m1 + eps);                                     \
      for (int64_t i = 0; i < dim_m1; i++) o[i] = FROM(TO(s[i]) / m * TO(alpha[i]));   \
    }                                                                                  \
  }                                                                                    \
                                                                                       \
  /* cpu_backend.rs:711-750 */                                                         \
  static void layer_norm_##SUF(ST *dst, const ST *src, const ST *w, const ST *b,       \
                               int64_t dim_m1, int64_t d, float eps, int remove_mean) { \
    _Pragma("omp parallel for schedule(static)") for (int64_t r = 0; r < d; r++) {     \
      const ST *s = src + r * dim_m1;                                                  \
      ST *o = dst + r * dim_m1;                                                        \
      float sum = -0.0f;                                                               \
      for (int64_t i = 0; i < dim_m1; i++) sum = sum + TO(s[i]);                       \
      float mean = sum / (float)dim_m1;                                                \
      float var = -0.0f;                                                               \
      for (int64_t i = 0; i < dim_m1; i++) {                                           \
        float diff = TO(s[i]) - mean;                                                  \
        var = var + diff * diff;                                                       \
      }                                                                                \
      var = var / (float)dim_m1;                                                       \
      float inv_std = 1.0f / sqrtf(var + eps);                                         \
      for (int64_t i = 0; i < dim_m1; i++) {                                           \
        float centered = remove_mean ? TO(s[i]) - mean : TO(s[i]);                     \
        float normalized = centered * inv_std;                                         \
        o[i] = FROM(normalized * TO(w[i]) + TO(b[i]));                                 \
      }                                                                                \
    }                                                                                  \
  }                                                                                    \
                                                                                       \
  /* cpu_backend.rs:667-689 */                                                         \
  static void softmax_##SUF(ST *dst, const ST *src, int64_t dim_m1, int64_t d) {       \
    _Pragma("omp parallel for schedule(static)") for (int64_t r = 0; r < d; r++) {     \
      const ST *s = src + r * dim_m1;                                                  \
      ST *o = dst + r * dim_m1;                                                        \
      float mx = -INFINITY;                                                            \
      for (int64_t i = 0; i < dim_m1; i++) mx = fmaxf(TO(s[i]), mx);                   \
      for (int64_t i = 0; i < dim_m1; i++) o[i] = FROM(expf(tb_##SUF(TO(s[i]) - mx))); \
      float sum_exp = -0.0f;                                                           \
      for (int64_t i = 0; i < dim_m1; i++) sum_exp = sum_exp + TO(o[i]);               \
      for (int64_t i = 0; i < dim_m1; i++) o[i] = FROM(TO(o[i]) / sum_exp);            \
    }                                                                                  \
  }                                                                                    \
                                                                                       \
  /* cpu_backend.rs:647-665 */                                                         \
  static void mask_##SUF(ST *dst, int64_t bh, int64_t t1, int64_t t2, int64_t off) {   \
    for (int64_t b = 0; b < bh; b++)                                                   \
      for (int64_t i1 = 0; i1 < t1; i1++)                                              \
        for (int64_t i2 = off + i1 + 1; i2 < t2; i2++)                                 \
          dst[b * t1 * t2 + i1 * t2 + i2] = FROM(-INFINITY);                           \
  }                                                                                    \
                                                                                       \
  /* cpu_backend.rs:359-392: T arithmetic, each product and sum rounded to T */        \
  static void rope_##SUF(ST *dst, const ST *src, const ST *cos_, const ST *sin_,       \
                         int64_t b, int64_t h, int64_t t, int64_t d, int64_t pos) {    \
    const ST *cs = cos_ + pos * d / 2;                                                 \
    const ST *sn = sin_ + pos * d / 2;                                                 \
    _Pragma("omp parallel for schedule(static)") for (int64_t c = 0; c < b * h; c++) { \
      const ST *s = src + c * t * d;                                                   \
      ST *o = dst + c * t * d;                                                         \
      for (int64_t it = 0; it < t; it++) {                                             \
        for (int64_t id = 0; id < d / 2; id++) {                                       \
          int64_t i1 = it * d + id, i2 = i1 + d / 2, ics = it * (d / 2) + id;          \
          float x1 = TO(s[i1]), x2 = TO(s[i2]), cv = TO(cs[ics]), sv = TO(sn[ics]);    \
          o[i1] = FROM(tb_##SUF(x1 * cv) - tb_##SUF(x2 * sv));                         \
          o[i2] = FROM(tb_##SUF(x1 * sv) + tb_##SUF(x2 * cv));                         \
        }                                                                              \
      }                                                                                \
    }                                                                                  \
  }                                                                                    \
                                                                                       \
  /* cpu_backend.rs:394-422 */                                                         \
  static void rope_i_##SUF(ST *dst, const ST *src, const ST *cos_, const ST *sin_,     \
                           int64_t b, int64_t h, int64_t t, int64_t d, int64_t pos) {  \
    const ST *cs = cos_ + pos * d / 2;                                                 \
    const ST *sn = sin_ + pos * d / 2;                                                 \
    _Pragma("omp parallel for schedule(static)") for (int64_t c = 0; c < b * h; c++) { \
      const ST *s = src + c * t * d;                                                   \
      ST *o = dst + c * t * d;                                                         \
      for (int64_t j = 0; j < t * d / 2; j++) {                                        \
        float x1 = TO(s[2 * j]), x2 = TO(s[2 * j + 1]), cv = TO(cs[j]), sv = TO(sn[j]); \
        o[2 * j] = FROM(tb_##SUF(x1 * cv) - tb_##SUF(x2 * sv));                        \
        o[2 * j + 1] = FROM(tb_##SUF(x1 * sv) + tb_##SUF(x2 * cv));                    \
      }                                                                                \
    }                                                                                  \
  }                                                                                    \
                                                                                       \
  /* cpu_backend.rs:197-204 (GeluErf), :213-215 (Silu) and the exp of one element   \
     of the softmax, :681 ((s - max).exp() on T: exp in f32, rounded to T) */          \
  static void unary_##SUF(ST *dst, const ST *src, int64_t len, int op) {               \
    if (op == 2) {                                                                     \
      for (int64_t i = 0; i < len; i++) dst[i] = FROM(expf(TO(src[i])));               \
    } else if (op == 0) {                                                              \
      for (int64_t i = 0; i < len; i++) {                                              \
        float s = TO(src[i]);                                                          \
        float e = tb_##SUF(expf(tb_##SUF(0.0f - s)));                                  \
        dst[i] = FROM(s / tb_##SUF(1.0f + e));                                         \
      }                                                                                \
    } else {                                                                           \
      for (int64_t i = 0; i < len; i++) {                                              \
        float x = TO(src[i]);                                                          \
        float erf_val = erff(x * kFrac1Sqrt2);                                         \
        dst[i] = FROM(x * 0.5f * (1.0f + erf_val));                                    \
      }                                                                                \
    }                                                                                  \
  }                                                                                    \
                                                                                       \
  static inline float binop_##SUF(float a, float b, int op) {                          \
    switch (op) {                                                                      \
      case 0: return a + b;                                                            \
      case 1: return a - b;                                                            \
      case 2: return a * b;                                                            \
      default: return a / b;                                                           \
    }                                                                                  \
  }                                                                                    \
                                                                                       \
  /* cpu_backend.rs:224-258 */                                                         \
  static void binary_##SUF(ST *dst, const ST *l, const ST *r, int64_t len, int op) {   \
    for (int64_t i = 0; i < len; i++) dst[i] = FROM(binop_##SUF(TO(l[i]), TO(r[i]), op)); \
  }                                                                                    \
                                                                                       \
  /* cpu_backend.rs:1379-1387 */                                                       \
  static void bcast_rows_##SUF(ST *dst, const ST *l, const ST *r, int64_t rows,        \
                               int64_t cols, int op) {                                 \
    for (int64_t i0 = 0; i0 < rows; i0++)                                              \
      for (int64_t i1 = 0; i1 < cols; i1++)                                            \
        dst[i0 * cols + i1] = FROM(binop_##SUF(TO(l[i0 * cols + i1]), TO(r[i1]), op)); \
  }                                                                                    \
                                                                                       \
  /* mimi.rs:1162-1185 (variant 0: i / half_dim), llama.rs:406-434 (variant 1) */      \
  static void tables_##SUF(ST *cos_, ST *sin_, int64_t head_dim, int64_t max_pos,      \
                           float theta, int variant) {                                 \
    int64_t half = head_dim / 2;                                                       \
    for (int64_t p = 0; p < max_pos; p++) {                                            \
      for (int64_t i = 0; i < half; i++) {                                             \
        float freq = variant == 0 ? 1.0f / powf(theta, (float)i / (float)half)         \
                                  : 1.0f / powf(theta, 2.0f * (float)i / (float)head_dim); \
        float angle = (float)p * freq;                                                 \
        cos_[p * half + i] = FROM(cosf(angle));                                        \
        sin_[p * half + i] = FROM(sinf(angle));                                        \
      }                                                                                \
    }                                                                                  \
  }

/* Batched matmul with the reference's gemm contract (cpu_backend.rs:45-88,
 * 425-540): T inputs widened to f32, products accumulated in f32, the sum
 * rounded to T once. The gemm crate's blocked summation order is not
 * reproducible outside it; here the accumulation is sequential in k with
 * fused multiply-adds (its x86-64 microkernels use FMA). */
#define XO_DEFINE_MATMUL(SUF, ST, TO, FROM)                                            \
  static void matmul_##SUF(ST *dst, const ST *lhs, const ST *rhs, int64_t batch,       \
                           int64_t m, int64_t n, int64_t k, int trans_rhs) {           \
    _Pragma("omp parallel for schedule(static)") for (int64_t bm = 0; bm < batch * m; bm++) { \
      const int64_t bi = bm / m;                                                       \
      const ST *a = lhs + bm * k;                                                      \
      const ST *bb = rhs + bi * n * k;                                                 \
      for (int64_t j = 0; j < n; j++) {                                                \
        float acc = 0.0f;                                                              \
        for (int64_t x = 0; x < k; x++) {                                              \
          const float rv = trans_rhs ? TO(bb[j * k + x]) : TO(bb[x * n + j]);          \
          acc = fmaf(TO(a[x]), rv, acc);                                               \
        }                                                                              \
        dst[bm * n + j] = FROM(acc);                                                   \
      }                                                                                \
    }                                                                                  \
  }

XO_DEFINE_MATMUL(f32, float, F32_TO, F32_FROM)
XO_DEFINE_MATMUL(bf16, uint16_t, BF16_TO, BF16_FROM)
XO_DEFINE_MATMUL(f16, uint16_t, F16_TO, F16_FROM)

XO_DEFINE(f32, float, F32_TO, F32_FROM)
XO_DEFINE(bf16, uint16_t, BF16_TO, BF16_FROM)
XO_DEFINE(f16, uint16_t, F16_TO, F16_FROM)

#define XO_DISPATCH(DT, CALL_F16, CALL_BF16, CALL_F32) \
  do {                                                \
    switch (DT) {                                     \
      case 0: CALL_F16; break;                        \
      case 1: CALL_BF16; break;                       \
      default: CALL_F32; break;                       \
    }                                                 \
  } while (0)

void xo_rms_norm(int dt, void *dst, const void *src, const void *alpha, int64_t dim_m1,
                 int64_t d, float eps) {
  XO_DISPATCH(dt, rms_norm_f16(dst, src, alpha, dim_m1, d, eps),
              rms_norm_bf16(dst, src, alpha, dim_m1, d, eps),
              rms_norm_f32(dst, src, alpha, dim_m1, d, eps));
}

void xo_layer_norm(int dt, void *dst, const void *src, const void *w, const void *b,
                   int64_t dim_m1, int64_t d, float eps, int remove_mean) {
  XO_DISPATCH(dt, layer_norm_f16(dst, src, w, b, dim_m1, d, eps, remove_mean),
              layer_norm_bf16(dst, src, w, b, dim_m1, d, eps, remove_mean),
              layer_norm_f32(dst, src, w, b, dim_m1, d, eps, remove_mean));
}

void xo_matmul(int dt, void *dst, const void *lhs, const void *rhs, int64_t batch, int64_t m,
               int64_t n, int64_t k, int trans_rhs) {
  XO_DISPATCH(dt, matmul_f16(dst, lhs, rhs, batch, m, n, k, trans_rhs),
              matmul_bf16(dst, lhs, rhs, batch, m, n, k, trans_rhs),
              matmul_f32(dst, lhs, rhs, batch, m, n, k, trans_rhs));
}

void xo_softmax(int dt, void *dst, const void *src, int64_t dim_m1, int64_t d) {
  XO_DISPATCH(dt, softmax_f16(dst, src, dim_m1, d), softmax_bf16(dst, src, dim_m1, d),
              softmax_f32(dst, src, dim_m1, d));
}

void xo_apply_causality_mask(int dt, void *dst, int64_t bh, int64_t t1, int64_t t2,
                             int64_t offset) {
  XO_DISPATCH(dt, mask_f16(dst, bh, t1, t2, offset), mask_bf16(dst, bh, t1, t2, offset),
              mask_f32(dst, bh, t1, t2, offset));
}

void xo_rope(int dt, void *dst, const void *src, const void *c, const void *s, int64_t b,
             int64_t h, int64_t t, int64_t d, int64_t pos) {
  XO_DISPATCH(dt, rope_f16(dst, src, c, s, b, h, t, d, pos),
              rope_bf16(dst, src, c, s, b, h, t, d, pos),
              rope_f32(dst, src, c, s, b, h, t, d, pos));
}

void xo_rope_i(int dt, void *dst, const void *src, const void *c, const void *s, int64_t b,
               int64_t h, int64_t t, int64_t d, int64_t pos) {
  XO_DISPATCH(dt, rope_i_f16(dst, src, c, s, b, h, t, d, pos),
              rope_i_bf16(dst, src, c, s, b, h, t, d, pos),
              rope_i_f32(dst, src, c, s, b, h, t, d, pos));
}

void xo_unary(int dt, void *dst, const void *src, int64_t len, int op) {
  XO_DISPATCH(dt, unary_f16(dst, src, len, op), unary_bf16(dst, src, len, op),
              unary_f32(dst, src, len, op));
}

void xo_binary(int dt, void *dst, const void *l, const void *r, int64_t len, int op) {
  XO_DISPATCH(dt, binary_f16(dst, l, r, len, op), binary_bf16(dst, l, r, len, op),
              binary_f32(dst, l, r, len, op));
}

void xo_broadcast_binary_rows(int dt, void *dst, const void *l, const void *r, int64_t rows,
                              int64_t cols, int op) {
  XO_DISPATCH(dt, bcast_rows_f16(dst, l, r, rows, cols, op),
              bcast_rows_bf16(dst, l, r, rows, cols, op),
              bcast_rows_f32(dst, l, r, rows, cols, op));
}

void xo_rope_tables(int dt, void *c, void *s, int64_t head_dim, int64_t max_pos, float theta,
                    int variant) {
  XO_DISPATCH(dt, tables_f16(c, s, head_dim, max_pos, theta, variant),
              tables_bf16(c, s, head_dim, max_pos, theta, variant),
              tables_f32(c, s, head_dim, max_pos, theta, variant));
}

/* cpu_backend.rs:624-645: for each left slice, copy the selected rows. */
void xo_index_select(int64_t elem_bytes, void *dst, const void *src, const uint32_t *ids,
                     int64_t n_ids, int64_t left, int64_t src_dim, int64_t right) {
  const int64_t rb = right * elem_bytes;
  for (int64_t l = 0; l < left; l++) {
    for (int64_t i = 0; i < n_ids; i++) {
      const int64_t src_off = l * src_dim * rb + (int64_t)ids[i] * rb;
      const int64_t dst_off = l * n_ids * rb + i * rb;
      memcpy((char *)dst + dst_off, (const char *)src + src_off, (size_t)rb);
    }
  }
}
