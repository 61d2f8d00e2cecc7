// xn_act.cu - SiLU, GELU(erf) and fused SwiGLU, elementwise, for sm_100a.
//
// Reference semantics (mimi-rs/src/cpu_backend.rs):
//   Silu    :213-215  s / (1 + exp(0 - s))     every op in T arithmetic
//   GeluErf :197-204  T(x*0.5*(1+erf(x*FRAC_1_SQRT_2)))  in f32, one rounding
//   SwiGLU  = `gate.silu()` then `mul(up)` (mimi-rs/src/models/llama.rs:256-263)
//             = T(T(silu(g)) * u)
//
// Design: 16-byte vector loads/stores, U accesses per thread issued before any
// math so each thread keeps U*16 (or 2*U*16 for SwiGLU) bytes in flight.
#include <type_traits>

#include "xn_common.cuh"
#include "xn_internal.h"

namespace xn {
namespace {

// f32 value of std::f32::consts::FRAC_1_SQRT_2.
constexpr float kFrac1Sqrt2 = 0.707106781186547524400844362104849039f;

__device__ __forceinline__ float gelu_erf(float x) {
  const float erf_val = erff(__fmul_rn(x, kFrac1Sqrt2));
  return __fmul_rn(__fmul_rn(x, 0.5f), __fadd_rn(1.f, erf_val));
}

// bf16 pairs with native bf16x2 arithmetic. For +, - and * of two bf16
// values, one rounding of the exact result (the bf16x2 instructions) equals the
// reference's f32 operation followed by rounding to bf16, so every step below
// that is such an operation is the reference's step.
//
// e = T(exp(-s)): 2^(x log2 e) for x = -s with log2 e = kL2eHi + kL2eLo, where
// kL2eHi has 16 significant bits, so x * kL2eHi (x has 8) is exact; the low
// part enters as the factor 2^(x kL2eLo) = 1 + c, c to second order (|x
// kL2eLo| < 2^-9). The result carries the error of the hardware ex2 only.
// x is clamped to [-110, 100] first (exp(x) overflows to inf above 88.8 and
// rounds to 0 below -103.9, so no result changes; NaN passes through), which
// keeps c finite, and kL2eLo > 0 keeps c >= 0 where ex2 overflows (inf * c
// then stays inf). A result that would be subnormal is flushed: it only feeds
// T(1 + e) = 1.
//
// y = T(s / d) for bf16 s and d = T(1 + e): s * rcp.approx(d) is within 2^-20
// (relative) of s / d, also where the reciprocal is subnormal (d > 2^126, where
// it keeps 21 or more significant bits), and
// a quotient of two bf16 values is never within 2^-18 of a bf16 rounding
// midpoint (s = m * d with m a 9-bit odd significand would need the odd part of
// m * d, at least 257, to equal the odd part of s, at most 255), so it rounds
// to the IEEE quotient's bf16 value. d = inf gives s * 0, the IEEE s / inf.
//
// test_unary_bf16_exhaustive runs every finite bf16 input through this
// function against the oracle's glibc expf and IEEE division.
constexpr float kL2eHi = 0x1.7154p+0f;
constexpr float kL2eLo = 0x1.d94aep-18f;

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The same reciprocal without the handling of subnormal inputs and results,
// for arguments known to lie in [1, 3].
__device__ __forceinline__ float rcp_approx_ftz(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// T(s / d) for f16 values s and d >= 1 (SiLU's d = T(1 + e)), without the
// IEEE division routine. q0 = s * rcp(d), refined once with the exact
// remainder: q1 = q0 + (s - d q0) * rcp(d) is s / d rounded once to f32 (up
// to a term of the square of the reciprocal's error), so within 2^-24 of s / d
// relative. Over every finite f16 s and its d, a quotient that is not an f32
// value is at least 2^-22.78 (relative) from an f16 rounding midpoint, so q1
// rounds to the f16 value of the IEEE f32 quotient; an f32-exact quotient
// comes out exact. copysign restores the sign of zero quotients (s = -0).
// Where the remainder step meets an infinity (s = +inf, or d = inf) it gives
// NaN, and q0 is then the IEEE quotient (s / inf = -0 for finite s < 0, inf / 1,
// -inf / inf = NaN).
__device__ __forceinline__ float div_f16_by_d(float s, float d) {
  const float r = rcp_approx(d);
  const float q0 = __fmul_rn(s, r);
  const float rem = __fmaf_rn(-d, q0, s);
  const float q1 = copysignf(__fmaf_rn(rem, r, q0), q0);
  return isnan(q1) ? q0 : q1;
}

template <typename T>
__device__ __forceinline__ float silu_t(float s) {
  // (T::zero() - s).exp(), then T::one() + e, then s / (...), each rounded to T.
  const float e = Elem<T>::round(expf(Elem<T>::round(__fsub_rn(0.f, s))));
  const float d = Elem<T>::round(__fadd_rn(1.f, e));
  if constexpr (std::is_same_v<T, __half>) {
    return div_f16_by_d(s, d);
  } else {
    return __fdiv_rn(s, d);
  }
}

// silu_t<__half> on an element pair. e = T(exp(-s)): as for bf16 below,
// 2^(x log2 e) for x = -s, but with a 13-bit piece of log2 e (kL2eHi16), so
// that x * kL2eHi16 is exact for an f16 x (11 significant bits); the low part
// enters as the factor 1 + c to second order (|x kL2eLo16| < 2^-8.5 for
// |x| <= 40, so the third-order term is below 2^-29 relative). x is clamped to [-40, 40] first: exp(x) rounds to f16 0 below
// -17.4 and to inf above 11.09, so no result changes, and NaN passes through.
// The result carries the error of the hardware ex2 only;
// test_silu_f16_exhaustive runs every finite f16 input against glibc's expf.
// The f16 additions are f16x2 instructions: 1 + e in f32 is exact for
// e >= 2^-13 and below 1 + 2^-11 (which rounds to 1) otherwise, so its f16
// rounding is the f16x2 sum's. The division is div_f16_by_d on f32 pairs.
__device__ __forceinline__ __half2 silu_f16x2(__half2 s) {
  const __half2 xh = __hmin2_nan(__hmax2_nan(__hneg2(s), __float2half2_rn(-40.f)), __float2half2_rn(40.f));
  const float2 ef = exp_split_f16(__half22float2(xh));
  const __half2 e = __floats2half2_rn(ef.x, ef.y);
  const __half2 d = __hadd2(__float2half2_rn(1.f), e);
  const float2 sf = __half22float2(s), df = __half22float2(d);
  const float2 r = make_float2(rcp_approx(df.x), rcp_approx(df.y));
  const float2 q0 = __fmul2_rn(sf, r);
  const float2 rem = __ffma2_rn(make_float2(-df.x, -df.y), q0, sf);
  const float2 q1 = __ffma2_rn(rem, r, q0);
  const float y0 = copysignf(q1.x, q0.x), y1 = copysignf(q1.y, q0.y);
  return __floats2half2_rn(isnan(y0) ? q0.x : y0, isnan(y1) ? q0.y : y1);
}

__device__ __forceinline__ uint32_t h2_bits(__half2 v) { return *reinterpret_cast<uint32_t *>(&v); }
__device__ __forceinline__ __half2 bits_h2(uint32_t w) { return *reinterpret_cast<__half2 *>(&w); }

__device__ __forceinline__ uint4 silu_f16x8(uint4 v) {
  return make_uint4(h2_bits(silu_f16x2(bits_h2(v.x))), h2_bits(silu_f16x2(bits_h2(v.y))),
                    h2_bits(silu_f16x2(bits_h2(v.z))), h2_bits(silu_f16x2(bits_h2(v.w))));
}

// T(T(silu(g)) * u): a product of two f16 values is exact in f32, so the
// f16x2 multiply rounds as the reference's f32 product rounded to f16 does.
__device__ __forceinline__ uint4 swiglu_f16x8(uint4 g, uint4 u) {
  return make_uint4(h2_bits(__hmul2(silu_f16x2(bits_h2(g.x)), bits_h2(u.x))),
                    h2_bits(__hmul2(silu_f16x2(bits_h2(g.y)), bits_h2(u.y))),
                    h2_bits(__hmul2(silu_f16x2(bits_h2(g.z)), bits_h2(u.z))),
                    h2_bits(__hmul2(silu_f16x2(bits_h2(g.w)), bits_h2(u.w))));
}

__device__ __forceinline__ __nv_bfloat162 silu_bf16x2(__nv_bfloat162 s) {
  const __nv_bfloat162 xb = __hmin2_nan(__hmax2_nan(__hneg2(s), __float2bfloat162_rn(-110.f)),
                                        __float2bfloat162_rn(100.f));
  const float2 x = bf2_to_f2(*reinterpret_cast<const uint32_t *>(&xb));
  const float2 th = __fmul2_rn(x, splat2(kL2eHi));
  const float2 tl = __fmul2_rn(x, splat2(kL2eLo));
  const float2 eh = make_float2(ex2_approx_ftz(th.x), ex2_approx_ftz(th.y));
  const float2 c = __fmul2_rn(tl, __ffma2_rn(tl, splat2(kLn2SqHalf), splat2(kLn2)));
  const float2 ef = __ffma2_rn(eh, c, eh);
  const __nv_bfloat162 e = __floats2bfloat162_rn(ef.x, ef.y);
  const __nv_bfloat162 d = __hadd2(__float2bfloat162_rn(1.f), e);  // T::one() + e
  const float2 sf = bf2_to_f2(*reinterpret_cast<const uint32_t *>(&s));
  const float2 df = bf2_to_f2(*reinterpret_cast<const uint32_t *>(&d));
  const float2 y = __fmul2_rn(sf, make_float2(rcp_approx(df.x), rcp_approx(df.y)));
  return __floats2bfloat162_rn(y.x, y.y);
}

__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t *>(&v); }
__device__ __forceinline__ __nv_bfloat162 bits_bf2(uint32_t w) { return *reinterpret_cast<__nv_bfloat162 *>(&w); }

__device__ __forceinline__ uint4 silu_bf16x8(uint4 v) {
  return make_uint4(bf2_bits(silu_bf16x2(bits_bf2(v.x))), bf2_bits(silu_bf16x2(bits_bf2(v.y))),
                    bf2_bits(silu_bf16x2(bits_bf2(v.z))), bf2_bits(silu_bf16x2(bits_bf2(v.w))));
}

__device__ __forceinline__ uint4 swiglu_bf16x8(uint4 g, uint4 u) {
  return make_uint4(bf2_bits(__hmul2(silu_bf16x2(bits_bf2(g.x)), bits_bf2(u.x))),
                    bf2_bits(__hmul2(silu_bf16x2(bits_bf2(g.y)), bits_bf2(u.y))),
                    bf2_bits(__hmul2(silu_bf16x2(bits_bf2(g.z)), bits_bf2(u.z))),
                    bf2_bits(__hmul2(silu_bf16x2(bits_bf2(g.w)), bits_bf2(u.w))));
}

// GELU(erf) for 16-bit T, on element pairs: y = x*0.5*(1 + erf(x/sqrt2)) in
// f32 as the reference computes it, with erf from
//   erfc(a) = exp(-a^2) * F(a),  a = min(|z|, 4),
// F(a) = erfc(a) e^{a^2} a degree-7 polynomial in t = 1 / (1 + a/2) (relative
// error 2^-22.5 on [0, 4]; coefficients from fit_gelu_erfc.py), t from the
// hardware reciprocal and exp from the hardware ex2. erf(z) = sign(z) (1 -
// erfc(a)), so for z < 0 the f32 value 1 + erf is erfc(a) rounded to erf's
// 2^-24 grid, as the reference's 1 + erff(z) is. At a = 4, 1 - erfc rounds to
// 1: |z| >= 4 gives erf = +-1, f32's value there (a NaN x stays NaN through
// x * 0.5). |z| < 2^-10: erf = z * 2/sqrt(pi), which keeps 1 + erf exact for
// the smallest x, whose f32 products are subnormal. The error of this erf is
// about 2^-21 relative in erfc and 2^-21 absolute in erf, well inside a 16-bit
// output's half ulp, so it only matters near a rounding midpoint:
// test_unary_bf16_exhaustive runs every finite bf16 input against glibc's erff
// (f32 keeps CUDA's erff).
__device__ constexpr float kErfcF[8] = {0x1.a02292p-12f, 0x1.1c1feap-2f, 0x1.354df8p-2f, 0x1.bae5c4p-3f,
                                        0x1.18f908p-3f,  0x1.367d7ep-2f, -0x1.454b7ep-2f, 0x1.4c22eap-4f};
constexpr float kTwoOverSqrtPi = 0x1.20dd76p+0f;

__device__ __forceinline__ float2 gelu_erf2(float2 x) {
  const float2 z = __fmul2_rn(x, splat2(kFrac1Sqrt2));
  const float2 a = make_float2(fminf(fabsf(z.x), 4.f), fminf(fabsf(z.y), 4.f));
  const float2 u = __ffma2_rn(a, splat2(0.5f), splat2(1.f));
  const float2 t = make_float2(rcp_approx_ftz(u.x), rcp_approx_ftz(u.y));  // u in [1, 3]
  float2 q = splat2(kErfcF[7]);
#pragma unroll
  for (int i = 6; i >= 0; --i) q = __ffma2_rn(q, t, splat2(kErfcF[i]));
  const float2 tt = __fmul2_rn(__fmul2_rn(a, a), splat2(-kLog2e));
  const float2 erfc = __fmul2_rn(make_float2(ex2_approx_ftz(tt.x), ex2_approx_ftz(tt.y)), q);
  const float2 om = __ffma2_rn(erfc, splat2(-1.f), splat2(1.f));  // 1 - erfc, one rounding
  const float2 zs = __fmul2_rn(z, splat2(kTwoOverSqrtPi));
  const float2 erf = make_float2(a.x < 0x1p-10f ? zs.x : copysignf(om.x, z.x),
                                 a.y < 0x1p-10f ? zs.y : copysignf(om.y, z.y));
  return __fmul2_rn(__fmul2_rn(x, splat2(0.5f)), __fadd2_rn(splat2(1.f), erf));
}

template <typename T, int OP>
__device__ __forceinline__ float unary_op(float x) {
  if constexpr (OP == XN_UNARY_SILU) {
    return silu_t<T>(x);
  } else if constexpr (std::is_same_v<T, float>) {
    return gelu_erf(x);
  } else {
    return gelu_erf2(make_float2(x, x)).x;
  }
}

constexpr int kBlock = 256;
constexpr int kUnroll = 4;
// Accesses per thread of the unary kernel on large tensors: 8 (128 bytes in
// flight, one input) measured 2-4 points of the copy peak above 4 for bf16 /
// f16 SiLU and GELU at 67 M - 1 G elements, and 2 lost 3-10; SwiGLU, with two
// inputs, keeps kUnroll (8 accesses of each lost 3-10 points there).
constexpr int kUnaryUnroll = 8;

// The op on one 16-byte vector of T.
template <typename T, int OP>
__device__ __forceinline__ uint4 unary_vec(uint4 raw) {
  constexpr int N = Elem<T>::kVec;
  if constexpr (std::is_same_v<T, __nv_bfloat16> && OP == XN_UNARY_SILU) {
    return silu_bf16x8(raw);
  } else if constexpr (std::is_same_v<T, __half> && OP == XN_UNARY_SILU) {
    return silu_f16x8(raw);
  } else if constexpr (!std::is_same_v<T, float> && OP == XN_UNARY_GELU_ERF) {
    float2 v2[N / 2];
    Pairs<T>::unpack(raw, v2);
#pragma unroll
    for (int j = 0; j < N / 2; ++j) v2[j] = gelu_erf2(v2[j]);
    return Pairs<T>::pack(v2);
  } else {
    float v[N];
    unpack<T>(raw, v);
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] = unary_op<T, OP>(v[j]);
    return pack<T>(v);
  }
}

// kU accesses per thread: kUnaryUnroll for large tensors; 1 for tensors whose
// one-access grid fits in one wave (8 blocks per SM), where the per-thread
// chain of work, not bandwidth, sets the time.
template <typename T, int OP, bool kVector, int kU>
__global__ void __launch_bounds__(kBlock) unary_kernel(void *dst, const void *src, int64_t n) {
  griddep_wait();
  griddep_release();
  constexpr int N = kVector ? Elem<T>::kVec : 1;
  const int64_t nacc = n / N;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kBlock * kU + threadIdx.x;
  const T *s = static_cast<const T *>(src);
  T *d = static_cast<T *>(dst);
  if constexpr (kVector) {
    uint4 raw[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = base + u * kBlock;
      if (i < nacc) raw[u] = ld_stream(s + i * N);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = base + u * kBlock;
      if (i < nacc) st_vec(d + i * N, unary_vec<T, OP>(raw[u]));
    }
    // Ragged tail (< N elements), handled by block 0.
    if (blockIdx.x == 0) {
      for (int64_t e = nacc * N + threadIdx.x; e < n; e += kBlock)
        d[e] = Elem<T>::from_f32(unary_op<T, OP>(Elem<T>::to_f32(s[e])));
    }
  } else {
    float v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = base + u * kBlock;
      if (i < n) v[u] = Elem<T>::to_f32(s[i]);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = base + u * kBlock;
      if (i < n) d[i] = Elem<T>::from_f32(unary_op<T, OP>(v[u]));
    }
  }
}

// SwiGLU over [rows, cols] with row strides; grid.x covers the columns of a
// row (in accesses of N elements), grid.y strides over rows.
template <typename T, bool kVector>
__global__ void __launch_bounds__(kBlock) swiglu_kernel(void *dst, const void *gate, const void *up,
                                                         int64_t rows, int64_t cols, int64_t gs,
                                                         int64_t us) {
  griddep_wait();
  griddep_release();
  constexpr int N = kVector ? Elem<T>::kVec : 1;
  const int64_t cacc = cols / N;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kBlock * kUnroll + threadIdx.x;
  const T *g = static_cast<const T *>(gate);
  const T *u_ = static_cast<const T *>(up);
  T *d = static_cast<T *>(dst);
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const T *gr = g + r * gs;
    const T *ur = u_ + r * us;
    T *dr = d + r * cols;
    if constexpr (kVector) {
      uint4 rg[kUnroll], ru[kUnroll];
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        const int64_t i = c0 + k * kBlock;
        if (i < cacc) {
          rg[k] = ld_stream(gr + i * N);
          ru[k] = ld_stream(ur + i * N);
        }
      }
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        const int64_t i = c0 + k * kBlock;
        if (i < cacc) {
          if constexpr (std::is_same_v<T, __nv_bfloat16>) {
            st_vec(dr + i * N, swiglu_bf16x8(rg[k], ru[k]));
          } else if constexpr (std::is_same_v<T, __half>) {
            st_vec(dr + i * N, swiglu_f16x8(rg[k], ru[k]));
          } else {
            float vg[N], vu[N];
            unpack<T>(rg[k], vg);
            unpack<T>(ru[k], vu);
#pragma unroll
            for (int j = 0; j < N; ++j) vg[j] = __fmul_rn(Elem<T>::round(silu_t<T>(vg[j])), vu[j]);
            st_vec(dr + i * N, pack<T>(vg));
          }
        }
      }
    } else {
      float vg[kUnroll], vu[kUnroll];
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        const int64_t i = c0 + k * kBlock;
        if (i < cols) {
          vg[k] = Elem<T>::to_f32(gr[i]);
          vu[k] = Elem<T>::to_f32(ur[i]);
        }
      }
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        const int64_t i = c0 + k * kBlock;
        if (i < cols) dr[i] = Elem<T>::from_f32(__fmul_rn(Elem<T>::round(silu_t<T>(vg[k])), vu[k]));
      }
    }
  }
}

// dst = T(x + T(branch * ls[col])) (or T(x + branch)) over [rows, cols]: the
// reference's LayerScale::forward (broadcast_mul, cpu_backend.rs:1379-1387)
// followed by `xs.add` (mimi.rs:1441-1444). Blocks are bx x by threads: bx (a
// power of two, up to 256) spans a row's accesses, by = 256 / bx rows, so short
// rows still fill whole blocks. A thread keeps one column, loads its layer
// scale once and handles kUnroll rows by apart; grid.y strides over row groups.
template <typename T, bool kVector>
__global__ void __launch_bounds__(kBlock) residual_kernel(void *dst, const void *x, const void *branch,
                                                           const void *ls, int64_t rows, int64_t cols,
                                                           int bx_log2) {
  griddep_wait();
  griddep_release();
  constexpr int N = kVector ? Elem<T>::kVec : 1;
  const int bx = 1 << bx_log2, by = kBlock >> bx_log2;
  const int64_t cacc = cols / N;
  const int64_t c = static_cast<int64_t>(blockIdx.x) * bx + (threadIdx.x & (bx - 1));
  if (c >= cacc) return;  // no block barrier follows
  const int ty = threadIdx.x >> bx_log2;
  const T *xs = static_cast<const T *>(x) + c * N;
  const T *bs = static_cast<const T *>(branch) + c * N;
  T *ds = static_cast<T *>(dst) + c * N;
  float vs[N];
  if (ls != nullptr) {
    if constexpr (kVector) {
      unpack<T>(ld_cached(static_cast<const T *>(ls) + c * N), vs);
    } else {
      vs[0] = Elem<T>::to_f32(static_cast<const T *>(ls)[c]);
    }
  }
  const int64_t rstep = static_cast<int64_t>(gridDim.y) * by * kUnroll;
  for (int64_t r0 = static_cast<int64_t>(blockIdx.y) * by * kUnroll + ty; r0 < rows; r0 += rstep) {
    if constexpr (kVector) {
      uint4 rx[kUnroll], rb[kUnroll];
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        const int64_t r = r0 + static_cast<int64_t>(k) * by;
        if (r < rows) {
          rx[k] = ld_stream(xs + r * cols);
          rb[k] = ld_stream(bs + r * cols);
        }
      }
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        const int64_t r = r0 + static_cast<int64_t>(k) * by;
        if (r < rows) {
          float vx[N], vb[N];
          unpack<T>(rx[k], vx);
          unpack<T>(rb[k], vb);
          if (ls != nullptr) {
#pragma unroll
            for (int j = 0; j < N; ++j) vb[j] = Elem<T>::round(__fmul_rn(vb[j], vs[j]));
          }
#pragma unroll
          for (int j = 0; j < N; ++j) vx[j] = __fadd_rn(vx[j], vb[j]);
          st_vec(ds + r * cols, pack<T>(vx));
        }
      }
    } else {
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        const int64_t r = r0 + static_cast<int64_t>(k) * by;
        if (r >= rows) break;
        float b = Elem<T>::to_f32(bs[r * cols]);
        if (ls != nullptr) b = Elem<T>::round(__fmul_rn(b, vs[0]));
        ds[r * cols] = Elem<T>::from_f32(__fadd_rn(Elem<T>::to_f32(xs[r * cols]), b));
      }
    }
  }
}

template <typename T>
int launch_residual(void *dst, const void *x, const void *branch, const void *ls, int64_t rows, int64_t cols,
                    cudaStream_t st) {
  constexpr int V = Elem<T>::kVec;
  const bool vec = cols % V == 0 && is_aligned16(dst) && is_aligned16(x) && is_aligned16(branch) && is_aligned16(ls);
  // Without a layer scale the columns do not matter: the contiguous tensor is
  // reshaped to rows of one block's width (kBlock accesses) when it divides.
  const int64_t unit = static_cast<int64_t>(kBlock) * (vec ? V : 1);
  if (ls == nullptr && (rows * cols) % unit == 0) {
    rows = rows * cols / unit;
    cols = unit;
  }
  const int64_t cacc = vec ? cols / V : cols;
  int bx_log2 = 0;
  while ((int64_t{1} << bx_log2) < cacc && (1 << bx_log2) < kBlock) ++bx_log2;
  const int64_t bx = int64_t{1} << bx_log2, by = kBlock / bx;
  const int64_t gx = ceil_div(cacc, bx);
  if (gx > 0x7fffffffLL) return fail(XN_E_INVALID, "xn_residual_add: row too long");
  int64_t gy = ceil_div(rows, by * kUnroll);
  if (gy > 65535) gy = 65535;
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy));
  if (vec)
    launch_k(residual_kernel<T, true>, grid, dim3(kBlock), 0, st, dst, x, branch, ls, rows, cols, bx_log2);
  else
    launch_k(residual_kernel<T, false>, grid, dim3(kBlock), 0, st, dst, x, branch, ls, rows, cols, bx_log2);
  return check_launch("xn_residual_add");
}

template <typename T, int kU>
void launch_unary_u(void *dst, const void *src, int64_t n, int op, bool vec, int64_t grid, cudaStream_t st) {
  if (op == XN_UNARY_SILU) {
    if (vec)
      launch_k(unary_kernel<T, XN_UNARY_SILU, true, kU>, dim3(grid), dim3(kBlock), 0, st, dst, src, n);
    else
      launch_k(unary_kernel<T, XN_UNARY_SILU, false, kU>, dim3(grid), dim3(kBlock), 0, st, dst, src, n);
  } else {
    if (vec)
      launch_k(unary_kernel<T, XN_UNARY_GELU_ERF, true, kU>, dim3(grid), dim3(kBlock), 0, st, dst, src, n);
    else
      launch_k(unary_kernel<T, XN_UNARY_GELU_ERF, false, kU>, dim3(grid), dim3(kBlock), 0, st, dst, src, n);
  }
}

template <typename T>
int launch_unary(void *dst, const void *src, int64_t n, int op, cudaStream_t st) {
  constexpr int V = Elem<T>::kVec;
  const bool vec = is_aligned16(dst) && is_aligned16(src);
  const int64_t nacc = vec ? n / V : n;
  const int64_t per_block = static_cast<int64_t>(kBlock) * kUnaryUnroll;
  if (ceil_div(nacc > 0 ? nacc : 1, static_cast<int64_t>(kBlock)) <= static_cast<int64_t>(sm_count()) * 8) {
    launch_unary_u<T, 1>(dst, src, n, op, vec, ceil_div(nacc > 0 ? nacc : 1, kBlock), st);
  } else {
    const int64_t grid = ceil_div(nacc, per_block);
    if (grid > 0x7fffffffLL) return fail(XN_E_INVALID, "xn_unary: too many elements");
    launch_unary_u<T, kUnaryUnroll>(dst, src, n, op, vec, grid, st);
  }
  return check_launch("xn_unary");
}

template <typename T>
int launch_swiglu(void *dst, const void *gate, const void *up, int64_t rows, int64_t cols, int64_t gs,
                  int64_t us, cudaStream_t st) {
  constexpr int V = Elem<T>::kVec;
  // Contiguous operands are one long row: better load balance, no row loop.
  if (gs == cols && us == cols && rows > 1) {
    cols = rows * cols;
    gs = us = cols;
    rows = 1;
  }
  const bool vec = is_aligned16(dst) && is_aligned16(gate) && is_aligned16(up) && cols % V == 0 &&
                   gs % V == 0 && us % V == 0;
  const int64_t cacc = vec ? cols / V : cols;
  const int64_t gx = ceil_div(cacc, static_cast<int64_t>(kBlock) * kUnroll);
  if (gx > 0x7fffffffLL) return fail(XN_E_INVALID, "xn_swiglu: row too long");
  const int64_t gy = rows < 65535 ? rows : 65535;
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy));
  if (vec)
    launch_k(swiglu_kernel<T, true>, dim3(grid), dim3(kBlock), 0, st, dst, gate, up, rows, cols, gs, us);
  else
    launch_k(swiglu_kernel<T, false>, dim3(grid), dim3(kBlock), 0, st, dst, gate, up, rows, cols, gs, us);
  return check_launch("xn_swiglu");
}

}  // namespace
}  // namespace xn

extern "C" {

int xn_unary(void *dst, const void *src, int64_t n, int op, int dtype, void *stream) {
  using namespace xn;
  if (!is_float_dtype(dtype)) return fail(XN_E_DTYPE, "xn_unary: unsupported dtype %d", dtype);
  if (op != XN_UNARY_SILU && op != XN_UNARY_GELU_ERF) return fail(XN_E_INVALID, "xn_unary: unknown op %d", op);
  if (n < 0) return fail(XN_E_INVALID, "xn_unary: negative size");
  if (n == 0) return ok();
  if (dst == nullptr || src == nullptr) return fail(XN_E_INVALID, "xn_unary: null dst or src");
  XN_DISPATCH_FLOAT(dtype, return launch_unary<T>(dst, src, n, op, as_stream(stream)));
  return fail(XN_E_DTYPE, "xn_unary: unsupported dtype %d", dtype);
}

int xn_residual_add(void *dst, const void *x, const void *branch, const void *layer_scale, int64_t rows,
                    int64_t cols, int dtype, void *stream) {
  using namespace xn;
  if (!is_float_dtype(dtype)) return fail(XN_E_DTYPE, "xn_residual_add: unsupported dtype %d", dtype);
  if (rows < 0 || cols < 0) return fail(XN_E_INVALID, "xn_residual_add: negative size");
  if (rows == 0 || cols == 0) return ok();
  if (dst == nullptr || x == nullptr || branch == nullptr) return fail(XN_E_INVALID, "xn_residual_add: null pointer");
  XN_DISPATCH_FLOAT(dtype, return launch_residual<T>(dst, x, branch, layer_scale, rows, cols, as_stream(stream)));
  return fail(XN_E_DTYPE, "xn_residual_add: unsupported dtype %d", dtype);
}

int xn_swiglu(void *dst, const void *gate, const void *up, int64_t rows, int64_t cols,
              int64_t gate_stride, int64_t up_stride, int dtype, void *stream) {
  using namespace xn;
  if (!is_float_dtype(dtype)) return fail(XN_E_DTYPE, "xn_swiglu: unsupported dtype %d", dtype);
  if (rows < 0 || cols < 0) return fail(XN_E_INVALID, "xn_swiglu: negative size");
  if (rows == 0 || cols == 0) return ok();
  if (gate_stride < cols || up_stride < cols)
    return fail(XN_E_INVALID, "xn_swiglu: row stride smaller than cols (gate %lld, up %lld, cols %lld)",
                (long long)gate_stride, (long long)up_stride, (long long)cols);
  if (dst == nullptr || gate == nullptr || up == nullptr) return fail(XN_E_INVALID, "xn_swiglu: null pointer");
  XN_DISPATCH_FLOAT(dtype, return launch_swiglu<T>(dst, gate, up, rows, cols, gate_stride, up_stride,
                                                   as_stream(stream)));
  return fail(XN_E_DTYPE, "xn_swiglu: unsupported dtype %d", dtype);
}

}  // extern "C"
