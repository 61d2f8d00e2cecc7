// xn_common.cuh - shared device helpers for the sm_100a fused layer-op kernels.
//
// Every kernel here is HBM-bandwidth bound. The helpers below give:
//   * element traits: load/convert to f32 and round an f32 back to the element
//     type T with round-to-nearest-even, so a kernel can reproduce each point
//     where the reference CPU backend rounds a T-typed intermediate;
//   * 16-byte vector loads/stores with explicit cache hints (streamed data is
//     read with L1::no_allocate so weights and tables keep L1);
//   * sub-warp / multi-warp reductions for "row groups" of power-of-two threads.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

namespace xn {

// ---------------------------------------------------------------------------
// Programmatic dependent launch (sm_90+). Every kernel of the library begins
// with griddep_wait(), which returns once the previous kernel of the stream
// has completed and its memory operations are visible (immediately when the
// launch did not allow early scheduling), then griddep_release(), which lets
// the next such kernel be scheduled as soon as every block of this one has
// started. Nothing is read before the wait, so results never depend on it.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Element traits. `round` maps an f32 value to the nearest T and back to f32:
// it is the value the reference would hold after one T-typed operation.
// ---------------------------------------------------------------------------
template <typename T>
struct Elem;

template <>
struct Elem<float> {
  static constexpr int kVec = 4;  // elements per 16-byte vector
  __device__ __forceinline__ static float to_f32(float x) { return x; }
  __device__ __forceinline__ static float from_f32(float x) { return x; }
  __device__ __forceinline__ static float round(float x) { return x; }
};

template <>
struct Elem<__nv_bfloat16> {
  static constexpr int kVec = 8;
  __device__ __forceinline__ static float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ __forceinline__ static __nv_bfloat16 from_f32(float x) { return __float2bfloat16_rn(x); }
  __device__ __forceinline__ static float round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
};

template <>
struct Elem<__half> {
  static constexpr int kVec = 8;
  __device__ __forceinline__ static float to_f32(__half x) { return __half2float(x); }
  __device__ __forceinline__ static __half from_f32(float x) { return __float2half_rn(x); }
  __device__ __forceinline__ static float round(float x) { return __half2float(__float2half_rn(x)); }
};

// ---------------------------------------------------------------------------
// 16-byte vector memory access.
// ---------------------------------------------------------------------------
// Streamed, read-once data: do not allocate in L1. This is a coherent load
// (no .nc), so it stays correct when the kernel also writes the same buffer
// (dst or residual_out aliasing src is allowed by the C ABI).
__device__ __forceinline__ uint4 ld_stream(const void *p) {
  uint4 r;
  asm volatile("ld.global.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Reused data (weights, cos/sin tables, codebooks): read-only, cached.
__device__ __forceinline__ uint4 ld_cached(const void *p) {
  return __ldg(reinterpret_cast<const uint4 *>(p));
}

__device__ __forceinline__ uint2 ld_cached8(const void *p) {
  return __ldg(reinterpret_cast<const uint2 *>(p));
}

// Plain coherent load, for buffers a kernel may also write (aliasing allowed).
__device__ __forceinline__ uint4 ld_plain(const void *p) {
  return *reinterpret_cast<const uint4 *>(p);
}

__device__ __forceinline__ void st_vec(void *p, uint4 v) { *reinterpret_cast<uint4 *>(p) = v; }

// Row accesses of AW 32-bit words (AW = 4: 16 bytes, 2: 8 bytes, 1: 4 bytes)
// held in the low words of a uint4; the other words are 0. Rows whose byte
// width is a multiple of 8 or 4 but not of 16 (16-bit rows of even width,
// f32 rows of even width) keep one access per 8 / 4 bytes instead of falling
// back to element accesses.
template <int AW>
__device__ __forceinline__ uint4 ld_stream_w(const void *p) {
  if constexpr (AW == 4) {
    return ld_stream(p);
  } else if constexpr (AW == 2) {
    uint4 r = make_uint4(0u, 0u, 0u, 0u);
    asm volatile("ld.global.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
  } else {
    uint4 r = make_uint4(0u, 0u, 0u, 0u);
    asm volatile("ld.global.L1::no_allocate.u32 %0, [%1];" : "=r"(r.x) : "l"(p));
    return r;
  }
}

template <int AW>
__device__ __forceinline__ uint4 ld_cached_w(const void *p) {
  if constexpr (AW == 4) {
    return __ldg(reinterpret_cast<const uint4 *>(p));
  } else if constexpr (AW == 2) {
    const uint2 v = __ldg(reinterpret_cast<const uint2 *>(p));
    return make_uint4(v.x, v.y, 0u, 0u);
  } else {
    return make_uint4(__ldg(reinterpret_cast<const unsigned int *>(p)), 0u, 0u, 0u);
  }
}

template <int AW>
__device__ __forceinline__ void st_w(void *p, uint4 v) {
  if constexpr (AW == 4) {
    *reinterpret_cast<uint4 *>(p) = v;
  } else if constexpr (AW == 2) {
    *reinterpret_cast<uint2 *>(p) = make_uint2(v.x, v.y);
  } else {
    *reinterpret_cast<unsigned int *>(p) = v.x;
  }
}

// Returns v unchanged through moves the compiler cannot see through. Used to
// make a second pass over packed register data unpack it again instead of
// keeping the first pass's unpacked f32 copies live (which doubles register
// use for 16-bit rows).
__device__ __forceinline__ uint4 opaque(uint4 v) {
  asm volatile("mov.b32 %0, %0;\n\tmov.b32 %1, %1;\n\tmov.b32 %2, %2;\n\tmov.b32 %3, %3;"
               : "+r"(v.x), "+r"(v.y), "+r"(v.z), "+r"(v.w));
  return v;
}

// The j-th 32-bit word of a 16-byte vector (j a compile-time constant after
// unrolling).
__device__ __forceinline__ uint32_t u4_word(const uint4 &v, int j) {
  return j == 0 ? v.x : (j == 1 ? v.y : (j == 2 ? v.z : v.w));
}

// Unpack / pack 16 bytes as kVec values of T widened to f32.
template <typename T>
__device__ __forceinline__ void unpack(const uint4 &v, float (&f)[Elem<T>::kVec]);

template <>
__device__ __forceinline__ void unpack<float>(const uint4 &v, float (&f)[4]) {
  f[0] = __uint_as_float(v.x);
  f[1] = __uint_as_float(v.y);
  f[2] = __uint_as_float(v.z);
  f[3] = __uint_as_float(v.w);
}

// bf16 is the high half of an f32: widening is a shift (low element) and a
// mask (high element), one integer operation each.
__device__ __forceinline__ float2 bf2_to_f2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

__device__ __forceinline__ float2 h2_to_f2(uint32_t w) {
  __half2 h = *reinterpret_cast<__half2 *>(&w);
  return __half22float2(h);
}

template <>
__device__ __forceinline__ void unpack<__nv_bfloat16>(const uint4 &v, float (&f)[8]) {
  float2 a = bf2_to_f2(v.x), b = bf2_to_f2(v.y), c = bf2_to_f2(v.z), d = bf2_to_f2(v.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

template <>
__device__ __forceinline__ void unpack<__half>(const uint4 &v, float (&f)[8]) {
  float2 a = h2_to_f2(v.x), b = h2_to_f2(v.y), c = h2_to_f2(v.z), d = h2_to_f2(v.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

template <typename T>
__device__ __forceinline__ uint4 pack(const float (&f)[Elem<T>::kVec]);

template <>
__device__ __forceinline__ uint4 pack<float>(const float (&f)[4]) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                    __float_as_uint(f[3]));
}

__device__ __forceinline__ uint32_t f2_to_bf2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ uint32_t f2_to_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&h);
}

template <>
__device__ __forceinline__ uint4 pack<__nv_bfloat16>(const float (&f)[8]) {
  return make_uint4(f2_to_bf2(f[0], f[1]), f2_to_bf2(f[2], f[3]), f2_to_bf2(f[4], f[5]),
                    f2_to_bf2(f[6], f[7]));
}

template <>
__device__ __forceinline__ uint4 pack<__half>(const float (&f)[8]) {
  return make_uint4(f2_to_h2(f[0], f[1]), f2_to_h2(f[2], f[3]), f2_to_h2(f[4], f[5]),
                    f2_to_h2(f[6], f[7]));
}

// ---------------------------------------------------------------------------
// A 16-byte vector as adjacent element pairs in f32, for the sm_100 paired f32
// instructions (__fadd2_rn / __fmul2_rn / __ffma2_rn: two IEEE f32 operations
// per instruction, each rounded exactly like its scalar form). bf16 widens by
// bit placement (one shift or mask per element); packing rounds a pair with
// one cvt.rn.{bf16x2,f16x2}.f32.
// ---------------------------------------------------------------------------
template <typename T>
struct Pairs;

template <>
struct Pairs<float> {
  static constexpr int kP = 2;  // pairs per 16-byte vector
  __device__ __forceinline__ static void unpack(const uint4 &v, float2 (&p)[2]) {
    p[0] = make_float2(__uint_as_float(v.x), __uint_as_float(v.y));
    p[1] = make_float2(__uint_as_float(v.z), __uint_as_float(v.w));
  }
  __device__ __forceinline__ static uint4 pack(const float2 (&p)[2]) {
    return make_uint4(__float_as_uint(p[0].x), __float_as_uint(p[0].y), __float_as_uint(p[1].x),
                      __float_as_uint(p[1].y));
  }
};

template <>
struct Pairs<__nv_bfloat16> {
  static constexpr int kP = 4;
  __device__ __forceinline__ static void unpack(const uint4 &v, float2 (&p)[4]) {
    p[0] = bf2_to_f2(v.x);
    p[1] = bf2_to_f2(v.y);
    p[2] = bf2_to_f2(v.z);
    p[3] = bf2_to_f2(v.w);
  }
  __device__ __forceinline__ static uint4 pack(const float2 (&p)[4]) {
    return make_uint4(f2_to_bf2(p[0].x, p[0].y), f2_to_bf2(p[1].x, p[1].y), f2_to_bf2(p[2].x, p[2].y),
                      f2_to_bf2(p[3].x, p[3].y));
  }
};

template <>
struct Pairs<__half> {
  static constexpr int kP = 4;
  __device__ __forceinline__ static void unpack(const uint4 &v, float2 (&p)[4]) {
    p[0] = h2_to_f2(v.x);
    p[1] = h2_to_f2(v.y);
    p[2] = h2_to_f2(v.z);
    p[3] = h2_to_f2(v.w);
  }
  __device__ __forceinline__ static uint4 pack(const float2 (&p)[4]) {
    return make_uint4(f2_to_h2(p[0].x, p[0].y), f2_to_h2(p[1].x, p[1].y), f2_to_h2(p[2].x, p[2].y),
                      f2_to_h2(p[3].x, p[3].y));
  }
};

__device__ __forceinline__ float2 splat2(float v) { return make_float2(v, v); }

// h = T(x + T(b * s)) (with s) or T(x + b) (without) on a 16-byte vector: the
// reference's LayerScale multiply and residual add, each a T operation that
// rounds its f32 result to T. For bf16 / f16 the paired instructions round
// the exact result once, which gives the same T value:
//   * the product of two 8- or 11-bit significands is exact in f32 (a bf16
//     product in the subnormal range has at most 16 significant bits, so f32
//     rounding cannot move it onto a bf16 midpoint either);
//   * an f32 sum of two T values is inexact only when the smaller term is
//     below 2^-15 of the larger, far inside half a T ulp, so both roundings
//     return the larger term's neighbourhood value.
template <typename T>
__device__ __forceinline__ uint32_t t2_add(uint32_t a, uint32_t b);
template <typename T>
__device__ __forceinline__ uint32_t t2_mul(uint32_t a, uint32_t b);

template <>
__device__ __forceinline__ uint32_t t2_add<__nv_bfloat16>(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hadd2(*reinterpret_cast<__nv_bfloat162 *>(&a), *reinterpret_cast<__nv_bfloat162 *>(&b));
  return *reinterpret_cast<uint32_t *>(&r);
}
template <>
__device__ __forceinline__ uint32_t t2_mul<__nv_bfloat16>(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hmul2(*reinterpret_cast<__nv_bfloat162 *>(&a), *reinterpret_cast<__nv_bfloat162 *>(&b));
  return *reinterpret_cast<uint32_t *>(&r);
}
template <>
__device__ __forceinline__ uint32_t t2_add<__half>(uint32_t a, uint32_t b) {
  __half2 r = __hadd2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b));
  return *reinterpret_cast<uint32_t *>(&r);
}
template <>
__device__ __forceinline__ uint32_t t2_mul<__half>(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b));
  return *reinterpret_cast<uint32_t *>(&r);
}

// AW: the access width in 32-bit words (see ld_stream_w); only those words
// are computed.
template <typename T, int AW = 4>
__device__ __forceinline__ uint4 residual_vec(uint4 x, uint4 b, const void *s) {
  if constexpr (std::is_same<T, float>::value) {
    static_assert(AW >= 2, "f32 accesses hold whole element pairs");
    constexpr int KP = AW / 2;
    float2 bp[2], xp[2];
    Pairs<float>::unpack(b, bp);
    Pairs<float>::unpack(x, xp);
    if (s != nullptr) {
      float2 sp[2];
      Pairs<float>::unpack(ld_cached_w<AW>(s), sp);
#pragma unroll
      for (int j = 0; j < KP; ++j) bp[j] = __fmul2_rn(bp[j], sp[j]);
    }
#pragma unroll
    for (int j = 0; j < KP; ++j) xp[j] = __fadd2_rn(xp[j], bp[j]);
    if constexpr (KP == 1) xp[1] = make_float2(0.f, 0.f);
    return Pairs<float>::pack(xp);
  } else {
    uint32_t xw[4] = {x.x, x.y, x.z, x.w}, bw[4] = {b.x, b.y, b.z, b.w};
    if (s != nullptr) {
      const uint4 sv = ld_cached_w<AW>(s);
      const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
      for (int j = 0; j < AW; ++j) bw[j] = t2_mul<T>(bw[j], sw[j]);
    }
#pragma unroll
    for (int j = 0; j < AW; ++j) xw[j] = t2_add<T>(xw[j], bw[j]);
#pragma unroll
    for (int j = AW; j < 4; ++j) xw[j] = 0u;
    return make_uint4(xw[0], xw[1], xw[2], xw[3]);
  }
}

// residual_vec's arithmetic on a whole 16-byte vector with the layer-scale
// vector already loaded (sv, or nullptr for no scale), for a scale held in
// shared memory. The f32 form uses scalar IEEE operations: with the paired
// instructions in this form, the residual outputs were measured one ulp off
// the reference's product-then-sum for some elements.
template <typename T>
__device__ __forceinline__ uint4 residual_vec_sv(uint4 x, uint4 b, const uint4 *sv) {
  if constexpr (std::is_same<T, float>::value) {
    float2 bp[2], xp[2];
    Pairs<float>::unpack(b, bp);
    Pairs<float>::unpack(x, xp);
    if (sv != nullptr) {
      float2 sp[2];
      Pairs<float>::unpack(*sv, sp);
#pragma unroll
      for (int j = 0; j < 2; ++j) bp[j] = make_float2(__fmul_rn(bp[j].x, sp[j].x), __fmul_rn(bp[j].y, sp[j].y));
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) xp[j] = make_float2(__fadd_rn(xp[j].x, bp[j].x), __fadd_rn(xp[j].y, bp[j].y));
    return Pairs<float>::pack(xp);
  } else {
    uint32_t xw[4] = {x.x, x.y, x.z, x.w}, bw[4] = {b.x, b.y, b.z, b.w};
    if (sv != nullptr) {
      const uint32_t sw[4] = {sv->x, sv->y, sv->z, sv->w};
#pragma unroll
      for (int j = 0; j < 4; ++j) bw[j] = t2_mul<T>(bw[j], sw[j]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) xw[j] = t2_add<T>(xw[j], bw[j]);
    return make_uint4(xw[0], xw[1], xw[2], xw[3]);
  }
}

// Half a vector (8 bytes): kVec/2 values, used for the interleaved-RoPE tables.
template <typename T>
__device__ __forceinline__ void unpack_half(const uint2 &v, float (&f)[Elem<T>::kVec / 2]);

template <>
__device__ __forceinline__ void unpack_half<float>(const uint2 &v, float (&f)[2]) {
  f[0] = __uint_as_float(v.x);
  f[1] = __uint_as_float(v.y);
}

template <>
__device__ __forceinline__ void unpack_half<__nv_bfloat16>(const uint2 &v, float (&f)[4]) {
  float2 a = bf2_to_f2(v.x), b = bf2_to_f2(v.y);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}

template <>
__device__ __forceinline__ void unpack_half<__half>(const uint2 &v, float (&f)[4]) {
  float2 a = h2_to_f2(v.x), b = h2_to_f2(v.y);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}

// Scalar element access for the unaligned / ragged fallbacks.
template <typename T>
__device__ __forceinline__ float ld_elem(const void *base, int64_t i) {
  return Elem<T>::to_f32(reinterpret_cast<const T *>(base)[i]);
}

template <typename T>
__device__ __forceinline__ void st_elem(void *base, int64_t i, float v) {
  reinterpret_cast<T *>(base)[i] = Elem<T>::from_f32(v);
}

// Half-split rotation of one 16-byte chunk of each half:
//   y1 = T(T(x1*c) - T(x2*s)),  y2 = T(T(x1*s) + T(x2*c)).
// bf16 / f16 use the native paired instructions, which round each product and
// sum once, exactly as the reference's T arithmetic does (the product of two
// 8- or 11-bit significands is exact in f32; see residual_vec for the sum).
template <typename T>
__device__ __forceinline__ void rotate_halfsplit(const uint4 &x1, const uint4 &x2, const uint4 &c, const uint4 &s,
                                                 uint4 &y1, uint4 &y2) {
  if constexpr (std::is_same_v<T, float>) {
    float a[4], b[4], cv[4], sv[4], o1[4], o2[4];
    unpack<T>(x1, a);
    unpack<T>(x2, b);
    unpack<T>(c, cv);
    unpack<T>(s, sv);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      o1[j] = __fsub_rn(__fmul_rn(a[j], cv[j]), __fmul_rn(b[j], sv[j]));
      o2[j] = __fadd_rn(__fmul_rn(a[j], sv[j]), __fmul_rn(b[j], cv[j]));
    }
    y1 = pack<T>(o1);
    y2 = pack<T>(o2);
  } else {
    using T2 = std::conditional_t<std::is_same_v<T, __half>, __half2, __nv_bfloat162>;
    const uint32_t *pa = &x1.x, *pb = &x2.x, *pc = &c.x, *ps = &s.x;
    uint32_t o1[4], o2[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const T2 a = *reinterpret_cast<const T2 *>(pa + j), b = *reinterpret_cast<const T2 *>(pb + j);
      const T2 cv = *reinterpret_cast<const T2 *>(pc + j), sv = *reinterpret_cast<const T2 *>(ps + j);
      const T2 r1 = __hsub2(__hmul2(a, cv), __hmul2(b, sv));
      const T2 r2 = __hadd2(__hmul2(a, sv), __hmul2(b, cv));
      o1[j] = *reinterpret_cast<const uint32_t *>(&r1);
      o2[j] = *reinterpret_cast<const uint32_t *>(&r2);
    }
    y1 = make_uint4(o1[0], o1[1], o1[2], o1[3]);
    y2 = make_uint4(o2[0], o2[1], o2[2], o2[3]);
  }
}

// Interleaved rotation of one 16-byte vector: pairs (x[2j], x[2j+1]) with
// c_j, s_j from the kVec/2 table values in c / s:
//   y[2j] = T(T(x[2j]*c) - T(x[2j+1]*s)),  y[2j+1] = T(T(x[2j]*s) + T(x[2j+1]*c)).
// For bf16 / f16 a pair is one 32-bit word w = (a, b): m1 = w*(c,c) = (ac, bc)
// and m2 = w*(s,s) = (as, bs) are paired products; swapping m2's halves and
// negating the low one gives (-bs, as), and one paired add gives
// (ac - bs, bc + as). Negation is exact and x - y is x + (-y) in IEEE
// arithmetic, so every result is the reference's T value.
template <typename T>
__device__ __forceinline__ uint4 rotate_interleaved(const uint4 &x, const uint2 &c, const uint2 &s) {
  if constexpr (std::is_same_v<T, float>) {
    const float cv[2] = {__uint_as_float(c.x), __uint_as_float(c.y)};
    const float sv[2] = {__uint_as_float(s.x), __uint_as_float(s.y)};
    const float xv[4] = {__uint_as_float(x.x), __uint_as_float(x.y), __uint_as_float(x.z), __uint_as_float(x.w)};
    float y[4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float a = xv[2 * j], b = xv[2 * j + 1];
      y[2 * j] = __fsub_rn(__fmul_rn(a, cv[j]), __fmul_rn(b, sv[j]));
      y[2 * j + 1] = __fadd_rn(__fmul_rn(a, sv[j]), __fmul_rn(b, cv[j]));
    }
    return make_uint4(__float_as_uint(y[0]), __float_as_uint(y[1]), __float_as_uint(y[2]), __float_as_uint(y[3]));
  } else {
    const uint32_t xw[4] = {x.x, x.y, x.z, x.w};
    const uint32_t cw[2] = {c.x, c.y}, sw[2] = {s.x, s.y};
    uint32_t y[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t sel = (j & 1) ? 0x3232u : 0x1010u;  // splat the low or high half
      const uint32_t cc = __byte_perm(cw[j >> 1], 0u, sel), ss = __byte_perm(sw[j >> 1], 0u, sel);
      const uint32_t m1 = t2_mul<T>(xw[j], cc);
      const uint32_t m2 = t2_mul<T>(xw[j], ss);
      const uint32_t neg_swapped = __byte_perm(m2, 0u, 0x1032u) ^ 0x00008000u;  // (-bs, as)
      y[j] = t2_add<T>(m1, neg_swapped);
    }
    return make_uint4(y[0], y[1], y[2], y[3]);
  }
}

// ---------------------------------------------------------------------------
// Reductions inside a row group of `tpr` threads (power of two, 1..1024).
// Groups smaller than a warp use xor-shuffles that stay inside the group (the
// offsets below tpr, largest first, unrolled: no loop counter per step);
// larger groups combine per-warp partials through shared memory `red`, which
// must hold one float per warp of the block. The combination order is fixed,
// so results are deterministic run to run.
//
// kReuse = false drops the trailing barrier that protects `red` from the
// caller's next write to it. That is safe when every reduction of a row has
// its own `red` array and each one is reached by every thread: a warp writes
// an array again only after passing the barrier of a later reduction, which
// every warp reaches only after its own reads of that array.
// ---------------------------------------------------------------------------
template <bool kReuse = true>
__device__ __forceinline__ float group_sum(float v, int tpr, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    if (o < tpr) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (tpr <= 32) return v;
  const int warp = threadIdx.x >> 5;
  const int wpr = tpr >> 5;
  const int first = (warp / wpr) * wpr;
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  float s = red[first];
  for (int w = 1; w < wpr; ++w) s = __fadd_rn(s, red[first + w]);
  if constexpr (kReuse) __syncthreads();  // `red` may be reused by the caller's next reduction
  return s;
}

template <bool kReuse = true>
__device__ __forceinline__ float group_max(float v, int tpr, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    if (o < tpr) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (tpr <= 32) return v;
  const int warp = threadIdx.x >> 5;
  const int wpr = tpr >> 5;
  const int first = (warp / wpr) * wpr;
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  float s = red[first];
  for (int w = 1; w < wpr; ++w) s = fmaxf(s, red[first + w]);
  if constexpr (kReuse) __syncthreads();
  return s;
}

// ---------------------------------------------------------------------------
// Division. The reference divides in f32 with IEEE round-to-nearest; these
// helpers return the same f32 result more cheaply.
// ---------------------------------------------------------------------------
// x / d for many x and one d, given r = __frcp_rn(d) (correctly rounded 1/d):
// q0 = RN(x*r) is within one ulp of x/d, rem = x - d*q0 is exact with an FMA,
// and RN(q0 + rem*r) is the correctly rounded quotient (Markstein's theorem;
// no overflow is possible where it is used: |x/d| stays far inside the f32
// range). d > 0, so the quotient has the sign of x (and of q0): copysign keeps
// -0 / d == -0, which the correction step alone would turn into +0.
// d = +inf (an RMSNorm row whose sum of squares overflowed) gives r = 0, and
// -d * q0 would be -inf * 0 = NaN; with 0 in its place the steps return
// q0 = x * 0 = +-0 for finite x and NaN for x = +-inf, the IEEE quotients.
__device__ __forceinline__ float neg_divisor(float d) { return isinf(d) ? 0.f : -d; }

__device__ __forceinline__ float div_by(float x, float d, float r) {
  const float q0 = __fmul_rn(x, r);
  const float rem = __fmaf_rn(neg_divisor(d), q0, x);
  return copysignf(__fmaf_rn(rem, r, q0), q0);
}

// exp(x) for a bf16 value x <= 0 (softmax's T(x - max)), accurate enough
// that rounding it to bf16 gives the reference's T(exp(x)) (f32 exp, then
// round to bf16): 2^(x * log2 e) with one f32 multiply (relative error
// <= 2^-24 of t, so at most |t| * 2^-24 * ln 2 <= 2^-17.5 in the result for
// |t| < 134, where results still reach the bf16 range) and the hardware 2^t
// approximation (ex2.approx.f32, subnormal results kept). A result can only
// round differently where exp(x) lies within that error of a bf16 rounding
// midpoint; the softmax tests run every non-positive bf16 input (2^15 values)
// through both softmax paths against glibc and find none. Not used for f32 or
// f16, whose finer output grids would expose the error, nor for positive
// arguments (SiLU's exp(-s)), which were not proven.
constexpr float kLog2e = 0x1.715476p+0f;
constexpr float kLn2 = 0x1.62e43p-1f;
constexpr float kLn2SqHalf = 0x1.ebfbep-3f;

// exp(x) for f16 values x with |x| <= 40 (a pair), accurate to the hardware
// ex2's error: 2^(x kL2eHi16) (kL2eHi16 has 13 significant bits, x 11, so the
// product is exact in f32) times 1 + c, c = t ln2 + (t ln2)^2 / 2 for the low
// part t = x kL2eLo16 (|t| < 2^-8.5, so the dropped third-order term is below
// 2^-29 relative). Callers clamp to [-40, 40], where exp's f16 value is
// already 0 or inf beyond.
constexpr float kL2eHi16 = 0x1.715p+0f;
constexpr float kL2eLo16 = 0x1.1d94aep-14f;

// 2^t by the hardware approximation, subnormal results kept.
__device__ __forceinline__ float ex2_approx(float t) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(t));
  return y;
}

// The same approximation with subnormal results flushed to zero, which saves
// the instructions that keep them. For t >= -126 (normal results) it returns
// the value of ex2_approx: the softmax tests run every bf16 argument that
// takes this path through it against glibc.
__device__ __forceinline__ float ex2_approx_ftz(float t) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(t));
  return y;
}

__device__ __forceinline__ float exp_of_bf16(float x) { return ex2_approx(__fmul_rn(x, kLog2e)); }

__device__ __forceinline__ float2 exp_split_f16(float2 x) {
  const float2 th = __fmul2_rn(x, make_float2(kL2eHi16, kL2eHi16));
  const float2 tl = __fmul2_rn(x, make_float2(kL2eLo16, kL2eLo16));
  const float2 eh = make_float2(ex2_approx_ftz(th.x), ex2_approx_ftz(th.y));
  const float2 c = __fmul2_rn(tl, __ffma2_rn(tl, make_float2(kLn2SqHalf, kLn2SqHalf), make_float2(kLn2, kLn2)));
  return __ffma2_rn(eh, c, eh);
}

// exp of a non-positive argument as the T-typed reference computes it, before
// the rounding to T.
template <typename T>
__device__ __forceinline__ float exp_t(float x) {
  if constexpr (std::is_same_v<T, __nv_bfloat16>) {
    return exp_of_bf16(x);
  } else {
    return expf(x);
  }
}

// c + widen(w's low half), c + widen(w's high half) for a packed 16-bit pair
// w, each rounded once to f32: sm_100's mixed-precision add, which takes the
// 16-bit operand as it is, so the pair needs no unpacking. The same values as
// __fadd2_rn(c, widened w).
template <typename T>
__device__ __forceinline__ float2 add2_widen(uint32_t w, float2 c);

template <>
__device__ __forceinline__ float2 add2_widen<__nv_bfloat16>(uint32_t w, float2 c) {
  float2 d;
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\tadd.rn.f32.bf16 %0, lo, %3;\n\tadd.rn.f32.bf16 %1, hi, %4;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "r"(w), "f"(c.x), "f"(c.y));
  return d;
}

template <>
__device__ __forceinline__ float2 add2_widen<__half>(uint32_t w, float2 c) {
  float2 d;
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\tadd.rn.f32.f16 %0, lo, %3;\n\tadd.rn.f32.f16 %1, hi, %4;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "r"(w), "f"(c.x), "f"(c.y));
  return d;
}

// c + lo*lo, c + hi*hi for a packed 16-bit pair (lo, hi), each rounded once to
// f32: sm_100's mixed-precision fma on the stored halves, the same values as
// __ffma2_rn(x, x, c) on the widened pair.
template <typename T>
__device__ __forceinline__ float2 sq_add2_widen(uint32_t w, float2 c);

template <>
__device__ __forceinline__ float2 sq_add2_widen<__nv_bfloat16>(uint32_t w, float2 c) {
  float2 d;
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\tfma.rn.f32.bf16 %0, lo, lo, %3;\n\tfma.rn.f32.bf16 %1, hi, hi, %4;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "r"(w), "f"(c.x), "f"(c.y));
  return d;
}

template <>
__device__ __forceinline__ float2 sq_add2_widen<__half>(uint32_t w, float2 c) {
  float2 d;
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\tfma.rn.f32.f16 %0, lo, lo, %3;\n\tfma.rn.f32.f16 %1, hi, hi, %4;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "r"(w), "f"(c.x), "f"(c.y));
  return d;
}

// div_by on an element pair, for dividends that are never -0 (exp results):
// with x = +0 every step is +0, so the sign fix-up is not needed. nd = -d,
// r = __frcp_rn(d) in both lanes.
__device__ __forceinline__ float2 div_nonneg2(float2 x, float2 nd, float2 r) {
  const float2 q0 = __fmul2_rn(x, r);
  const float2 rem = __ffma2_rn(nd, q0, x);
  return __ffma2_rn(rem, r, q0);
}

__host__ __device__ __forceinline__ bool aligned16(const void *p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// ---------------------------------------------------------------------------
// Bulk copies from global into this block's shared memory: cp.async.bulk, the
// untiled form of the TMA engine, completing on an mbarrier of the block.
// Both addresses 16-byte aligned, size a multiple of 16 bytes.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes the initialised barriers visible to the copy engine; a block barrier
// must follow before other threads use them.
__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// Orders shared-memory accesses made (or synchronised with) before it ahead of
// bulk copies issued after it: a buffer whose reads the block has finished is
// then safe to refill.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// L2 policy for data read once: its lines are the first to go.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Arms `bar` (one arrival, `bytes` of transactions) and starts the copy of
// `bytes` from global `src` to shared `dst`; the barrier's phase completes
// when the bytes have landed.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                          uint64_t policy) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Waits until the phase of `bar` with the given parity has completed. Gives up
// after `limit` polls (each poll may suspend the thread for a short,
// hardware-chosen time) and returns false, so a copy that never completes
// cannot hang the kernel.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t limit) {
  const uint32_t a = smem_u32(bar);
  for (uint32_t i = 0; i < limit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

}  // namespace xn
