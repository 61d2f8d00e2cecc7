// xn_softmax.cu - row softmax (optionally fused with the causal mask) and the
// stand-alone in-place causal mask, for sm_100a.
//
// Reference semantics: mimi-rs/src/cpu_backend.rs:667-689 (softmax) and
// :647-665 (apply_causality_mask). Per row, in T arithmetic:
//   max = max_j x_j ; e_j = T(exp(T(x_j - max))) ; sum = sum_j f32(e_j)
//   y_j = T(f32(e_j) / sum)
// With the mask fused, columns j > offset + i (i = query index of the row) are
// not read and produce exactly 0, which is what exp(-inf - max) / sum gives
// in the reference's mask-then-softmax composite.
//
// Design: like the norm kernels, a row group of tpr threads holds the whole row
// in registers (one HBM read, one HBM write per element); max and sum are
// group reductions. Narrower rows prefetch the next row into registers; wide
// rows (up to 64 KB) are streamed into shared memory by bulk copies instead.
// Rows wider than that, or wider than 16384 elements in the scalar path, use
// a three-pass kernel.
#include <math.h>
#include <cstdlib>

#include <cooperative_groups.h>

#include <type_traits>

#include "xn_common.cuh"
#include "xn_internal.h"

namespace xn {
namespace {

struct SoftmaxParams {
  void *dst;
  const void *src;
  int64_t rows;
  int64_t cols;
  int64_t t1;      // query rows per (b, h) slice when causal
  int64_t offset;  // position of the first query
  int causal;
  int tpr;
  int nvec;
  int scaled;      // apply x = T(x * scale) first (the attention score scale)
  float scale;
  int *err_flag;        // optional device word: XN_DEVERR_WAIT when a bounded wait gave up
  uint32_t wait_polls;  // polls before a stage wait gives up (softmax_staged_kernel)
};

__device__ __forceinline__ int64_t row_limit(const SoftmaxParams &p, int64_t row) {
  if (!p.causal) return p.cols;
  const int64_t lim = p.offset + (row % p.t1) + 1;
  return lim < p.cols ? lim : p.cols;
}

// Paired 16-bit types for the packed (vector) path.
template <typename T>
struct Pair;
template <>
struct Pair<__nv_bfloat16> {
  using T2 = __nv_bfloat162;
  __device__ __forceinline__ static T2 splat(float v) { return __float2bfloat162_rn(v); }
  __device__ __forceinline__ static float2 to_f2(T2 v) { return bf2_to_f2(*reinterpret_cast<uint32_t *>(&v)); }
  __device__ __forceinline__ static T2 from_f2(float a, float b) { return __floats2bfloat162_rn(a, b); }
  __device__ __forceinline__ static T2 neg_inf() { return splat(-INFINITY); }
  static constexpr uint32_t kNegInfBits = 0xff80ff80u, kPosInfBits = 0x7f807f80u, kNanBits = 0x7fc07fc0u;
  // Keeps the low element, sets the high one to -inf.
  __device__ __forceinline__ static T2 mask_high(T2 v) {
    return __halves2bfloat162(__low2bfloat16(v), __float2bfloat16(-INFINITY));
  }
  // Both halves set to the low element.
  __device__ __forceinline__ static T2 low2(T2 v) { return __low2bfloat162(v); }
  __device__ __forceinline__ static T2 high2(T2 v) { return __high2bfloat162(v); }
  // Keeps the high element, sets the low one to -inf.
  __device__ __forceinline__ static T2 mask_low(T2 v) {
    return __halves2bfloat162(__float2bfloat16(-INFINITY), __high2bfloat16(v));
  }
};
template <>
struct Pair<__half> {
  using T2 = __half2;
  __device__ __forceinline__ static T2 splat(float v) { return __float2half2_rn(v); }
  __device__ __forceinline__ static float2 to_f2(T2 v) { return __half22float2(v); }
  __device__ __forceinline__ static T2 from_f2(float a, float b) { return __floats2half2_rn(a, b); }
  __device__ __forceinline__ static T2 neg_inf() { return splat(-INFINITY); }
  static constexpr uint32_t kNegInfBits = 0xfc00fc00u, kPosInfBits = 0x7c007c00u, kNanBits = 0x7e007e00u;
  __device__ __forceinline__ static T2 mask_high(T2 v) {
    return __halves2half2(__low2half(v), __float2half(-INFINITY));
  }
  __device__ __forceinline__ static T2 low2(T2 v) { return __low2half2(v); }
  __device__ __forceinline__ static T2 high2(T2 v) { return __high2half2(v); }
  __device__ __forceinline__ static T2 mask_low(T2 v) {
    return __halves2half2(__float2half(-INFINITY), __high2half(v));
  }
};

// Row accesses: U = uint4 (16 bytes, every dtype) or uint32_t (one 16-bit
// pair, for 16-bit rows of even width whose 16-byte alignment fails).
template <typename U>
__device__ __forceinline__ U load_access(const void *p) {
  if constexpr (sizeof(U) == 16) {
    return ld_stream(p);
  } else {
    U r;
    asm volatile("ld.global.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
  }
}

template <typename U>
__device__ __forceinline__ void store_access(void *p, U v) {
  *reinterpret_cast<U *>(p) = v;
}

// Scalar rows (widths that are not a multiple of the 16-byte vector, or
// unaligned pointers): one row per row group, NV elements per thread held in
// registers. Steps, in the reference's T arithmetic (cpu_backend.rs:667-689):
// [x = T(x * scale)], max, e = T(exp(T(x - max))), sum of f32(e),
// y = T(e / sum). Causal rows (kCausal) treat columns past
// offset + (row % t1) as -inf: they are neither read nor exp'd and give 0.
template <typename T, int NV, bool kCausal>
__global__ void __launch_bounds__(512) softmax_rows_kernel(const SoftmaxParams p) {
  griddep_wait();
  griddep_release();
  __shared__ float red[32];
  const int tpr = p.tpr;
  const int g = threadIdx.x / tpr;
  const int lr = threadIdx.x - g * tpr;
  const int rpb = blockDim.x / tpr;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * rpb + g;
  const bool active = row < p.rows;
  const int cols = static_cast<int>(p.cols);
  int lim = active ? cols : 0;
  if constexpr (kCausal) {
    if (active) {
      const int64_t l = p.offset + (row % p.t1) + 1;
      lim = l < cols ? static_cast<int>(l) : cols;
    }
  }
  const T *src = static_cast<const T *>(p.src) + row * p.cols;
  T *dst = static_cast<T *>(p.dst) + row * p.cols;

  float x[NV];
  float mx = -INFINITY;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int e = lr + k * tpr;
    x[k] = -INFINITY;  // masked and padding entries: exp(-inf - max) = 0
    if (e < lim) {
      x[k] = Elem<T>::to_f32(src[e]);
      if (p.scaled) x[k] = Elem<T>::round(__fmul_rn(x[k], Elem<T>::round(p.scale)));
    }
    mx = fmaxf(mx, x[k]);
  }
  mx = group_max(mx, tpr, red);
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    x[k] = Elem<T>::round(exp_t<T>(Elem<T>::round(__fsub_rn(x[k], mx))));
    s = __fadd_rn(s, x[k]);
  }
  s = group_sum(s, tpr, red);
  const float rs = __frcp_rn(s);
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int e = lr + k * tpr;
    if (active && e < p.nvec) dst[e] = Elem<T>::from_f32(div_by(x[k], s, rs));
  }
}

// Per-thread steps of one vector row, shared by the register-prefetching and
// the shared-memory-staged kernels. `cur` holds the thread's NV vectors of the
// row: vector k starts at element (lr + k * tpr) * N. Vectors starting at or
// past `lim` need not hold data: the first step overwrites them.
//
// For 16-bit T the row stays packed: the max, the subtraction and the scale
// run as paired bf16x2 / f16x2 instructions, which round exactly once as the
// reference's T operations do.

// [x = T(x * scale)] on the live elements, -inf elsewhere, in place; returns
// the thread's maximum. Live elements are the row positions [0, lim); with
// kWin the accesses cover an aligned window around the row and row position 0
// sits at window position `lo` (elements before it belong to the previous
// row), otherwise lo = 0. For 16-bit T, `mn` receives the minimum of the
// thread's live elements (+inf when it has none), which tells softmax_exp
// whether any of its exp results can be subnormal.
// kDead: accesses wholly past `lim` (common with a causal mask or a window)
// are set to -inf at once; otherwise the rare padding access takes the
// per-element path, which keeps the check off the common path.
// kDead without a window (causal rows): the tests are made per slot k, on the
// elements [(g0 + k * tpr) * N, (g0 + k * tpr + tpr) * N) that the row group's
// tpr threads hold in it (g0: the group's first vector), so the whole group
// takes one branch: a dead slot, a live slot, or the one slot holding the
// row's last live element, where each thread masks its access with bit
// selects instead of per-element branches (kSlot: 16-bit rows, where it
// measured faster; f32 rows measured slower with it, and the
// shared-memory-staged kernel keeps the per-thread tests, with which ptxas
// holds its row in registers without spilling).
template <typename T, bool kDead, bool kWin>
constexpr bool kSlotTests = kDead && !kWin && !std::is_same_v<T, float>;

template <typename T, int NV, typename U, bool kWin = false, bool kDead = false,
          bool kSlot = kSlotTests<T, kDead, kWin>>
__device__ __forceinline__ float softmax_prep(U (&cur)[NV], int lr, int tpr, int lim, const SoftmaxParams &p,
                                              float &mn, int lo = 0, int g0 = 0) {
  constexpr int N = static_cast<int>(sizeof(U) / sizeof(T));
  static_assert(!kSlot || (kDead && !kWin), "slot tests are for masked rows without a window");
  const int lo_ = kWin ? lo : 0;
  if constexpr (std::is_same_v<T, float>) {
    static_assert(sizeof(U) == 16, "f32 rows use 16-byte accesses");
    mn = -INFINITY;  // not used for f32
    float m = -INFINITY;
    const float2 sc = splat2(p.scale);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int a0 = (lr + k * tpr) * N - lo_;  // row position of the access's first element
      float2 *x2 = reinterpret_cast<float2 *>(&cur[k]);
      float *x = reinterpret_cast<float *>(&cur[k]);
      if constexpr (kSlot) {
        const int s0 = (g0 + k * tpr) * N;
        if (s0 >= lim) {
          x2[0] = x2[1] = splat2(-INFINITY);
        } else if (s0 + tpr * N <= lim) {
          if (p.scaled) {
            x2[0] = __fmul2_rn(x2[0], sc);
            x2[1] = __fmul2_rn(x2[1], sc);
          }
        } else {
#pragma unroll
          for (int j = 0; j < N; ++j) {
            const float v = p.scaled ? __fmul_rn(x[j], p.scale) : x[j];
            x[j] = a0 + j < lim ? v : -INFINITY;
          }
        }
      } else if (kDead && a0 >= lim) {  // masked, or past the row (a window's spare accesses)
        x2[0] = x2[1] = splat2(-INFINITY);
      } else if ((!kWin || a0 >= 0) && a0 + N <= lim) {
        if (p.scaled) {
          x2[0] = __fmul2_rn(x2[0], sc);
          x2[1] = __fmul2_rn(x2[1], sc);
        }
      } else {  // an access holding a row end, or padding: -inf outside [0, lim)
#pragma unroll
        for (int j = 0; j < N; ++j) {
          if ((!kWin || a0 + j >= 0) && a0 + j < lim) {
            if (p.scaled) x[j] = __fmul_rn(x[j], p.scale);
          } else {
            x[j] = -INFINITY;
          }
        }
      }
      m = fmaxf(m, fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3])));
    }
    return m;
  } else {
    using P = Pair<T>;
    using T2 = typename P::T2;
    constexpr int W = N / 2;
    T2 mx2 = P::neg_inf(), mn2 = P::splat(INFINITY);
    const T2 sc2 = P::splat(p.scale);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int a0 = (lr + k * tpr) * N - lo_;
      T2 *w = reinterpret_cast<T2 *>(&cur[k]);
      if constexpr (kSlot) {
        const int s0 = (g0 + k * tpr) * N;
        if (s0 >= lim) {
#pragma unroll
          for (int j = 0; j < W; ++j) w[j] = P::neg_inf();
        } else if (s0 + tpr * N <= lim) {
#pragma unroll
          for (int j = 0; j < W; ++j) {
            if (p.scaled) w[j] = __hmul2(w[j], sc2);
            mn2 = __hmin2(mn2, w[j]);
          }
        } else {
          // Element 2j of the access is the low half of word j; nl of the
          // access's elements are live (none when nl <= 0).
          const int nl = lim - a0;
#pragma unroll
          for (int j = 0; j < W; ++j) {
            if (p.scaled) w[j] = __hmul2(w[j], sc2);
            const uint32_t m = nl > 2 * j + 1 ? 0xffffffffu : (nl > 2 * j ? 0x0000ffffu : 0u);
            const uint32_t v = *reinterpret_cast<const uint32_t *>(&w[j]);
            const uint32_t live = v & m;
            const uint32_t lo_bits = live | (P::kPosInfBits & ~m);  // +inf where masked, for the minimum
            *reinterpret_cast<uint32_t *>(&w[j]) = live | (P::kNegInfBits & ~m);
            mn2 = __hmin2(mn2, *reinterpret_cast<const T2 *>(&lo_bits));
          }
        }
      } else if (kDead && a0 >= lim) {  // masked, or past the row (a window's spare accesses)
#pragma unroll
        for (int j = 0; j < W; ++j) w[j] = P::neg_inf();
      } else if ((!kWin || a0 >= 0) && a0 + N <= lim) {
#pragma unroll
        for (int j = 0; j < W; ++j) {
          if (p.scaled) w[j] = __hmul2(w[j], sc2);
          mn2 = __hmin2(mn2, w[j]);
        }
      } else {  // an access holding a row end, or padding: -inf outside [0, lim)
#pragma unroll
        for (int j = 0; j < W; ++j) {
          const int ra = a0 + 2 * j;  // row positions of the pair's elements: ra, ra + 1
          const bool la = (!kWin || ra >= 0) && ra < lim, lb = (!kWin || ra + 1 >= 0) && ra + 1 < lim;
          if (la && lb) {
            if (p.scaled) w[j] = __hmul2(w[j], sc2);
            mn2 = __hmin2(mn2, w[j]);
          } else if (la) {
            if (p.scaled) w[j] = __hmul2(w[j], sc2);
            mn2 = __hmin2(mn2, P::low2(w[j]));
            w[j] = P::mask_high(w[j]);
          } else if (kWin && lb) {
            if (p.scaled) w[j] = __hmul2(w[j], sc2);
            mn2 = __hmin2(mn2, P::high2(w[j]));
            w[j] = P::mask_low(w[j]);
          } else {
            w[j] = P::neg_inf();
          }
        }
      }
#pragma unroll
      for (int j = 0; j < W; ++j) mx2 = __hmax2(mx2, w[j]);
    }
    const float2 nf = P::to_f2(mn2);
    mn = fminf(nf.x, nf.y);
    const float2 mf = P::to_f2(mx2);
    return fmaxf(mf.x, mf.y);
  }
}

// Whether access k of thread lr is skipped as wholly masked (kSkip). For
// 16-bit rows without a window the test is per slot (softmax_prep's kSlot),
// the same for the whole row group: the masked accesses of the slot holding
// the row's last live element then take the arithmetic on their -inf
// entries, which gives the same +0.
template <typename T, int NV, bool kSkip, typename U, bool kWin = false>
__device__ __forceinline__ bool access_dead(int lr, int k, int tpr, int lim, int lo, int g0) {
  constexpr int N = static_cast<int>(sizeof(U) / sizeof(T));
  if constexpr (!kSkip)
    return false;
  else if constexpr (kSlotTests<T, kSkip, kWin>)
    return (g0 + k * tpr) * N >= lim;
  else
    return (lr + k * tpr) * N - lo >= lim;
}

// e = T(exp(T(x - mx))) in place (exp(-inf) = 0 for masked and padding
// entries); returns the thread's f32 sum of e, kept as two interleaved partial
// sums. mx is the row maximum, a T value; mn is softmax_prep's minimum.
//
// bf16: exp(d) = 2^(d log2 e) (exp_of_bf16). When mn - mx >= -86, every
// d = T(x - mx) of the thread is >= -86 (rounding is monotonic, and the f32
// difference is within half an f32 ulp of the exact one, which bf16's 0.5
// spacing at 86 absorbs), so 2^(d log2 e) >= 2^-124.1 is normal and the
// flush-to-zero form gives the same values with fewer instructions. Otherwise
// (a row reaching below -86 relative to its max, an infinite input, a NaN)
// the thread takes the form that keeps subnormals.
//
// kSkip: vectors starting at or past `lim` hold only masked entries; they
// become +0 without the arithmetic (the same values and sums: exp(-inf) = +0).
template <typename T, int NV, bool kSkip, typename U, bool kWin = false>
__device__ __forceinline__ float softmax_exp(U (&cur)[NV], float mx, float mn, int lr, int tpr, int lim,
                                             int lo = 0, int g0 = 0) {
  constexpr int N = static_cast<int>(sizeof(U) / sizeof(T));
  const int lo_ = kWin ? lo : 0;
  float2 s2 = make_float2(0.f, 0.f);
  if constexpr (std::is_same_v<T, float>) {
    const float2 nmx = splat2(-mx);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      if (access_dead<T, NV, kSkip, U, kWin>(lr, k, tpr, lim, lo_, g0)) {
        cur[k] = U{};
        continue;
      }
      float2 *x2 = reinterpret_cast<float2 *>(&cur[k]);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float2 d = __fadd2_rn(x2[j], nmx);
        x2[j] = make_float2(expf(d.x), expf(d.y));
        s2 = __fadd2_rn(s2, x2[j]);
      }
    }
  } else {
    using P = Pair<T>;
    using T2 = typename P::T2;
    const T2 m2 = P::splat(mx);  // exact: the max is a T value
    // T(exp(...)) of one T(x - max) pair, by the form `kind` selects.
    auto exp_pair = [](float2 d, auto kind) -> T2 {
      if constexpr (std::is_same_v<T, __nv_bfloat16>) {
        const float2 t = __fmul2_rn(d, splat2(kLog2e));
        if constexpr (decltype(kind)::value)
          return P::from_f2(ex2_approx_ftz(t.x), ex2_approx_ftz(t.y));
        else
          return P::from_f2(ex2_approx(t.x), ex2_approx(t.y));
      } else {
        return P::from_f2(expf(d.x), expf(d.y));
      }
    };
    auto run = [&](auto kind) {
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        if (access_dead<T, NV, kSkip, U, kWin>(lr, k, tpr, lim, lo_, g0)) {
          cur[k] = U{};
          continue;
        }
        T2 *w = reinterpret_cast<T2 *>(&cur[k]);
#pragma unroll
        for (int j = 0; j < N / 2; ++j) {
          const T2 e = exp_pair(P::to_f2(__hsub2(w[j], m2)), kind);  // T(exp(T(x - max)))
          s2 = add2_widen<T>(*reinterpret_cast<const uint32_t *>(&e), s2);
          w[j] = e;
        }
      }
    };
    if (std::is_same_v<T, __nv_bfloat16> && __fsub_rn(mn, mx) >= -86.f)
      run(std::true_type{});
    else
      run(std::false_type{});
  }
  return __fadd_rn(s2.x, s2.y);
}

// y = T(e / s) for the accesses below nvec, stored to the row at dst_row.
// s >= 1 for a live row: its maximum contributes exp(0). kSkip: the accesses
// that softmax_exp skipped hold only masked entries, whose quotient 0 / s is
// +0, stored without the division; or NaN when s is NaN (a live +inf or NaN,
// or a row whose live entries are all -inf: the reference's masked outputs
// are NaN then too). kWin: dst_row points at the window start; accesses that
// reach outside the row's `cols` elements store only the row's own elements.
template <typename T, typename U>
__device__ __forceinline__ U nan_access() {
  uint32_t w = 0x7fc00000u;
  if constexpr (!std::is_same_v<T, float>) w = Pair<T>::kNanBits;
  if constexpr (sizeof(U) == 16)
    return make_uint4(w, w, w, w);
  else
    return w;
}

template <typename T, int NV, bool kSkip, typename U, bool kWin = false>
__device__ __forceinline__ void softmax_store(U (&cur)[NV], float s, T *dst_row, int lr, int tpr, int nvec,
                                              int lim, int lo = 0, int cols = 0, int g0 = 0) {
  constexpr int N = static_cast<int>(sizeof(U) / sizeof(T));
  const int lo_ = kWin ? lo : 0;
  const float2 rs = splat2(__frcp_rn(s)), ns = splat2(-s);
  // f32 rows divide their skipped (+0) accesses too: 0 / s gives the NaN of a
  // NaN sum by itself, and measured faster than a separate NaN pass.
  constexpr bool kSkipDiv = kSkip && !std::is_same_v<T, float>;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int vi = lr + k * tpr;
    if (vi < nvec) {
      const int a0 = vi * N - lo_;
      if (access_dead<T, NV, kSkipDiv, U, kWin>(lr, k, tpr, lim, lo_, g0)) {
        // masked: already +0
      } else if constexpr (std::is_same_v<T, float>) {
        float2 *x2 = reinterpret_cast<float2 *>(&cur[k]);
        x2[0] = div_nonneg2(x2[0], ns, rs);
        x2[1] = div_nonneg2(x2[1], ns, rs);
      } else {
        using P = Pair<T>;
        using T2 = typename P::T2;
        T2 *w = reinterpret_cast<T2 *>(&cur[k]);
#pragma unroll
        for (int j = 0; j < N / 2; ++j) {
          const float2 q = div_nonneg2(P::to_f2(w[j]), ns, rs);
          w[j] = P::from_f2(q.x, q.y);
        }
      }
      if (!kWin || (a0 >= 0 && a0 + N <= cols)) {
        store_access<U>(dst_row + vi * N, cur[k]);
      } else {
        const T *el = reinterpret_cast<const T *>(&cur[k]);
#pragma unroll
        for (int j = 0; j < N; ++j)
          if (a0 + j >= 0 && a0 + j < cols) dst_row[vi * N + j] = el[j];
      }
    }
  }
  if (kSkipDiv && isnan(s)) {
    // Rare, and after the loop so that it costs the loop nothing: with a NaN
    // sum every output of the row is NaN (e / NaN), the skipped ones included.
    const U nan = nan_access<T, U>();
    const T *el = reinterpret_cast<const T *>(&nan);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int vi = lr + k * tpr;
      if (vi < nvec) {
        const int a0 = vi * N - lo_;
        if (!kWin || (a0 >= 0 && a0 + N <= cols)) {
          store_access<U>(dst_row + vi * N, nan);
        } else {
#pragma unroll
          for (int j = 0; j < N; ++j)
            if (a0 + j >= 0 && a0 + j < cols) dst_row[vi * N + j] = el[j];
        }
      }
    }
  }
}

// Vector rows, persistent and prefetching: each row group walks rows
// row, row + step, ... (step = all groups of the grid) and issues the loads of
// its next row before computing the current one, so HBM reads stay in flight
// through the reductions and the exp / divide work. Arithmetic as
// softmax_rows_kernel. The loop bound depends only on the block, so blocks
// whose row groups span several warps keep their __syncthreads uniform.
// Causal rows of 5 or 6 accesses per thread skip the register prefetch
// (kPrefetch): the kernel is issue-bound, and without the second row's
// registers twice the warps are resident (bf16 1536 columns: 0.68 -> 0.77 of
// the copy peak, f32 2560: 0.72 -> 0.77); the plain kernel and the other
// shapes measured the same or better with the prefetch.
template <typename T, int NV, bool kCausal, typename U, bool kWin>
constexpr bool kPipePrefetch = !(kCausal && sizeof(U) == 16 && (NV == 5 || NV == 6));

template <typename T, int NV, bool kCausal, typename U, bool kWin>
__global__ void __launch_bounds__(512, (NV * sizeof(U) >= 80 && kPipePrefetch<T, NV, kCausal, U, kWin>) ? 1 : 2)
    softmax_pipe_kernel(const SoftmaxParams p) {
  griddep_wait();
  griddep_release();
  constexpr int N = static_cast<int>(sizeof(U) / sizeof(T));
  // One scratch array per reduction of a row (see group_sum's kReuse).
  __shared__ float red_max[32], red_sum[32];
  const int tpr = p.tpr;
  const int g = threadIdx.x / tpr;
  const int lr = threadIdx.x - g * tpr;
  const int rpb = blockDim.x / tpr;
  const int64_t step = static_cast<int64_t>(gridDim.x) * rpb;
  const int cols = static_cast<int>(p.cols);
  const T *src = static_cast<const T *>(p.src);
  T *dst = static_cast<T *>(p.dst);
  // Causal rows: the query index q = row % t1 is carried along the walk
  // (row += step means q += step % t1, wrapped), not divided per row.
  // In 32 bits: t1 <= 2^30 (checked on the host) and an offset at or past the
  // row width leaves every row whole, so off + q + 1 and q + q_step stay below 2^31.
  const int t1 = kCausal ? static_cast<int>(p.t1) : 1;
  const int q_step = kCausal ? static_cast<int>(step % t1) : 0;
  const int off = kCausal ? static_cast<int>(p.offset < p.cols ? p.offset : p.cols) : 0;
  // kWin: rows of a width that is not a multiple of N, read through the
  // 16-byte-aligned window around each row. The row starting at element
  // row * cols sits at window position lo = (row * cols) % N, carried along
  // the walk like q. Every loaded 16-byte block holds an element of the
  // tensor, so none reaches past the pages it occupies.
  const int lo_step = kWin ? static_cast<int>((step % N) * (p.cols % N) % N) : 0;
  auto row_lim = [&](int64_t r, int q) -> int {
    if (r >= p.rows) return 0;
    if constexpr (kCausal) {
      const int l = off + q + 1;
      return l < cols ? l : cols;
    } else {
      return cols;
    }
  };
  // lim = 0 marks a row past the end: nothing is loaded (e0 < lim already
  // excludes every access without a window; with one, e0 - lo < 0 would admit
  // the first).
  auto load_row = [&](int64_t r, int lim, int lo, U (&buf)[NV]) {
    if (kWin && lim == 0) return;
    const T *w = src + r * p.cols - lo;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int e0 = (lr + k * tpr) * N;
      if (e0 - lo < lim) buf[k] = load_access<U>(w + e0);
    }
  };
  constexpr bool kPrefetch = kPipePrefetch<T, NV, kCausal, U, kWin>;
  U cur[NV], nxt[kPrefetch ? NV : 1];
  int64_t row = static_cast<int64_t>(blockIdx.x) * rpb + g;
  int q = kCausal ? static_cast<int>(row % t1) : 0;
  int lo = kWin ? static_cast<int>((row % N) * (p.cols % N) % N) : 0;
  int lim = row_lim(row, q);
  load_row(row, lim, lo, cur);
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * rpb; base < p.rows; base += step, row += step) {
    int qn = q + q_step;
    if (qn >= t1) qn -= t1;
    int lon = lo + lo_step;
    if (lon >= N) lon -= N;
    const int lim_next = row_lim(row + step, qn);
    if constexpr (kPrefetch) load_row(row + step, lim_next, lon, nxt);  // prefetch the next row of this group
    float mn;
    const float mx =
        group_max<false>(softmax_prep<T, NV, U, kWin, kCausal || kWin>(cur, lr, tpr, lim, p, mn, lo), tpr, red_max);
    // Window rows skip the arithmetic of their spare accesses like masked ones.
    const float s = group_sum<false>(softmax_exp<T, NV, kCausal || kWin, U, kWin>(cur, mx, mn, lr, tpr, lim, lo),
                                     tpr, red_sum);
    if (row < p.rows) {
      if constexpr (kWin) {
        softmax_store<T, NV, true, U, true>(cur, s, dst + row * p.cols - lo, lr, tpr, (lo + cols + N - 1) / N, lim,
                                            lo, cols);
      } else {
        softmax_store<T, NV, kCausal, U>(cur, s, dst + row * p.cols, lr, tpr, p.nvec, lim);
      }
    }
    if constexpr (kPrefetch) {
#pragma unroll
      for (int k = 0; k < NV; ++k) cur[k] = nxt[k];
    }
    q = qn;
    lo = lon;
    lim = lim_next;
    if constexpr (!kPrefetch) load_row(row + step, lim_next, lon, cur);
  }
}

// Vector rows staged through shared memory: one block per row, persistent over
// rows blockIdx.x, blockIdx.x + gridDim.x, ... Thread 0 streams each row into
// one of `stages` shared-memory buffers with a bulk copy (the TMA engine),
// `stages` rows ahead, so the prefetch depth costs no registers and each
// thread keeps only NV vectors of the current row. Causal rows copy only their
// first `lim` columns (rounded up to the 16-byte vector). Arithmetic as
// softmax_pipe_kernel; the block reductions go through shared memory.
//
// A bulk copy that does not complete within p.wait_polls polls (it cannot
// happen with valid arguments; the limit guards against a hang) makes the
// whole block stop: it waits, bounded by kStageWaitLimit, for its copies still
// in flight (so none lands in shared memory after the block exits), writes NaN
// to every row it has not finished and sets XN_DEVERR_WAIT in the caller's
// error word, so the failure shows in the output and the status instead of as
// a hang.
constexpr int kMaxStages = 4;
constexpr uint32_t kStageWaitLimit = 1u << 22;

template <typename T, int NV, bool kCausal, bool kSkip>
__global__ void __launch_bounds__(512) softmax_staged_kernel(const SoftmaxParams p, int stages,
                                                                              int stage_bytes) {
  griddep_wait();
  griddep_release();
  constexpr int N = Elem<T>::kVec;
  extern __shared__ __align__(128) unsigned char stage_buf[];
  __shared__ uint64_t full[kMaxStages];
  __shared__ float red_max[32], red_sum[32];
  const int tid = threadIdx.x, tpr = blockDim.x, warps = tpr >> 5;
  const int64_t step = gridDim.x;
  const int cols = static_cast<int>(p.cols);
  const T *src = static_cast<const T *>(p.src);
  T *dst = static_cast<T *>(p.dst);
  // Query index tracking as in softmax_pipe_kernel, once for the row being
  // computed (q) and once for the next row to copy (q_in, thread 0 only).
  const int t1 = kCausal ? static_cast<int>(p.t1) : 1;
  const int q_step = kCausal ? static_cast<int>(step % t1) : 0;
  const int off = kCausal ? static_cast<int>(p.offset < p.cols ? p.offset : p.cols) : 0;
  auto lim_of = [&](int q) -> int {
    if constexpr (kCausal) {
      const int l = off + q + 1;
      return l < cols ? l : cols;
    } else {
      return cols;
    }
  };
  auto next_q = [&](int q) -> int {
    q += q_step;
    return q >= t1 ? q - t1 : q;
  };
  int q = kCausal ? static_cast<int>(blockIdx.x % t1) : 0;
  // The copy side's state lives in shared memory: only thread 0 uses it, once
  // per row, and registers stay free for the row values.
  __shared__ int64_t row_in;  // next row to copy
  __shared__ int q_in, s_in;  // its query index and buffer
  auto copy_next = [&]() {  // thread 0
    const int64_t r = row_in;
    const int b = s_in;
    const uint32_t bytes = static_cast<uint32_t>((lim_of(q_in) + N - 1) / N) * 16u;
    bulk_load(stage_buf + static_cast<size_t>(b) * stage_bytes, src + r * p.cols, bytes, &full[b], l2_evict_first());
    row_in = r + step;
    q_in = next_q(q_in);
    s_in = b + 1 == stages ? 0 : b + 1;
  };
  if (tid == 0) {
    for (int b = 0; b < stages; ++b) mbar_init(&full[b], 1);
    mbar_init_fence();
    row_in = blockIdx.x;
    q_in = q;
    s_in = 0;
    for (int b = 0; b < stages && row_in < p.rows; ++b) copy_next();
  }
  __syncthreads();
  int s = 0;
  uint32_t parity = 0;
  for (int64_t row = blockIdx.x; row < p.rows; row += step) {
    const int lim = lim_of(q);
    const bool arrived = mbar_wait(&full[s], parity, p.wait_polls);
    const uint4 *buf = reinterpret_cast<const uint4 *>(stage_buf + static_cast<size_t>(s) * stage_bytes);
    uint4 cur[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int vi = tid + k * tpr;
      if (vi * N < lim) cur[k] = buf[vi];
    }
    float mn;
    float m = softmax_prep<T, NV, uint4, false, kSkip, false>(cur, tid, tpr, lim, p, mn);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((tid & 31) == 0) red_max[tid >> 5] = m;
    // The block barrier of the max also tells every thread whether any wait gave up.
    if (__syncthreads_or(!arrived)) {
      if (tid == 0) {  // let the copies still in flight land before the block exits
        int sw = s;
        uint32_t pw = parity;
        for (int64_t r = row; r < row_in; r += step) {
          mbar_wait(&full[sw], pw, kStageWaitLimit);
          if (++sw == stages) {
            sw = 0;
            pw ^= 1u;
          }
        }
      }
      const uint4 nan4 = std::is_same_v<T, float> ? make_uint4(0x7fc00000u, 0x7fc00000u, 0x7fc00000u, 0x7fc00000u)
                                                  : (std::is_same_v<T, __half> ? make_uint4(0x7e007e00u, 0x7e007e00u,
                                                                                            0x7e007e00u, 0x7e007e00u)
                                                                               : make_uint4(0x7fc07fc0u, 0x7fc07fc0u,
                                                                                            0x7fc07fc0u, 0x7fc07fc0u));
      for (int64_t r = row; r < p.rows; r += step)
        for (int vi = tid; vi < p.nvec; vi += tpr) st_vec(dst + r * p.cols + vi * N, nan4);
      if (tid == 0 && p.err_flag != nullptr) atomicOr(p.err_flag, XN_DEVERR_WAIT);
      return;
    }
    // Every thread has read buffer s: refill it with the row `stages` ahead.
    if (tid == 0 && row_in < p.rows) {
      fence_async_smem();
      copy_next();
    }
    float mx = red_max[0];
    for (int w = 1; w < warps; ++w) mx = fmaxf(mx, red_max[w]);
    // kSkip: masked vectors skip the arithmetic (they become +0 directly). It
    // pays off when rows are mostly masked and costs about 5% when they are
    // mostly live; the launcher picks it from the mask's average live share.
    const float sum = group_sum<false>(softmax_exp<T, NV, kSkip>(cur, mx, mn, tid, tpr, lim), tpr, red_sum);
    softmax_store<T, NV, kSkip>(cur, sum, dst + row * p.cols, tid, tpr, p.nvec, lim);
    if (++s == stages) {
      s = 0;
      parity ^= 1u;
    }
    q = next_q(q);
  }
}

// Vector rows wider than the staged kernel's 64 KB: one thread-block cluster
// of up to kMaxCluster blocks per row (grid.x = rows * cluster size). Block
// rank r holds vectors [r * per, (r + 1) * per) of the row in registers
// (per = blockDim.x * NV), so the row crosses HBM once. Each block reduces its
// part, writes the partial max (then sum) into a slot of every block's shared
// memory through distributed shared memory, and after a cluster barrier
// combines the slots in rank order (deterministic). Arithmetic as
// softmax_pipe_kernel. Every thread reaches both cluster barriers, and after
// the second one blocks read only their own shared memory, so a block may
// exit while the others finish. (A persistent form that walks rows measured
// slower: each row's cluster barriers, which release prior memory accesses,
// then wait for the previous row's global stores.)
constexpr int kMaxCluster = 8;
constexpr int kClusterThreads = 512;
constexpr int kClusterNv = 4;

template <typename T, int NV, bool kCausal>
__global__ void __launch_bounds__(kClusterThreads, 2) softmax_cluster_kernel(const SoftmaxParams p) {
  griddep_wait();
  griddep_release();
  namespace cg = cooperative_groups;
  constexpr int N = Elem<T>::kVec;
  cg::cluster_group cluster = cg::this_cluster();
  const int csize = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  __shared__ float red_max[32], red_sum[32];
  __shared__ float cmax[kMaxCluster], csum[kMaxCluster];
  const int tid = threadIdx.x, tpr = blockDim.x;
  const int64_t row = blockIdx.x / csize;
  const int v0 = rank * tpr * NV;  // first vector of this block
  const int cols = static_cast<int>(p.cols);
  int lim = cols;
  if constexpr (kCausal) {
    const int64_t l = (p.offset < p.cols ? p.offset : p.cols) + row % p.t1 + 1;
    lim = l < cols ? static_cast<int>(l) : cols;
  }
  const T *src = static_cast<const T *>(p.src) + row * p.cols;
  uint4 cur[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int e0 = (v0 + tid + k * tpr) * N;
    if (e0 < lim) cur[k] = ld_stream(src + e0);
  }
  float mn;
  const float m =
      group_max<false>(softmax_prep<T, NV, uint4, false, kCausal>(cur, v0 + tid, tpr, lim, p, mn, 0, v0), tpr,
                       red_max);
  if (tid == 0) {
    for (int r = 0; r < csize; ++r) *cluster.map_shared_rank(&cmax[rank], r) = m;
  }
  cluster.sync();
  float mx = cmax[0];
  for (int r = 1; r < csize; ++r) mx = fmaxf(mx, cmax[r]);
  const float s =
      group_sum<false>(softmax_exp<T, NV, kCausal>(cur, mx, mn, v0 + tid, tpr, lim, 0, v0), tpr, red_sum);
  if (tid == 0) {
    for (int r = 0; r < csize; ++r) *cluster.map_shared_rank(&csum[rank], r) = s;
  }
  cluster.sync();
  float sum = csum[0];
  for (int r = 1; r < csize; ++r) sum = __fadd_rn(sum, csum[r]);
  softmax_store<T, NV, kCausal>(cur, sum, static_cast<T *>(p.dst) + row * p.cols, v0 + tid, tpr, p.nvec, lim, 0, 0,
                                v0);
}

// Rows wider than the register budget: one block per row, three passes; the
// second pass writes T(exp(...)) to dst and the third rescales it in place.
template <typename T>
__global__ void __launch_bounds__(1024) softmax_loop_kernel(const SoftmaxParams p) {
  griddep_wait();
  griddep_release();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t base = row * p.cols;
  const int64_t lim = row_limit(p, row);
  const T *src = static_cast<const T *>(p.src);
  T *dst = static_cast<T *>(p.dst);
  const int tpr = blockDim.x;
  auto load = [&](int64_t c) -> float {
    const float x = Elem<T>::to_f32(src[base + c]);
    return p.scaled ? Elem<T>::round(__fmul_rn(x, Elem<T>::round(p.scale))) : x;
  };
  float mx = -INFINITY;
  for (int64_t c = threadIdx.x; c < lim; c += tpr) mx = fmaxf(mx, load(c));
  mx = group_max(mx, tpr, red);
  float s = 0.f;
  for (int64_t c = threadIdx.x; c < p.cols; c += tpr) {
    float e = 0.f;
    if (c < lim) {
      e = Elem<T>::round(exp_t<T>(Elem<T>::round(__fsub_rn(load(c), mx))));
      s = __fadd_rn(s, e);
    }
    dst[base + c] = Elem<T>::from_f32(e);
  }
  s = group_sum(s, tpr, red);
  for (int64_t c = threadIdx.x; c < p.cols; c += tpr)
    dst[base + c] = Elem<T>::from_f32(__fdiv_rn(Elem<T>::to_f32(dst[base + c]), s));
}

template <typename T, typename U, bool kCausal, bool kWin = false>
bool launch_softmax_pipe(const SoftmaxParams &p, int nv, int block, int64_t grid, cudaStream_t st) {
  switch (nv) {
    case 1: {
      auto k = softmax_pipe_kernel<T, 1, kCausal, U, kWin>;
      launch_k(k, dim3(persistent_grid(k, block, grid)), dim3(block), 0, st, p);
      return true;
    }
    case 2: {
      auto k = softmax_pipe_kernel<T, 2, kCausal, U, kWin>;
      launch_k(k, dim3(persistent_grid(k, block, grid)), dim3(block), 0, st, p);
      return true;
    }
    case 3:
      if constexpr (sizeof(U) == 16) {
        auto k = softmax_pipe_kernel<T, 3, kCausal, U, kWin>;
        launch_k(k, dim3(persistent_grid(k, block, grid)), dim3(block), 0, st, p);
        return true;
      }
      return false;
    case 4: {
      auto k = softmax_pipe_kernel<T, 4, kCausal, U, kWin>;
      launch_k(k, dim3(persistent_grid(k, block, grid)), dim3(block), 0, st, p);
      return true;
    }
    case 5:
      if constexpr (sizeof(U) == 16) {
        auto k = softmax_pipe_kernel<T, 5, kCausal, U, kWin>;
        launch_k(k, dim3(persistent_grid(k, block, grid)), dim3(block), 0, st, p);
        return true;
      }
      return false;
    case 6:
      if constexpr (sizeof(U) == 16) {
        auto k = softmax_pipe_kernel<T, 6, kCausal, U, kWin>;
        launch_k(k, dim3(persistent_grid(k, block, grid)), dim3(block), 0, st, p);
        return true;
      }
      return false;
    case 8: {
      auto k = softmax_pipe_kernel<T, 8, kCausal, U, kWin>;
      launch_k(k, dim3(persistent_grid(k, block, grid)), dim3(block), 0, st, p);
      return true;
    }
    default:
      return false;
  }
}

// How a row is read: whole 16-byte vectors, 16-byte vectors of the aligned
// window around a row whose width is not a multiple of the vector, 16-bit
// element pairs (4 bytes), or single elements.
enum class RowAccess { kScalar, kPair, kWindow, kVector };

// Returns false when no instantiated kernel has this shape (a dispatcher bug).
template <typename T, RowAccess kAccess, bool kCausal>
bool launch_softmax_regs_c(const SoftmaxParams &p, int nv, int block, int64_t grid, cudaStream_t st) {
  if constexpr (kAccess == RowAccess::kVector) {
    return launch_softmax_pipe<T, uint4, kCausal>(p, nv, block, grid, st);
  } else if constexpr (kAccess == RowAccess::kWindow) {
    return launch_softmax_pipe<T, uint4, kCausal, true>(p, nv, block, grid, st);
  } else if constexpr (kAccess == RowAccess::kPair && !std::is_same_v<T, float>) {
    return launch_softmax_pipe<T, uint32_t, kCausal>(p, nv, block, grid, st);
  } else {
    switch (nv) {
      case 1:
        launch_k(softmax_rows_kernel<T, 1, kCausal>, dim3(grid), dim3(block), 0, st, p);
        return true;
      case 2:
        launch_k(softmax_rows_kernel<T, 2, kCausal>, dim3(grid), dim3(block), 0, st, p);
        return true;
      case 4:
        launch_k(softmax_rows_kernel<T, 4, kCausal>, dim3(grid), dim3(block), 0, st, p);
        return true;
      case 8:
        launch_k(softmax_rows_kernel<T, 8, kCausal>, dim3(grid), dim3(block), 0, st, p);
        return true;
      default:
        return false;
    }
  }
}

template <typename T, RowAccess kAccess>
bool launch_softmax_regs(const SoftmaxParams &p, int nv, int block, int64_t grid, cudaStream_t st) {
  return p.causal ? launch_softmax_regs_c<T, kAccess, true>(p, nv, block, grid, st)
                  : launch_softmax_regs_c<T, kAccess, false>(p, nv, block, grid, st);
}

// Shared-memory-staged rows: blocks of up to 512 threads (launch_softmax_staged
// never launches more, for any NV), two stage buffers, 8 vectors per thread by
// default (kStagedNv); launch_softmax_staged takes 5 or 6 instead when they
// leave fewer empty access slots. Used, as measured on B200, for 16-bit rows of
// 256 to 4096 vectors (2048 to 32768 elements) and f32 rows of 2049 to 4096
// vectors (8196 to 16384 elements); narrower rows run as fast or faster in the
// register-prefetching kernel, and 4096 vectors (64 KB) is the widest row the
// 512 threads hold.
constexpr int kStagedNv = 8;
constexpr int64_t kStagedMaxVec = 4096;
constexpr int kStages = 2;

static_assert(kStages <= kMaxStages && kStages * kStagedMaxVec * 16 <= 200 * 1024,
              "the stage buffers must fit in one SM's shared memory");

template <typename T>
constexpr int64_t staged_min_vec() {
  return std::is_same_v<T, float> ? 2049 : 256;
}

template <typename T, bool kCausal, bool kSkip, int NV>
void launch_softmax_staged_nv(SoftmaxParams p, int64_t nvec, cudaStream_t st) {
  auto kernel = softmax_staged_kernel<T, NV, kCausal, kSkip>;
  const int block = static_cast<int>(ceil_div(ceil_div(nvec, NV), 32) * 32);
  const int stage_bytes = static_cast<int>(ceil_div(nvec * 16, 128) * 128);
  const size_t smem = static_cast<size_t>(kStages) * stage_bytes;
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, block, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const int64_t all = static_cast<int64_t>(per_sm) * sm_count();
  const int64_t grid = p.rows < all ? p.rows : all;
  p.tpr = block;
  p.nvec = static_cast<int>(nvec);
  launch_k(kernel, dim3(static_cast<unsigned>(grid)), dim3(block), smem, st, p, kStages, stage_bytes);
}

// Accesses per thread: the fewest access slots (threads rounded up to whole
// warps, times accesses per thread) among 8, 6 and 5, preferring 8. Every slot
// is issued whether or not it holds data, so rows of 320, 384 or 640 vectors
// (2560, 3072 and 5120 16-bit columns) take 5, 6 and 5 per thread with no
// empty slot instead of 8 with 37, 25 and 17% of them empty.
template <typename T, bool kCausal, bool kSkip>
void launch_softmax_staged(SoftmaxParams p, int64_t nvec, cudaStream_t st) {
  auto slots = [nvec](int nv) { return ceil_div(ceil_div(nvec, nv), 32) * 32 * nv; };
  const int64_t s8 = slots(kStagedNv), s6 = slots(6), s5 = slots(5);
  if (s5 < s8 && s5 < s6 && ceil_div(nvec, 5) <= 512)
    launch_softmax_staged_nv<T, kCausal, kSkip, 5>(p, nvec, st);
  else if (s6 < s8 && ceil_div(nvec, 6) <= 512)
    launch_softmax_staged_nv<T, kCausal, kSkip, 6>(p, nvec, st);
  else
    launch_softmax_staged_nv<T, kCausal, kSkip, kStagedNv>(p, nvec, st);
}

// One cluster of `csize` blocks per row, launched with programmatic dependent
// launch allowed as launch_k does.
template <auto kKernel>
void launch_softmax_cluster(const SoftmaxParams &p, int csize, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.rows * csize));
  cfg.blockDim = dim3(kClusterThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(csize);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  cudaLaunchKernelEx(&cfg, kKernel, p);
}

template <typename T>
int launch_softmax(SoftmaxParams p, cudaStream_t st) {
  constexpr int V = Elem<T>::kVec;
  const bool vec = p.cols % V == 0 && is_aligned16(p.dst) && is_aligned16(p.src);
  // Rows whose width is not a multiple of the vector (such as 250 attention
  // scores) in 16-byte-aligned tensors: 16-byte accesses over the aligned
  // window around each row, one access more than a vector row.
  const bool win = !vec && is_aligned16(p.dst) && is_aligned16(p.src) && p.cols >= V;
  // 16-bit rows of even width in tensors aligned to 4 bytes only: element
  // pairs, the same paired arithmetic with 4-byte accesses.
  const bool pair = !vec && !win && !std::is_same_v<T, float> && p.cols % 2 == 0 &&
                    (reinterpret_cast<uintptr_t>(p.dst) & 3u) == 0 && (reinterpret_cast<uintptr_t>(p.src) & 3u) == 0;
  const int n = (vec || win) ? V : (pair ? 2 : 1);
  // A window row spans up to ceil((V - 1 + cols) / V) vectors (its first
  // element at window position V - 1 at worst).
  const int64_t nvec = win ? (p.cols + 2 * V - 2) / V : p.cols / n;
  if (vec && nvec >= staged_min_vec<T>() && nvec <= kStagedMaxVec) {
    // Causal rows hold offset + q + 1 live columns, q = 0 .. t1 - 1: skip the
    // masked vectors when fewer than 3/4 of the columns are live on average
    // (square prefill masks are half live).
    const bool mostly_masked = p.causal && 4 * (2 * p.offset + p.t1 + 1) < 3 * 2 * p.cols;
    if (!p.causal)
      launch_softmax_staged<T, false, false>(p, nvec, st);
    else if (mostly_masked)
      launch_softmax_staged<T, true, true>(p, nvec, st);
    else
      launch_softmax_staged<T, true, false>(p, nvec, st);
    return check_launch("xn_softmax");
  }
  // exp needs more registers than the norms: groups of up to 512 threads with
  // up to 32 row values each keep rows of up to 16384 elements in registers.
  const int nv_cap = (32 / n) < 8 ? (32 / n) : 8;
  if (nvec <= 512LL * nv_cap) {
    int64_t tpr = pow2_ceil(ceil_div(nvec, 4));
    if (tpr > 512) tpr = 512;
    // Rows of more than 128 vectors (1024 16-bit or 512 f32 elements): 8
    // vectors per thread (the 128-register shape), so rows of up to 256
    // vectors sit in one warp and longer ones span half as many warps, with
    // fewer block barriers per row.
    if ((vec || win) && nvec > 128) tpr = pow2_ceil(ceil_div(nvec, 8));
    // Window rows of 17-64 vectors (Mimi's 250 attention columns: 33 bf16 / 64
    // f32 vectors) in groups of 8 threads with 5-8 accesses each rather than 16
    // with 3-4: fewer shuffle steps per row (bf16 250 columns: 0.41 -> 0.46 of
    // the copy peak, f32 0.73 -> 0.80, causal 0.39 -> 0.48 / 0.69 -> 0.76).
    // Whole-vector rows of that size measured slower so, and keep the wider groups.
    if (win && nvec > 16 && nvec <= 64) tpr = pow2_ceil(ceil_div(nvec, 8));
    // Pairs are 4-byte registers: 8 per thread cost little and halve the
    // reduction steps per element.
    if (pair) tpr = pow2_ceil(ceil_div(nvec, 8));
    int nv = static_cast<int>(pow2_ceil(ceil_div(nvec, tpr)));
    // Rows of 17-24 vectors per 8, 33-48 per 16, 65-96 per 32 threads (Mimi's
    // 250 attention columns through the window: 33; 768 16-bit columns: 96):
    // 3 accesses per thread instead of 4. Every access slot is issued whether
    // or not a lane holds data in it, so the fourth, empty in every lane,
    // would cost as much as a live one.
    if ((vec || win) && ceil_div(nvec, tpr) == 3) nv = 3;
    // Likewise 5 or 6 vectors per thread (rows of 1536 16-bit columns, of 768,
    // 1280, 1536, 2560, 3072 or 5120 f32 columns) take 5 or 6 slots instead
    // of 8.
    if ((vec || win) && nv == 8 && ceil_div(nvec, tpr) <= 6) nv = static_cast<int>(ceil_div(nvec, tpr));
    const int block = tpr < 256 ? 256 : static_cast<int>(tpr);
    const int64_t grid = ceil_div(p.rows, block / tpr);
    if (grid > 0x7fffffffLL) return fail(XN_E_INVALID, "xn_softmax: too many rows");
    p.tpr = static_cast<int>(tpr);
    p.nvec = static_cast<int>(nvec);
    const bool launched = vec    ? launch_softmax_regs<T, RowAccess::kVector>(p, nv, block, grid, st)
                          : win  ? launch_softmax_regs<T, RowAccess::kWindow>(p, nv, block, grid, st)
                          : pair ? launch_softmax_regs<T, RowAccess::kPair>(p, nv, block, grid, st)
                                 : launch_softmax_regs<T, RowAccess::kScalar>(p, nv, block, grid, st);
    if (!launched) return fail(XN_E_INVALID, "xn_softmax: internal error, no kernel for %d accesses per thread", nv);
  } else if (vec && nvec <= static_cast<int64_t>(kMaxCluster) * kClusterThreads * kClusterNv) {
    int csize = 2;
    while (static_cast<int64_t>(csize) * kClusterThreads * kClusterNv < nvec) csize *= 2;
    if (p.rows * csize > 0x7fffffffLL) return fail(XN_E_INVALID, "xn_softmax: too many rows");
    p.nvec = static_cast<int>(nvec);
    if (p.causal)
      launch_softmax_cluster<softmax_cluster_kernel<T, kClusterNv, true>>(p, csize, st);
    else
      launch_softmax_cluster<softmax_cluster_kernel<T, kClusterNv, false>>(p, csize, st);
  } else {
    if (p.rows > 0x7fffffffLL) return fail(XN_E_INVALID, "xn_softmax: too many rows");
    launch_k(softmax_loop_kernel<T>, dim3(static_cast<unsigned>(p.rows)), dim3(1024), 0, st, p);
  }
  return check_launch("xn_softmax");
}

// One warp per row i of a slice writes -inf to columns (offset + i, t2):
// 16-byte stores over the part of that range that is 16-byte aligned, element
// stores for the ends. Only the mrows = min(t1, t2 - offset - 1) rows of a
// slice that hold a masked column get a warp (grid.x, 8 per block); grid.y
// covers the bh slices (striding past 65535), so no thread divides by t1 and
// the blocks, in launch order, walk the tensor in memory order.
// I: the index type within a row and a slice, int when t1, t2 and the offset
// are below 2^30 (then first + 32 * N and every other index stay below 2^31),
// else int64_t; the row's base pointer is always formed in 64 bits.
template <typename T, typename I>
__global__ void __launch_bounds__(256) causal_mask_kernel(void *dst, int64_t bh, int64_t t1, int64_t t2,
                                                          int64_t offset, int64_t mrows) {
  griddep_wait();
  griddep_release();
  constexpr int N = Elem<T>::kVec;
  const I i = static_cast<I>(blockIdx.x) * 8 + static_cast<I>(threadIdx.x >> 5);
  if (i >= static_cast<I>(mrows)) return;
  const int lane = threadIdx.x & 31;
  const I w = static_cast<I>(t2);
  const I first = static_cast<I>(offset) + i + 1;  // < t2, as i < mrows
  const T ninf = Elem<T>::from_f32(-INFINITY);
  uint4 v;
  T *vt = reinterpret_cast<T *>(&v);
#pragma unroll
  for (int j = 0; j < N; ++j) vt[j] = ninf;
  for (int64_t b = blockIdx.y; b < bh; b += gridDim.y) {
    T *d = static_cast<T *>(dst) + (b * t1 + static_cast<int64_t>(i)) * t2;
    // [first, body0): head, [body0, body1): whole aligned vectors, [body1, t2): tail.
    const I mis = static_cast<I>((reinterpret_cast<uintptr_t>(d + first) & 15u) / sizeof(T));
    I body0 = mis == 0 ? first : first + (N - mis);
    if (body0 > w) body0 = w;
    const I body1 = body0 + ((w - body0) & ~static_cast<I>(N - 1));  // w - body0 >= 0
    if (first + lane < body0) d[first + lane] = ninf;  // the head is shorter than N <= 8 elements
    for (I c = body0 + static_cast<I>(lane) * N; c < body1; c += 32 * N) st_vec(d + c, v);
    if (body1 + lane < w) d[body1 + lane] = ninf;  // so is the tail
  }
}

// Rows of whole 16-byte vectors (t2 a multiple of the vector, dst 16-byte
// aligned): a warp per masked row as above, its lanes walking only the row's
// masked vectors from the one holding the first masked column. That vector
// keeps its live elements: lane 0 rewrites it (no other thread touches it), and
// the vectors after it are whole -inf stores. (Element stores of its masked
// part, one lane each, avoid the read but measured slower from 262144 rows:
// bf16 1024 columns 0.71 -> 0.63 of the copy peak.) t2 < 2^30 (checked on the host),
// so every in-row index is an int; the row base is formed in 64 bits.
template <typename T>
__global__ void __launch_bounds__(256) causal_mask_vec_kernel(void *dst, int64_t bh, int64_t t1, int t2v,
                                                              int64_t offset, int64_t mrows) {
  griddep_wait();
  griddep_release();
  constexpr int N = Elem<T>::kVec;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (i >= mrows) return;
  const int lane = threadIdx.x & 31;
  const int first = static_cast<int>(offset + i + 1);  // first masked column, < t2
  const int vf = first / N, rem = first - vf * N;
  const T ninf = Elem<T>::from_f32(-INFINITY);
  uint4 v;
  T *vt = reinterpret_cast<T *>(&v);
#pragma unroll
  for (int j = 0; j < N; ++j) vt[j] = ninf;
  const int v0 = rem != 0 ? vf + 1 : vf;  // first whole masked vector
  for (int64_t b = blockIdx.y; b < bh; b += gridDim.y) {
    uint4 *row = reinterpret_cast<uint4 *>(static_cast<T *>(dst) + (b * t1 + i) * static_cast<int64_t>(t2v) * N);
    if (rem != 0 && lane == 0) {
      uint4 w = row[vf];
      T *wt = reinterpret_cast<T *>(&w);
#pragma unroll
      for (int j = 0; j < N; ++j)
        if (j >= rem) wt[j] = ninf;
      row[vf] = w;
    }
    for (int c = v0 + lane; c < t2v; c += 32) row[c] = v;
  }
}

}  // namespace
}  // namespace xn

namespace xn {
namespace {
// Polls of a stage wait before it gives up: kStageWaitLimit, or the value of
// the environment variable XN_STAGE_WAIT_POLLS (read once per process), a
// diagnostic that lets a test make the wait give up on valid inputs.
uint32_t stage_wait_polls() {
  static const uint32_t polls = [] {
    const char *v = std::getenv("XN_STAGE_WAIT_POLLS");
    if (v == nullptr || *v == '\0') return kStageWaitLimit;
    const unsigned long n = std::strtoul(v, nullptr, 10);
    return n < kStageWaitLimit ? static_cast<uint32_t>(n) : kStageWaitLimit;
  }();
  return polls;
}

int softmax_entry(void *dst, const void *src, int64_t rows, int64_t cols, int scaled, float scale, int causal,
                  int64_t t1, int64_t offset, int dtype, void *stream, int *err_flag = nullptr) {
  if (!is_float_dtype(dtype)) return fail(XN_E_DTYPE, "xn_softmax: unsupported dtype %d", dtype);
  if (rows < 0 || cols < 0) return fail(XN_E_INVALID, "xn_softmax: negative size");
  if (causal && (t1 <= 0 || offset < 0 || rows % t1 != 0))
    return fail(XN_E_INVALID, "xn_softmax: causal mask needs t1 > 0 dividing rows and offset >= 0 (rows=%lld t1=%lld offset=%lld)",
                (long long)rows, (long long)t1, (long long)offset);
  if (causal && t1 > (int64_t{1} << 30))
    return fail(XN_E_INVALID, "xn_softmax: t1 = %lld query rows per slice exceeds 2^30", (long long)t1);
  if (rows == 0 || cols == 0) return ok();
  if (dst == nullptr || src == nullptr) return fail(XN_E_INVALID, "xn_softmax: null dst or src");
  SoftmaxParams p{dst,   src,   rows,   cols, causal ? t1 : 1, causal ? offset : 0, causal ? 1 : 0, 0, 0,
                  scaled, scale, err_flag, stage_wait_polls()};
  XN_DISPATCH_FLOAT(dtype, return launch_softmax<T>(p, as_stream(stream)));
  return fail(XN_E_DTYPE, "xn_softmax: unsupported dtype %d", dtype);
}
}  // namespace
}  // namespace xn

extern "C" {


int xn_softmax(void *dst, const void *src, int64_t rows, int64_t cols, int causal, int64_t t1,
               int64_t offset, int dtype, void *stream) {
  return xn::softmax_entry(dst, src, rows, cols, 0, 1.f, causal, t1, offset, dtype, stream);
}

int xn_softmax_scaled(void *dst, const void *src, int64_t rows, int64_t cols, float scale, int causal, int64_t t1,
                      int64_t offset, int dtype, void *stream) {
  return xn::softmax_entry(dst, src, rows, cols, 1, scale, causal, t1, offset, dtype, stream);
}

int xn_softmax_status(void *dst, const void *src, int64_t rows, int64_t cols, int scaled, float scale, int causal,
                      int64_t t1, int64_t offset, int *err_flag, int dtype, void *stream) {
  return xn::softmax_entry(dst, src, rows, cols, scaled ? 1 : 0, scale, causal, t1, offset, dtype, stream, err_flag);
}

int xn_causality_mask(void *dst, int64_t bh, int64_t t1, int64_t t2, int64_t offset, int dtype,
                      void *stream) {
  using namespace xn;
  if (!is_float_dtype(dtype)) return fail(XN_E_DTYPE, "xn_causality_mask: unsupported dtype %d", dtype);
  if (bh < 0 || t1 < 0 || t2 < 0 || offset < 0) return fail(XN_E_INVALID, "xn_causality_mask: negative size");
  if (bh == 0 || t1 == 0 || t2 == 0) return ok();
  if (dst == nullptr) return fail(XN_E_INVALID, "xn_causality_mask: null dst");
  // Rows i of a slice with a masked column: offset + i + 1 < t2.
  const int64_t mrows = t2 - offset - 1 < t1 ? t2 - offset - 1 : t1;
  if (mrows <= 0) return ok();
  const int64_t gx = ceil_div(mrows, 8);
  if (gx > 0x7fffffffLL) return fail(XN_E_INVALID, "xn_causality_mask: too many rows");
  const int64_t gy = bh < 65535 ? bh : 65535;
  const dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy));
  const bool narrow = t1 < (int64_t{1} << 30) && t2 < (int64_t{1} << 30) && offset < (int64_t{1} << 30);
  // Whole-vector rows: t2 a multiple of the 16-byte vector and dst aligned.
  const bool vec_rows = narrow && is_aligned16(dst) && (t2 * dtype_bytes(dtype)) % 16 == 0;
  XN_DISPATCH_FLOAT(dtype, if (vec_rows) launch_k(causal_mask_vec_kernel<T>, grid, dim3(256), 0, as_stream(stream), dst, bh, t1, static_cast<int>(t2 / Elem<T>::kVec), offset, mrows);
                    else if (narrow) launch_k(causal_mask_kernel<T, int>, grid, dim3(256), 0, as_stream(stream), dst, bh, t1, t2, offset, mrows);
                    else launch_k(causal_mask_kernel<T, int64_t>, grid, dim3(256), 0, as_stream(stream), dst, bh, t1, t2, offset, mrows);
                    return check_launch("xn_causality_mask"));
  return fail(XN_E_DTYPE, "xn_causality_mask: unsupported dtype %d", dtype);
}

}  // extern "C"
