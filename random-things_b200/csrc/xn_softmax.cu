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
// group reductions. Rows wider than 16384 elements use a three-pass kernel.
#include <math.h>

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
};

__device__ __forceinline__ int64_t row_limit(const SoftmaxParams &p, int64_t row) {
  if (!p.causal) return p.cols;
  const int64_t lim = p.offset + (row % p.t1) + 1;
  return lim < p.cols ? lim : p.cols;
}

template <typename T, bool kVector, int NV>
__global__ void __launch_bounds__(512) softmax_regs_kernel(const SoftmaxParams p) {
  constexpr int N = kVector ? Elem<T>::kVec : 1;
  __shared__ float red[32];
  const int tpr = p.tpr;
  const int g = threadIdx.x / tpr;
  const int lr = threadIdx.x - g * tpr;
  const int rpb = blockDim.x / tpr;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * rpb + g;
  const bool active = row < p.rows;
  const int64_t base = row * p.cols;
  const int64_t lim = active ? row_limit(p, row) : 0;
  const T *src = static_cast<const T *>(p.src);
  T *dst = static_cast<T *>(p.dst);

  float x[NV][N];
  float mx = -INFINITY;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int64_t e0 = static_cast<int64_t>(lr + k * tpr) * N;
    if (active && lr + k * tpr < p.nvec && e0 < lim) {
      if constexpr (kVector) {
        unpack<T>(ld_stream(src + base + e0), x[k]);
      } else {
        x[k][0] = Elem<T>::to_f32(src[base + e0]);
      }
#pragma unroll
      for (int j = 0; j < N; ++j) {
        if (e0 + j >= lim) {
          x[k][j] = -INFINITY;
        } else if (p.scaled) {
          x[k][j] = Elem<T>::round(__fmul_rn(x[k][j], p.scale));
        }
        mx = fmaxf(mx, x[k][j]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < N; ++j) x[k][j] = -INFINITY;
    }
  }
  mx = group_max(mx, tpr, red);
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int64_t e0 = static_cast<int64_t>(lr + k * tpr) * N;
#pragma unroll
    for (int j = 0; j < N; ++j) {
      if (e0 + j < lim) {
        x[k][j] = Elem<T>::round(expf(Elem<T>::round(__fsub_rn(x[k][j], mx))));
        s = __fadd_rn(s, x[k][j]);
      } else {
        x[k][j] = 0.f;
      }
    }
  }
  s = group_sum(s, tpr, red);
  const float rs = __frcp_rn(s);  // s >= 1: the row maximum contributes exp(0)
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int vi = lr + k * tpr;
    if (active && vi < p.nvec) {
      const int64_t e0 = static_cast<int64_t>(vi) * N;
      float y[N];
#pragma unroll
      for (int j = 0; j < N; ++j) y[j] = e0 + j < lim ? div_by(x[k][j], s, rs) : 0.f;
      if constexpr (kVector) {
        st_vec(dst + base + e0, pack<T>(y));
      } else {
        dst[base + e0] = Elem<T>::from_f32(y[0]);
      }
    }
  }
}

// Rows wider than the register budget: one block per row, three passes; the
// second pass writes T(exp(...)) to dst and the third rescales it in place.
template <typename T>
__global__ void __launch_bounds__(1024) softmax_loop_kernel(const SoftmaxParams p) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t base = row * p.cols;
  const int64_t lim = row_limit(p, row);
  const T *src = static_cast<const T *>(p.src);
  T *dst = static_cast<T *>(p.dst);
  const int tpr = blockDim.x;
  auto load = [&](int64_t c) -> float {
    const float x = Elem<T>::to_f32(src[base + c]);
    return p.scaled ? Elem<T>::round(__fmul_rn(x, p.scale)) : x;
  };
  float mx = -INFINITY;
  for (int64_t c = threadIdx.x; c < lim; c += tpr) mx = fmaxf(mx, load(c));
  mx = group_max(mx, tpr, red);
  float s = 0.f;
  for (int64_t c = threadIdx.x; c < p.cols; c += tpr) {
    float e = 0.f;
    if (c < lim) {
      e = Elem<T>::round(expf(Elem<T>::round(__fsub_rn(load(c), mx))));
      s = __fadd_rn(s, e);
    }
    dst[base + c] = Elem<T>::from_f32(e);
  }
  s = group_sum(s, tpr, red);
  for (int64_t c = threadIdx.x; c < p.cols; c += tpr)
    dst[base + c] = Elem<T>::from_f32(__fdiv_rn(Elem<T>::to_f32(dst[base + c]), s));
}

// Returns false when no instantiated kernel has this shape (a dispatcher bug).
template <typename T, bool kVector>
bool launch_softmax_regs(const SoftmaxParams &p, int nv, int block, int64_t grid, cudaStream_t st) {
  constexpr int N = kVector ? Elem<T>::kVec : 1;
  switch (nv) {
    case 1:
      softmax_regs_kernel<T, kVector, 1><<<grid, block, 0, st>>>(p);
      return true;
    case 2:
      softmax_regs_kernel<T, kVector, 2><<<grid, block, 0, st>>>(p);
      return true;
    case 4:
      softmax_regs_kernel<T, kVector, 4><<<grid, block, 0, st>>>(p);
      return true;
    case 8:
      if constexpr (8 * N <= 32) {
        softmax_regs_kernel<T, kVector, 8><<<grid, block, 0, st>>>(p);
        return true;
      }
      return false;
    default:
      return false;
  }
}

template <typename T>
int launch_softmax(SoftmaxParams p, cudaStream_t st) {
  constexpr int V = Elem<T>::kVec;
  const bool vec = p.cols % V == 0 && is_aligned16(p.dst) && is_aligned16(p.src);
  const int n = vec ? V : 1;
  const int64_t nvec = p.cols / n;
  // exp needs more registers than the norms: groups of up to 512 threads with
  // up to 32 row values each keep rows of up to 16384 elements in registers.
  const int nv_cap = (32 / n) < 8 ? (32 / n) : 8;
  if (nvec <= 512LL * nv_cap) {
    int64_t tpr = pow2_ceil(ceil_div(nvec, 4));
    if (tpr > 512) tpr = 512;
    const int nv = static_cast<int>(pow2_ceil(ceil_div(nvec, tpr)));
    const int block = tpr < 256 ? 256 : static_cast<int>(tpr);
    const int64_t grid = ceil_div(p.rows, block / tpr);
    if (grid > 0x7fffffffLL) return fail(XN_E_INVALID, "xn_softmax: too many rows");
    p.tpr = static_cast<int>(tpr);
    p.nvec = static_cast<int>(nvec);
    const bool launched = vec ? launch_softmax_regs<T, true>(p, nv, block, grid, st)
                              : launch_softmax_regs<T, false>(p, nv, block, grid, st);
    if (!launched) return fail(XN_E_INVALID, "xn_softmax: internal error, no kernel for %d accesses per thread", nv);
  } else {
    if (p.rows > 0x7fffffffLL) return fail(XN_E_INVALID, "xn_softmax: too many rows");
    softmax_loop_kernel<T><<<static_cast<unsigned>(p.rows), 1024, 0, st>>>(p);
  }
  return check_launch("xn_softmax");
}

// One warp per (b, i) row writes -inf to columns (offset + i, t2).
template <typename T>
__global__ void __launch_bounds__(256) causal_mask_kernel(void *dst, int64_t rows, int64_t t1,
                                                          int64_t t2, int64_t offset) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int64_t first = offset + (row % t1) + 1;
  T *d = static_cast<T *>(dst) + row * t2;
  const T ninf = Elem<T>::from_f32(-INFINITY);
  for (int64_t c = first + (threadIdx.x & 31); c < t2; c += 32) d[c] = ninf;
}

}  // namespace
}  // namespace xn

namespace xn {
namespace {
int softmax_entry(void *dst, const void *src, int64_t rows, int64_t cols, int scaled, float scale, int causal,
                  int64_t t1, int64_t offset, int dtype, void *stream) {
  if (!is_float_dtype(dtype)) return fail(XN_E_DTYPE, "xn_softmax: unsupported dtype %d", dtype);
  if (rows < 0 || cols < 0) return fail(XN_E_INVALID, "xn_softmax: negative size");
  if (causal && (t1 <= 0 || offset < 0 || rows % t1 != 0))
    return fail(XN_E_INVALID, "xn_softmax: causal mask needs t1 > 0 dividing rows and offset >= 0 (rows=%lld t1=%lld offset=%lld)",
                (long long)rows, (long long)t1, (long long)offset);
  if (rows == 0 || cols == 0) return ok();
  if (dst == nullptr || src == nullptr) return fail(XN_E_INVALID, "xn_softmax: null dst or src");
  SoftmaxParams p{dst, src, rows, cols, causal ? t1 : 1, causal ? offset : 0, causal ? 1 : 0, 0, 0, scaled, scale};
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

int xn_causality_mask(void *dst, int64_t bh, int64_t t1, int64_t t2, int64_t offset, int dtype,
                      void *stream) {
  using namespace xn;
  if (!is_float_dtype(dtype)) return fail(XN_E_DTYPE, "xn_causality_mask: unsupported dtype %d", dtype);
  if (bh < 0 || t1 < 0 || t2 < 0 || offset < 0) return fail(XN_E_INVALID, "xn_causality_mask: negative size");
  const int64_t rows = bh * t1;
  if (rows == 0 || t2 == 0) return ok();
  if (dst == nullptr) return fail(XN_E_INVALID, "xn_causality_mask: null dst");
  const int64_t grid = ceil_div(rows, 8);
  if (grid > 0x7fffffffLL) return fail(XN_E_INVALID, "xn_causality_mask: too many rows");
  XN_DISPATCH_FLOAT(dtype, causal_mask_kernel<T><<<grid, 256, 0, as_stream(stream)>>>(dst, rows, t1, t2, offset);
                    return check_launch("xn_causality_mask"));
  return fail(XN_E_DTYPE, "xn_causality_mask: unsupported dtype %d", dtype);
}

}  // extern "C"
