// xn_norm.cu - RMSNorm and LayerNorm over the last dimension, each with an
// optional fused residual add and layer-scale multiply, for sm_100a.
//
// Reference semantics: mimi-rs/src/cpu_backend.rs:691-709 (rms_norm) and
// :711-750 (layer_norm); the fused prologue restates the composite
// `LayerScale::forward` (broadcast_mul, cpu_backend.rs:1379-1387) followed by
// `Tensor::add` (binary Add, cpu_backend.rs:224-258) from
// mimi-rs/src/models/mimi.rs:1433-1439 and llama.rs:310-313.
//
// Design: a row is owned by a "row group" of tpr threads (power of two). The
// whole row is loaded into registers with 16-byte vector loads (NV vectors per
// thread), so every tensor crosses HBM exactly once: read src (+ branch),
// write residual_out (+ dst). The reductions are f32 shuffles inside the group
// (plus one shared-memory step when the group spans several warps). Rows too
// wide for registers (more than 4096 16-byte vectors: 32768 bf16 / 16384 f32
// elements) use a multi-pass kernel that re-reads the row from L2.
#include <type_traits>

#include "xn_common.cuh"
#include "xn_internal.h"

namespace xn {
namespace {

struct NormParams {
  void *dst;
  const void *src;
  const void *w;       // RMS alpha or LN weight (NULL = ones)
  const void *b;       // LN bias (NULL = zeros)
  const void *branch;  // optional residual branch
  const void *ls;      // optional layer scale [cols]
  void *res_out;       // optional residual output
  int64_t rows;
  int64_t cols;
  float eps;
  int remove_mean;
  int tpr;   // threads per row
  int nvec;  // accesses per row
};

// Scalar rows (widths that are not a multiple of the 16-byte vector, or
// unaligned pointers): one row per row group of tpr threads, NV elements per
// thread held in registers. All loads of a thread (src, then branch) are
// issued before any store; stores of residual_out / dst come last, which also
// makes exact aliasing of dst or residual_out with src safe. The arithmetic
// is the vector kernel's, one element at a time.
template <typename T, int NV, bool kLN, int kMaxBlock, bool kBranch>
__global__ void __launch_bounds__(kMaxBlock, kMaxBlock == 256 ? 4 : 1) norm_rows_kernel(const NormParams p) {
  griddep_wait();
  griddep_release();
  __shared__ float red[32];
  const int tpr = p.tpr;
  const int g = threadIdx.x / tpr;
  const int lr = threadIdx.x - g * tpr;
  const int rpb = blockDim.x / tpr;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * rpb + g;
  const bool active = row < p.rows;
  const int64_t base = row * p.cols;
  const T *src = static_cast<const T *>(p.src) + base;

  // 1) h = src (+ T(branch * ls)), each op rounded to T; invalid slots hold 0.
  float h[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int e = lr + k * tpr;
    h[k] = (active && e < p.nvec) ? Elem<T>::to_f32(src[e]) : 0.f;
  }
  if constexpr (kBranch) {
    const T *br = static_cast<const T *>(p.branch) + base;
    float b[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int e = lr + k * tpr;
      b[k] = (active && e < p.nvec) ? Elem<T>::to_f32(br[e]) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int e = lr + k * tpr;
      if (active && e < p.nvec) {
        float y = b[k];
        if (p.ls != nullptr) y = Elem<T>::round(__fmul_rn(y, ld_elem<T>(p.ls, e)));
        h[k] = Elem<T>::round(__fadd_rn(h[k], y));
        if (p.res_out != nullptr) st_elem<T>(p.res_out, base + e, h[k]);
      }
    }
  }

  // 2) Row statistics in f32, then 3) dst = T(norm(h) * w (+ b)).
  const float cols_f = __ll2float_rn(p.cols);
  if constexpr (kLN) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) s = __fadd_rn(s, h[k]);
    const float mean = __fdiv_rn(group_sum(s, tpr, red), cols_f);
    float v = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      if (lr + k * tpr < p.nvec) {
        const float d = __fsub_rn(h[k], mean);
        v = __fmaf_rn(d, d, v);
      }
    }
    const float var = __fdiv_rn(group_sum(v, tpr, red), cols_f);
    const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(var, p.eps)));
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int e = lr + k * tpr;
      if (active && e < p.nvec) {
        const float w = p.w != nullptr ? ld_elem<T>(p.w, e) : 1.f;
        const float b = p.b != nullptr ? ld_elem<T>(p.b, e) : 0.f;
        const float c = p.remove_mean ? __fsub_rn(h[k], mean) : h[k];
        st_elem<T>(p.dst, base + e, __fadd_rn(__fmul_rn(__fmul_rn(c, inv), w), b));
      }
    }
  } else {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) s = __fmaf_rn(h[k], h[k], s);
    const float m = __fsqrt_rn(__fadd_rn(__fdiv_rn(group_sum(s, tpr, red), cols_f), p.eps));
    const float r = __frcp_rn(m);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int e = lr + k * tpr;
      if (active && e < p.nvec) {
        const float w = p.w != nullptr ? ld_elem<T>(p.w, e) : 1.f;
        // T(x / m * alpha): the IEEE quotient x / m via div_by, then * alpha.
        st_elem<T>(p.dst, base + e, __fmul_rn(div_by(h[k], m, r), w));
      }
    }
  }
}

// The 16-byte vector path. Same row-group structure as norm_rows_kernel, with
// every f32 step on adjacent element pairs through the sm_100 paired
// instructions (two IEEE f32 operations per instruction, so per pair: LN one
// add for the sum, two for the centred squares, four in the epilogue; RMS one
// FMA for the sum of squares, four in the epilogue), bf16 widened by shift
// and mask, and the residual prologue on packed T pairs (residual_vec). The
// results per element are the same as the scalar forms: only the grouping of
// the row sums differs (two interleaved partial sums per thread).
// kMix (16-bit rows; LayerNorm without a residual branch, RMSNorm with or
// without): the sums with row elements use the mixed-precision add / fma on
// the stored elements instead of widening them first (fewer instructions; the
// same values). Chosen for row groups of 8 or more threads:
// with 4-thread groups (rows of 32 vectors) the shorter instruction stream
// reaches the per-vector weight loads sooner and waits on them, which measured
// slower.
template <typename T, int NV, bool kLN, int kMaxBlock, bool kBranch, bool kMix = false, int AW = 4>
__global__ void __launch_bounds__(kMaxBlock, kMaxBlock == 256 ? 4 : (kMaxBlock == 512 ? 2 : 1))
    norm_vec_kernel(const NormParams p) {
  griddep_wait();
  griddep_release();
  using P = Pairs<T>;
  constexpr int KPF = P::kP;                                // element pairs in a 16-byte vector
  constexpr int KP = std::is_same_v<T, float> ? AW / 2 : AW;  // ... in one access of AW words
  constexpr int N = Elem<T>::kVec * AW / 4;                 // elements per access
  // One scratch array per reduction (see group_sum's kReuse); one row per group.
  __shared__ float red_a[32], red_b[32];
  const int tpr = p.tpr;
  const int g = threadIdx.x / tpr;
  const int lr = threadIdx.x - g * tpr;
  const int rpb = blockDim.x / tpr;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * rpb + g;
  const bool active = row < p.rows;
  const int64_t base = row * p.cols;
  const T *src = static_cast<const T *>(p.src) + base;

  // 1) h = src (+ T(branch * ls)), packed; invalid slots hold +0.
  uint4 h[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int vi = lr + k * tpr;
    h[k] = make_uint4(0u, 0u, 0u, 0u);
    if (active && vi < p.nvec) h[k] = ld_stream_w<AW>(src + vi * N);
  }
  // Short rows per thread (NV <= 2, the shapes chosen for few or narrow rows),
  // and RMSNorm with a residual branch in 16-byte accesses up to its cap of 4:
  // fetch the weight / bias vectors together with the row, so their latency
  // is not added after the reductions (the fused residual RMSNorm at 16384 x
  // 1024: 0.87 -> 0.97 of the copy peak, bf16). Wider LayerNorm rows would
  // hold two more vectors per access and spill.
  constexpr bool kPre = NV <= 2 || (!kLN && kBranch && AW == 4 && NV <= 4);
  const T *wp = static_cast<const T *>(p.w);
  const T *bp = static_cast<const T *>(p.b);
  uint4 wpre[kPre ? NV : 1], bpre[kPre ? NV : 1];
  if constexpr (kPre) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int vi = lr + k * tpr;
      if (active && vi < p.nvec) {
        if (wp != nullptr) wpre[k] = ld_cached_w<AW>(wp + vi * N);
        if (kLN && bp != nullptr) bpre[k] = ld_cached_w<AW>(bp + vi * N);
      }
    }
  }
  if constexpr (kBranch) {
    const T *br = static_cast<const T *>(p.branch) + base;
    uint4 b[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int vi = lr + k * tpr;
      if (active && vi < p.nvec) b[k] = ld_stream_w<AW>(br + vi * N);
    }
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int vi = lr + k * tpr;
      if (active && vi < p.nvec)
        h[k] = residual_vec<T, AW>(h[k], b[k], p.ls != nullptr ? static_cast<const T *>(p.ls) + vi * N : nullptr);
    }
    if (p.res_out != nullptr) {
      T *ro = static_cast<T *>(p.res_out) + base;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int vi = lr + k * tpr;
        if (active && vi < p.nvec) st_w<AW>(ro + vi * N, h[k]);
      }
    }
  }

  // 2) Row statistics in f32, then 3) the epilogue dst = T(norm(h) * w (+ b)).
  const float cols_f = __ll2float_rn(p.cols);
  T *dst = static_cast<T *>(p.dst) + base;
  if constexpr (kLN && kMix && !std::is_same_v<T, float>) {
    // kMix: every f32 sum with a row element takes the element as it is
    // stored (sm_100's mixed-precision add, add2_widen), the same values as
    // widening it first; only the weight is widened.
    float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
#pragma unroll
      for (int j = 0; j < KP; ++j) s2 = add2_widen<T>(u4_word(h[k], j), s2);
    }
    const float mean = __fdiv_rn(group_sum<false>(__fadd_rn(s2.x, s2.y), tpr, red_a), cols_f);
    const float2 nmean = splat2(-mean);
    float2 v2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      if (lr + k * tpr < p.nvec) {
        const uint4 hk = opaque(h[k]);
#pragma unroll
        for (int j = 0; j < KP; ++j) {
          const float2 d = add2_widen<T>(u4_word(hk, j), nmean);
          v2 = __ffma2_rn(d, d, v2);
        }
      }
    }
    const float var = __fdiv_rn(group_sum<false>(__fadd_rn(v2.x, v2.y), tpr, red_b), cols_f);
    const float2 inv = splat2(__fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(var, p.eps))));
    const float2 nshift = splat2(p.remove_mean ? -mean : -0.f);  // -0: x + (-0) == x
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int vi = lr + k * tpr;
      if (active && vi < p.nvec) {
        const uint4 hk = opaque(h[k]);
        float2 x[KPF] = {}, w[KPF];
        if (wp != nullptr) {
          P::unpack(kPre ? wpre[k] : ld_cached_w<AW>(wp + vi * N), w);
        } else {
#pragma unroll
          for (int j = 0; j < KP; ++j) w[j] = splat2(1.f);
        }
#pragma unroll
        for (int j = 0; j < KP; ++j) x[j] = __fmul2_rn(__fmul2_rn(add2_widen<T>(u4_word(hk, j), nshift), inv), w[j]);
        if (bp != nullptr) {
          const uint4 bv = kPre ? bpre[k] : ld_cached_w<AW>(bp + vi * N);
#pragma unroll
          for (int j = 0; j < KP; ++j) x[j] = add2_widen<T>(u4_word(bv, j), x[j]);
        } else {
#pragma unroll
          for (int j = 0; j < KP; ++j) x[j] = __fadd2_rn(x[j], splat2(0.f));
        }
        st_w<AW>(dst + vi * N, P::pack(x));
      }
    }
  } else if constexpr (kLN) {
    float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      float2 x[KPF];
      P::unpack(h[k], x);
#pragma unroll
      for (int j = 0; j < KP; ++j) s2 = __fadd2_rn(s2, x[j]);
    }
    const float mean = __fdiv_rn(group_sum<false>(__fadd_rn(s2.x, s2.y), tpr, red_a), cols_f);
    const float2 nmean = splat2(-mean);
    float2 v2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      if (lr + k * tpr < p.nvec) {
        float2 x[KPF];
        P::unpack(opaque(h[k]), x);
#pragma unroll
        for (int j = 0; j < KP; ++j) {
          const float2 d = __fadd2_rn(x[j], nmean);
          v2 = __ffma2_rn(d, d, v2);
        }
      }
    }
    const float var = __fdiv_rn(group_sum<false>(__fadd_rn(v2.x, v2.y), tpr, red_b), cols_f);
    const float2 inv = splat2(__fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(var, p.eps))));
    // x + (-0) == x exactly (signed zeros included), so "no centring" is the
    // same instruction with a -0 shift.
    const float2 nshift = splat2(p.remove_mean ? -mean : -0.f);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int vi = lr + k * tpr;
      if (active && vi < p.nvec) {
        float2 x[KPF] = {}, w[KPF], b[KPF];
        P::unpack(opaque(h[k]), x);
        if (wp != nullptr) {
          P::unpack(kPre ? wpre[k] : ld_cached_w<AW>(wp + vi * N), w);
        } else {
#pragma unroll
          for (int j = 0; j < KP; ++j) w[j] = splat2(1.f);
        }
        if (bp != nullptr) {
          P::unpack(kPre ? bpre[k] : ld_cached_w<AW>(bp + vi * N), b);
        } else {
#pragma unroll
          for (int j = 0; j < KP; ++j) b[j] = splat2(0.f);
        }
#pragma unroll
        for (int j = 0; j < KP; ++j)
          x[j] = __fadd2_rn(__fmul2_rn(__fmul2_rn(__fadd2_rn(x[j], nshift), inv), w[j]), b[j]);
        st_w<AW>(dst + vi * N, P::pack(x));
      }
    }
  } else if constexpr (kMix && !std::is_same_v<T, float>) {
    // kMix: the squares summed straight from the stored elements (sm_100's
    // mixed-precision fma, sq_add2_widen: the same values), and div_by's
    // quotient steps with the remainder's sign flipped: nrem = m*q0 - x is
    // exactly -(x - m*q0), so q0 - nrem*r is the same value, and where x = +-0
    // the zeros combine to the sign of x, so no copysign fix-up is needed
    // (m = inf: 0 in m's place, q0 = x * 0 as in neg_divisor).
    float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
#pragma unroll
      for (int j = 0; j < KP; ++j) s2 = sq_add2_widen<T>(u4_word(h[k], j), s2);
    }
    const float s = group_sum<false>(__fadd_rn(s2.x, s2.y), tpr, red_a);
    const float m = __fsqrt_rn(__fadd_rn(__fdiv_rn(s, cols_f), p.eps));
    const float r = __frcp_rn(m);
    const float2 pm2 = splat2(isinf(m) ? 0.f : m), r2 = splat2(r);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int vi = lr + k * tpr;
      if (active && vi < p.nvec) {
        float2 x[KPF] = {}, w[KPF];
        P::unpack(opaque(h[k]), x);
        if (wp != nullptr) {
          P::unpack(kPre ? wpre[k] : ld_cached_w<AW>(wp + vi * N), w);
        } else {
#pragma unroll
          for (int j = 0; j < KP; ++j) w[j] = splat2(1.f);
        }
#pragma unroll
        for (int j = 0; j < KP; ++j) {
          const float2 q0 = __fmul2_rn(x[j], r2);
          const float2 nrem = __ffma2_rn(pm2, q0, make_float2(-x[j].x, -x[j].y));
          const float2 q = __ffma2_rn(make_float2(-nrem.x, -nrem.y), r2, q0);
          x[j] = __fmul2_rn(q, w[j]);
        }
        st_w<AW>(dst + vi * N, P::pack(x));
      }
    }
  } else {
    float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      float2 x[KPF];
      P::unpack(h[k], x);
#pragma unroll
      for (int j = 0; j < KP; ++j) s2 = __ffma2_rn(x[j], x[j], s2);
    }
    const float s = group_sum<false>(__fadd_rn(s2.x, s2.y), tpr, red_a);
    const float m = __fsqrt_rn(__fadd_rn(__fdiv_rn(s, cols_f), p.eps));
    const float r = __frcp_rn(m);
    const float2 nm2 = splat2(neg_divisor(m)), r2 = splat2(r);  // m = inf: see neg_divisor
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int vi = lr + k * tpr;
      if (active && vi < p.nvec) {
        float2 x[KPF] = {}, w[KPF];
        P::unpack(opaque(h[k]), x);
        if (wp != nullptr) {
          P::unpack(kPre ? wpre[k] : ld_cached_w<AW>(wp + vi * N), w);
        } else {
#pragma unroll
          for (int j = 0; j < KP; ++j) w[j] = splat2(1.f);
        }
#pragma unroll
        for (int j = 0; j < KP; ++j) {
          // T(x / m * alpha), the quotient by div_by's steps on a pair.
          const float2 q0 = __fmul2_rn(x[j], r2);
          const float2 rem = __ffma2_rn(nm2, q0, x[j]);
          float2 q = __ffma2_rn(rem, r2, q0);
          q.x = copysignf(q.x, q0.x);
          q.y = copysignf(q.y, q0.y);
          x[j] = __fmul2_rn(q, w[j]);
        }
        st_w<AW>(dst + vi * N, P::pack(x));
      }
    }
  }
}

// RMSNorm rows whose byte width is not a multiple of 16 (such as 250 16-bit
// columns), taken R at a time: R = 16 / gcd(cols * s, 16) consecutive rows are
// a run of R * cols elements that starts and ends on a 16-byte boundary, so a
// group of tpr threads reads and writes it with aligned 16-byte accesses, as
// the vector kernel does a row. An access holds elements of one row, or of
// two where a row ends inside it (R - 1 accesses of a run). The weights (and
// the layer scale) are tiled R times in shared memory, so every access's
// weights are one aligned 16-byte load. Each access adds its sum of squares
// to the row (or two) it covers, and the R row sums of a run are reduced
// across the group together. Per element, the arithmetic is the vector
// kernel's (the same IEEE f32 operations in the same order), so the values
// match it; only the grouping of the row sums differs. tpr <= 32 (shuffle
// reductions only).
template <int R>
__device__ __forceinline__ void add_to_row(float (&acc)[R], int row, float v) {
#pragma unroll
  for (int r = 0; r < R; ++r)
    if (r == row) acc[r] = __fadd_rn(acc[r], v);
}

template <int R>
__device__ __forceinline__ float row_value(const float (&v)[R], int row) {
  float out = v[0];
#pragma unroll
  for (int r = 1; r < R; ++r)
    if (r == row) out = v[r];
  return out;
}

template <typename T, int NV, int R, bool kBranch>
__global__ void __launch_bounds__(256, 4) norm_run_kernel(const NormParams p) {
  griddep_wait();
  griddep_release();
  using P = Pairs<T>;
  constexpr int N = Elem<T>::kVec;
  constexpr int KP = P::kP;
  extern __shared__ __align__(16) unsigned char run_smem[];
  const int cols = static_cast<int>(p.cols);
  const int run_len = R * cols;  // = p.nvec * N, a multiple of the vector
  T *wt = reinterpret_cast<T *>(run_smem);
  T *lt = wt + run_len;
  const T *w = static_cast<const T *>(p.w);
  const T *ls = static_cast<const T *>(p.ls);
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    const T wc = w != nullptr ? w[c] : Elem<T>::from_f32(1.f);
#pragma unroll
    for (int r = 0; r < R; ++r) wt[r * cols + c] = wc;
    if constexpr (kBranch) {
      if (ls != nullptr) {
        const T lc = ls[c];
#pragma unroll
        for (int r = 0; r < R; ++r) lt[r * cols + c] = lc;
      }
    }
  }
  __syncthreads();
  const int tpr = p.tpr;
  const int g = threadIdx.x / tpr;
  const int lr = threadIdx.x - g * tpr;
  const int rpb = blockDim.x / tpr;
  const int64_t run = static_cast<int64_t>(blockIdx.x) * rpb + g;
  const bool active = run * R < p.rows;
  const int64_t base = run * run_len;
  // Per access: the run row of its first element and how many of its
  // elements come before the next row (>= N: all of them).
  int r0[NV], sp[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int e0 = (lr + k * tpr) * N;
    r0[k] = 0;
#pragma unroll
    for (int r = 1; r < R; ++r) r0[k] += e0 >= r * cols;
    sp[k] = (r0[k] + 1) * cols - e0;
  }
  auto live = [&](int k) { return active && lr + k * tpr < p.nvec; };

  // 1) h = src (+ T(branch * ls)), packed.
  const T *src = static_cast<const T *>(p.src) + base;
  uint4 h[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    h[k] = make_uint4(0u, 0u, 0u, 0u);
    if (live(k)) h[k] = ld_stream(src + (lr + k * tpr) * N);
  }
  if constexpr (kBranch) {
    const T *br = static_cast<const T *>(p.branch) + base;
    uint4 bv[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k)
      if (live(k)) bv[k] = ld_stream(br + (lr + k * tpr) * N);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      if (live(k)) {
        const int vi = lr + k * tpr;
        if (ls != nullptr) {
          const uint4 sv = *reinterpret_cast<const uint4 *>(lt + vi * N);
          h[k] = residual_vec_sv<T>(h[k], bv[k], &sv);
        } else {
          h[k] = residual_vec_sv<T>(h[k], bv[k], nullptr);
        }
        if (p.res_out != nullptr) st_vec(static_cast<T *>(p.res_out) + base + vi * N, h[k]);
      }
    }
  }

  // 2) Each row's sum of squares: an access's goes to its row, or is split.
  const float cols_f = __int2float_rn(cols);
  T *dst = static_cast<T *>(p.dst) + base;
  auto elem = [](const float2 (&x)[KP], int e) { return (e & 1) ? x[e >> 1].y : x[e >> 1].x; };
  float acc[R] = {};
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    if (!live(k)) continue;
    float2 x[KP];
    P::unpack(h[k], x);
    if (sp[k] >= N) {
      float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < KP; ++j) s2 = __ffma2_rn(x[j], x[j], s2);
      add_to_row(acc, r0[k], __fadd_rn(s2.x, s2.y));
    } else {
      float lo = 0.f, hi = 0.f;
#pragma unroll
      for (int e = 0; e < N; ++e) {
        const float v = elem(x, e);
        if (e < sp[k])
          lo = __fmaf_rn(v, v, lo);
        else
          hi = __fmaf_rn(v, v, hi);
      }
      add_to_row(acc, r0[k], lo);
      add_to_row(acc, r0[k] + 1, hi);
    }
  }
  float m[R], rc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    m[r] = __fsqrt_rn(__fadd_rn(__fdiv_rn(group_sum<false>(acc[r], tpr, nullptr), cols_f), p.eps));
    rc[r] = __frcp_rn(m[r]);
  }
  // 3) dst = T(x / m * alpha), each element with its own row's m.
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    if (!live(k)) continue;
    const int vi = lr + k * tpr;
    float2 x[KP], wv[KP];
    P::unpack(opaque(h[k]), x);
    P::unpack(*reinterpret_cast<const uint4 *>(wt + vi * N), wv);
    const float m_lo = row_value(m, r0[k]), r_lo = row_value(rc, r0[k]);
    if (sp[k] >= N) {
      // One row: the vector kernel's paired div_by steps.
      const float2 nm2 = splat2(neg_divisor(m_lo)), r2 = splat2(r_lo);
#pragma unroll
      for (int j = 0; j < KP; ++j) {
        const float2 q0 = __fmul2_rn(x[j], r2);
        const float2 rem = __ffma2_rn(nm2, q0, x[j]);
        float2 q = __ffma2_rn(rem, r2, q0);
        q.x = copysignf(q.x, q0.x);
        q.y = copysignf(q.y, q0.y);
        x[j] = __fmul2_rn(q, wv[j]);
      }
    } else {
      const float m_hi = row_value(m, r0[k] + 1), r_hi = row_value(rc, r0[k] + 1);
#pragma unroll
      for (int j = 0; j < KP; ++j) {
        // Per element: the two elements of a pair may belong to different rows.
        const bool fx = 2 * j < sp[k], fy = 2 * j + 1 < sp[k];
        x[j].x = __fmul_rn(div_by(x[j].x, fx ? m_lo : m_hi, fx ? r_lo : r_hi), wv[j].x);
        x[j].y = __fmul_rn(div_by(x[j].y, fy ? m_lo : m_hi, fy ? r_lo : r_hi), wv[j].y);
      }
    }
    st_vec(dst + vi * N, P::pack(x));
  }
}

// Rows wider than the register budget: one block per row, several passes.
template <typename T, bool kLN>
__global__ void __launch_bounds__(1024) norm_loop_kernel(const NormParams p) {
  griddep_wait();
  griddep_release();
  __shared__ float red[32];
  const int tpr = blockDim.x;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * p.cols;
  auto compute_h = [&](int64_t c) -> float {
    float x = ld_elem<T>(p.src, base + c);
    if (p.branch != nullptr) {
      float br = ld_elem<T>(p.branch, base + c);
      if (p.ls != nullptr) br = Elem<T>::round(__fmul_rn(br, ld_elem<T>(p.ls, c)));
      x = Elem<T>::round(__fadd_rn(x, br));
    }
    return x;
  };
  // After pass 1, residual_out holds h exactly (it may alias src).
  auto read_h = [&](int64_t c) -> float {
    return p.res_out != nullptr ? ld_elem<T>(p.res_out, base + c) : compute_h(c);
  };
  const float cols_f = __ll2float_rn(p.cols);
  float s = 0.f;
  for (int64_t c = threadIdx.x; c < p.cols; c += tpr) {
    const float h = compute_h(c);
    if (p.res_out != nullptr) st_elem<T>(p.res_out, base + c, h);
    s = __fadd_rn(s, kLN ? h : __fmul_rn(h, h));
  }
  s = group_sum(s, tpr, red);
  if constexpr (kLN) {
    const float mean = __fdiv_rn(s, cols_f);
    float v = 0.f;
    for (int64_t c = threadIdx.x; c < p.cols; c += tpr) {
      const float d = __fsub_rn(read_h(c), mean);
      v = __fadd_rn(v, __fmul_rn(d, d));
    }
    v = group_sum(v, tpr, red);
    const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(v, cols_f), p.eps)));
    for (int64_t c = threadIdx.x; c < p.cols; c += tpr) {
      const float h = read_h(c);
      const float cen = p.remove_mean ? __fsub_rn(h, mean) : h;
      const float w = p.w != nullptr ? ld_elem<T>(p.w, c) : 1.f;
      const float b = p.b != nullptr ? ld_elem<T>(p.b, c) : 0.f;
      st_elem<T>(p.dst, base + c, __fadd_rn(__fmul_rn(__fmul_rn(cen, inv), w), b));
    }
  } else {
    const float m = __fsqrt_rn(__fadd_rn(__fdiv_rn(s, cols_f), p.eps));
    for (int64_t c = threadIdx.x; c < p.cols; c += tpr) {
      const float w = p.w != nullptr ? ld_elem<T>(p.w, c) : 1.f;
      st_elem<T>(p.dst, base + c, __fmul_rn(__fdiv_rn(read_h(c), m), w));
    }
  }
}

// Accesses per thread: up to 8 in 256- and 512-thread blocks (4 with a
// branch, whose vectors are held too) and up to 4 in the 1024-thread shape
// used for the widest rows. Only shapes within the cap are instantiated.
template <bool kBranch, int kMaxBlock>
constexpr int kMaxNv = (kBranch || kMaxBlock > 512) ? 4 : 8;

// One launch of the row-group kernel with NV accesses per thread: the paired
// f32 kernel for 16-byte vectors, the scalar one otherwise.
template <typename T, bool kVector, int NV, bool kLN, int kMaxBlock, bool kBranch, int AW = 4>
void launch_nv(const NormParams &p, int block, int64_t grid, cudaStream_t st) {
  if constexpr (kVector) {
    if constexpr ((!kLN || !kBranch) && !std::is_same_v<T, float>) {
      if (p.tpr >= 8) {
        launch_k(norm_vec_kernel<T, NV, kLN, kMaxBlock, kBranch, true, AW>, dim3(grid), dim3(block), 0, st, p);
        return;
      }
    }
    launch_k(norm_vec_kernel<T, NV, kLN, kMaxBlock, kBranch, false, AW>, dim3(grid), dim3(block), 0, st, p);
  } else {
    launch_k(norm_rows_kernel<T, NV, kLN, kMaxBlock, kBranch>, dim3(grid), dim3(block), 0, st, p);
  }
}

// Returns false when no instantiated kernel has this shape (a dispatcher bug).
template <typename T, bool kVector, bool kLN, int kMaxBlock, bool kBranch, int AW = 4>
bool launch_regs_b(NormParams p, int nv, int block, int64_t grid, cudaStream_t st) {
  constexpr int cap = kMaxNv<kBranch, kMaxBlock>;
  switch (nv) {
    case 1:
      launch_nv<T, kVector, 1, kLN, kMaxBlock, kBranch, AW>(p, block, grid, st);
      return true;
    case 2:
      if constexpr (cap >= 2) {
        launch_nv<T, kVector, 2, kLN, kMaxBlock, kBranch, AW>(p, block, grid, st);
        return true;
      }
      return false;
    case 3:
      if constexpr (cap >= 4 && kVector) {
        launch_nv<T, kVector, 3, kLN, kMaxBlock, kBranch, AW>(p, block, grid, st);
        return true;
      }
      return false;
    case 4:
      if constexpr (cap >= 4) {
        launch_nv<T, kVector, 4, kLN, kMaxBlock, kBranch, AW>(p, block, grid, st);
        return true;
      }
      return false;
    case 6:
      if constexpr (cap >= 8 && kVector) {
        launch_nv<T, kVector, 6, kLN, kMaxBlock, kBranch, AW>(p, block, grid, st);
        return true;
      }
      return false;
    case 8:
      if constexpr (cap >= 8) {
        launch_nv<T, kVector, 8, kLN, kMaxBlock, kBranch, AW>(p, block, grid, st);
        return true;
      }
      return false;
    default:
      return false;
  }
}

// Register budgets per block size: 256-thread blocks run four per SM, the
// 512-thread vector shape two (so one row's loads overlap another's
// reductions), the 1024-thread shape one.
template <typename T, bool kVector, bool kLN, int AW = 4>
bool launch_regs(NormParams p, int nv, int block, int64_t grid, cudaStream_t st) {
  const bool branch = p.branch != nullptr;
  if (block <= 256) {
    return branch ? launch_regs_b<T, kVector, kLN, 256, true, AW>(p, nv, block, grid, st)
                  : launch_regs_b<T, kVector, kLN, 256, false, AW>(p, nv, block, grid, st);
  }
  if constexpr (AW != 4) return false;  // narrow accesses: 256-thread shapes only
  if constexpr (kVector) {
    if (block == 512 && nv > 4)
      return branch ? false : launch_regs_b<T, kVector, kLN, 512, false>(p, nv, block, grid, st);
  }
  return branch ? launch_regs_b<T, kVector, kLN, 1024, true>(p, nv, block, grid, st)
                : launch_regs_b<T, kVector, kLN, 1024, false>(p, nv, block, grid, st);
}

// Chooses the row-group shape and launches. Register budget: <= 32 f32 values
// of the row per thread, so rows of up to 32768 elements stay in registers.
// norm_run_kernel for RMSNorm rows whose byte width is not a multiple of 16,
// when runs are of 4 rows (2 or 4 for f32; odd 16-bit widths would need 8,
// whose row sums spill), the row count
// divides into runs, a run fits 32 threads of 4 accesses and its tiled
// weights fit 48 KB of shared memory; false leaves the rows to the other
// kernels. LayerNorm measured slower in this form (bf16 262144 x 250: 0.42
// with 4-byte accesses, 0.33 here, f32 0.81 against 0.71: its two reductions
// of R row values and the per-access row selections cost more than the wider
// accesses save).
template <typename T, bool kBranch>
bool launch_norm_run_r(const NormParams &p, int r, int64_t grid, size_t smem, cudaStream_t st) {
  switch (r) {
    case 2:
      launch_k(norm_run_kernel<T, 4, 2, kBranch>, dim3(grid), dim3(256), smem, st, p);
      return true;
    case 4:
      launch_k(norm_run_kernel<T, 4, 4, kBranch>, dim3(grid), dim3(256), smem, st, p);
      return true;
    default:
      return false;
  }
}

template <typename T>
bool try_launch_norm_run(NormParams p, cudaStream_t st) {
  constexpr int V = Elem<T>::kVec;
  const int64_t row_bytes = p.cols * static_cast<int64_t>(sizeof(T));
  if (row_bytes % 16 == 0 || p.cols <= 0) return false;
  const uintptr_t big = reinterpret_cast<uintptr_t>(p.dst) | reinterpret_cast<uintptr_t>(p.src) |
                        reinterpret_cast<uintptr_t>(p.branch) | reinterpret_cast<uintptr_t>(p.res_out);
  if ((big & 15u) != 0) return false;
  int64_t gcd = 16;
  while (row_bytes % gcd != 0) gcd /= 2;
  const int r = static_cast<int>(16 / gcd);
  // 16-bit rows of a multiple of 8 bytes (R = 2) keep the 8-byte accesses,
  // which measured a little faster (bf16 262144 x 100: 0.71 against 0.68).
  if (r > 4 || (sizeof(T) == 2 && r == 2) || p.rows % r != 0) return false;
  const bool branch = p.branch != nullptr;
  const int64_t nvec = r * p.cols / V;
  const int64_t tpr = pow2_ceil(ceil_div(nvec, static_cast<int64_t>(4)));
  if (tpr > 32) return false;
  const size_t smem = static_cast<size_t>(r * p.cols) * sizeof(T) * (branch ? 2 : 1);
  if (smem > 48 * 1024) return false;
  p.tpr = static_cast<int>(tpr);
  p.nvec = static_cast<int>(nvec);
  const int64_t grid = ceil_div(p.rows / r, 256 / tpr);
  if (grid > 0x7fffffffLL) return false;
  return branch ? launch_norm_run_r<T, true>(p, r, grid, smem, st)
                : launch_norm_run_r<T, false>(p, r, grid, smem, st);
}

template <typename T, bool kLN>
int launch_norm(NormParams p, cudaStream_t st, const char *op) {
  constexpr int V = Elem<T>::kVec;
  if constexpr (!kLN) {
    if (try_launch_norm_run<T>(p, st)) return check_launch(op);
  }
  const uintptr_t addr_bits = reinterpret_cast<uintptr_t>(p.dst) | reinterpret_cast<uintptr_t>(p.src) |
                              reinterpret_cast<uintptr_t>(p.w) | reinterpret_cast<uintptr_t>(p.b) |
                              reinterpret_cast<uintptr_t>(p.branch) | reinterpret_cast<uintptr_t>(p.ls) |
                              reinterpret_cast<uintptr_t>(p.res_out);
  const int64_t row_bytes = p.cols * static_cast<int64_t>(sizeof(T));
  // Access width in 32-bit words: 16-byte vectors when rows and pointers allow;
  // otherwise 8-byte (f32 or 16-bit rows whose bytes are a multiple of 8) or
  // 4-byte (16-bit rows of even width) accesses, which keep the vector
  // kernel's paired arithmetic for ragged widths (such as 250 columns) in
  // place of element accesses; those take the 256-thread shapes only.
  int aw = 0;
  if (row_bytes % 16 == 0 && (addr_bits & 15u) == 0)
    aw = 4;
  else if (row_bytes % 8 == 0 && (addr_bits & 7u) == 0)
    aw = 2;
  else if (sizeof(T) == 2 && row_bytes % 4 == 0 && (addr_bits & 3u) == 0)
    aw = 1;
  if (aw != 0 && aw != 4 && p.cols / (V * aw / 4) > 256LL * (p.branch != nullptr ? 4 : 8)) aw = 0;
  const bool vec = aw != 0;
  const int n = vec ? V * aw / 4 : 1;
  const int64_t nvec = p.cols / n;
  // Up to 32 row values per thread (16 with a branch, which doubles the
  // loads held in registers): rows of up to 32768 (16384) elements.
  // Row-group shape: 256-thread blocks take up to 8 accesses per thread (4
  // with a branch); wider vector rows without a branch use 512-thread groups
  // with 8; the rest groups of up to 1024 threads with up to 4.
  // LayerNorm rows of at most 32 vectors (256 bf16 columns) take 8-thread groups
  // with 4 accesses each rather than 4 with 8 (0.77 -> 0.80 of the copy peak at
  // 262144 x 256 bf16; rows of 64 vectors measured slower so).
  const int cap256 = (p.branch != nullptr || (kLN && aw == 4 && p.cols / V <= 32)) ? 4 : 8;
  int64_t tpr = 0;
  if (nvec <= 256LL * cap256) {
    tpr = pow2_ceil(ceil_div(nvec, vec ? cap256 : 4));
    if (tpr > 256) tpr = 256;
  } else if (vec && p.branch == nullptr && nvec > 512LL * 4 && nvec <= 512LL * 8) {
    tpr = 512;
  } else if (nvec <= 1024LL * 4) {
    tpr = pow2_ceil(ceil_div(nvec, 4));
  }
  // Few rows (decode steps): spread each row over more threads, down to one
  // access per thread, while the whole launch stays under 64K threads; this
  // shortens the per-thread chain and brings the weights forward (kPre).
  if (vec && tpr > 0 && tpr < 256) {
    while (tpr < 256 && tpr < nvec && p.rows * tpr * 2 <= 65536) tpr *= 2;
  }
  if (tpr > 0) {
    int nv = static_cast<int>(pow2_ceil(ceil_div(nvec, tpr)));
    // 5 or 6 accesses per thread (rows of 1536, 2560, 3072 or 5120 16-bit
    // columns): 6 instead of 8, and 3 instead of 4 (with a residual branch,
    // rows of 768, 1536 or 3072 16-bit columns). Every access slot is issued
    // whether or not a lane holds data in it, so empty slots cost as much as
    // full ones.
    if (vec && nv == 8 && ceil_div(nvec, tpr) <= 6) nv = 6;
    if (vec && nv == 4 && ceil_div(nvec, tpr) == 3) nv = 3;
    const int block = tpr < 256 ? 256 : static_cast<int>(tpr);
    const int64_t rpb = block / tpr;
    const int64_t grid = ceil_div(p.rows, rpb);
    if (grid > 0x7fffffffLL) return fail(XN_E_INVALID, "%s: too many rows (%lld)", op, (long long)p.rows);
    p.tpr = static_cast<int>(tpr);
    p.nvec = static_cast<int>(nvec);
    bool launched = false;
    if (aw == 4) {
      launched = launch_regs<T, true, kLN, 4>(p, nv, block, grid, st);
    } else if (aw == 2) {
      launched = launch_regs<T, true, kLN, 2>(p, nv, block, grid, st);
    } else if (aw == 1) {
      if constexpr (sizeof(T) == 2) launched = launch_regs<T, true, kLN, 1>(p, nv, block, grid, st);
    } else {
      launched = launch_regs<T, false, kLN>(p, nv, block, grid, st);
    }
    if (!launched) return fail(XN_E_INVALID, "%s: internal error, no kernel for %d accesses per thread", op, nv);
  } else {
    if (p.rows > 0x7fffffffLL) return fail(XN_E_INVALID, "%s: too many rows (%lld)", op, (long long)p.rows);
    launch_k(norm_loop_kernel<T, kLN>, dim3(static_cast<unsigned>(p.rows)), dim3(1024), 0, st, p);
  }
  return check_launch(op);
}

int check_norm_args(const char *op, const void *dst, const void *src, const void *branch,
                    const void *ls, int64_t rows, int64_t cols, float eps, int dtype) {
  if (!is_float_dtype(dtype)) return fail(XN_E_DTYPE, "%s: unsupported dtype %d", op, dtype);
  if (rows < 0 || cols < 0) return fail(XN_E_INVALID, "%s: negative size rows=%lld cols=%lld", op, (long long)rows, (long long)cols);
  if (!(eps > 0.f)) return fail(XN_E_INVALID, "%s: eps must be positive (got %g)", op, (double)eps);
  if (rows > 0 && cols > 0 && (dst == nullptr || src == nullptr))
    return fail(XN_E_INVALID, "%s: null dst or src", op);
  if (ls != nullptr && branch == nullptr)
    return fail(XN_E_INVALID, "%s: layer_scale given without a branch", op);
  return XN_OK;
}

}  // namespace
}  // namespace xn

extern "C" {

int xn_rms_norm(void *dst, const void *src, const void *alpha, const void *branch,
                const void *layer_scale, void *residual_out, int64_t rows, int64_t cols, float eps,
                int dtype, void *stream) {
  using namespace xn;
  const char *op = "xn_rms_norm";
  int rc = check_norm_args(op, dst, src, branch, layer_scale, rows, cols, eps, dtype);
  if (rc != XN_OK) return rc;
  if (rows == 0 || cols == 0) return ok();
  NormParams p{dst, src, alpha, nullptr, branch, layer_scale, residual_out, rows, cols, eps, 0, 0, 0};
  XN_DISPATCH_FLOAT(dtype, return launch_norm<T, false>(p, as_stream(stream), op));
  return fail(XN_E_DTYPE, "%s: unsupported dtype %d", op, dtype);
}

int xn_layer_norm(void *dst, const void *src, const void *weight, const void *bias,
                  const void *branch, const void *layer_scale, void *residual_out, int64_t rows,
                  int64_t cols, float eps, int remove_mean, int dtype, void *stream) {
  using namespace xn;
  const char *op = "xn_layer_norm";
  int rc = check_norm_args(op, dst, src, branch, layer_scale, rows, cols, eps, dtype);
  if (rc != XN_OK) return rc;
  if (rows == 0 || cols == 0) return ok();
  NormParams p{dst, src, weight, bias, branch, layer_scale, residual_out, rows, cols, eps,
               remove_mean ? 1 : 0, 0, 0};
  XN_DISPATCH_FLOAT(dtype, return launch_norm<T, true>(p, as_stream(stream), op));
  return fail(XN_E_DTYPE, "%s: unsupported dtype %d", op, dtype);
}

}  // extern "C"
