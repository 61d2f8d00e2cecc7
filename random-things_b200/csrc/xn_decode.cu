// xn_decode.cu - streaming decode on a ring-buffer KV cache, for sm_100a:
// the KV-cache append fused with RoPE on the packed QKV projection, and the
// decode attention (score, scale, causal mask, softmax, weighted sum of V) in
// one launch.
//
// Reference semantics:
//   * append: the narrow / reshape / transpose / contiguous split of the
//     in_proj output, rope_i on q and k (cpu_backend.rs:394-422 per element,
//     T arithmetic) and KvCache::append's cat + trim
//     (mimi-rs/src/models/mimi.rs:1122-1153, 1330-1354;
//     pocket_tts/src/mimi_transformer.rs:32-61, 122-137);
//   * attention: q.matmul_t(k) (f32 accumulation, T result), .scale(scale)
//     (T multiply), apply_causality_mask / the additive causal mask, softmax
//     (cpu_backend.rs:667-689), .matmul(v) (f32 accumulation, T result)
//     (mimi-rs/src/models/mimi.rs:1356-1371, pocket_tts/src/transformer.rs:134-145).
//
// Design: the cache never moves. A step writes its t new rows into ring
// slots (total + i) % cap, and the attention walks the last kv_len positions
// in logical (oldest-first) order through the same slot map, so the sums run
// in the reference's key order. One CTA per (batch, head, query) holds the
// query and the kv_len scores on chip: phase 1 gives each thread whole keys
// (a 16-byte-vector dot product per key, no shuffles), phase 2 gives each
// thread one 16-byte column block of V for a strided group of keys (many
// independent loads in flight), and the group partials are added in a fixed
// order.
#include <math.h>

#include <type_traits>

#include "xn_common.cuh"
#include "xn_internal.h"

namespace xn {
namespace {

constexpr int kMaxContext = 8192;  // scores held in shared memory (32 KB)
constexpr int kAttnThreads = 128;

struct AppendParams {
  void *q_out;
  void *k_cache;
  void *v_cache;
  const void *qkv;
  const void *cos;
  const void *sin;
  int64_t b, h, t, d, total, max_pos, cap;
  const int64_t *total_dev;
  int *err_flag;
  int64_t chunks;  // work items per head row: vectors (interleaved) or vectors of one half
};

__device__ __forceinline__ int64_t read_total(int64_t total, const int64_t *total_dev) {
  return total_dev != nullptr ? *total_dev : total;
}

// One item = one 16-byte vector (interleaved form; v copy) or one vector of
// each half (half-split form) of one head row of q, k or v at one step.
// Scalar form (kVector false): one rotation pair.
template <typename T, bool kInterleaved, bool kVector>
__global__ void __launch_bounds__(256) kv_append_rope_kernel(const AppendParams p) {
  griddep_wait();
  griddep_release();
  constexpr int V = kVector ? Elem<T>::kVec : 1;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (item >= p.b * p.t * 3 * p.h * p.chunks) return;
  const int64_t c = item % p.chunks;
  int64_t r = item / p.chunks;
  const int64_t hh = r % p.h;
  r /= p.h;
  const int which = static_cast<int>(r % 3);  // 0 q, 1 k, 2 v
  r /= 3;
  const int64_t i = r % p.t;
  const int64_t bi = r / p.t;
  const int64_t pos = read_total(p.total, p.total_dev) + i;
  if (pos < 0 || pos >= p.max_pos) {  // reachable with total_dev only (the host checks total)
    if (p.err_flag != nullptr) atomicOr(p.err_flag, 1);
    return;
  }
  const int64_t d = p.d, half = d / 2;
  const T *src = static_cast<const T *>(p.qkv) + ((bi * p.t + i) * 3 + which) * p.h * d + hh * d;
  T *dst;
  if (which == 0) {
    dst = static_cast<T *>(p.q_out) + ((bi * p.h + hh) * p.t + i) * d;
  } else {
    T *cache = static_cast<T *>(which == 1 ? p.k_cache : p.v_cache);
    dst = cache + ((bi * p.h + hh) * p.cap + pos % p.cap) * d;
  }
  // Element offsets of this item's two parts (vectors or scalars).
  const int64_t e1 = kInterleaved ? c * (kVector ? V : 2) : c * V;
  const int64_t e2 = kInterleaved ? e1 + 1 : e1 + half;  // scalar pair / second half
  const T *cs = static_cast<const T *>(p.cos) + pos * half;
  const T *sn = static_cast<const T *>(p.sin) + pos * half;
  if constexpr (kVector) {
    if constexpr (kInterleaved) {
      const uint4 x = ld_stream(src + e1);
      if (which == 2) {
        st_vec(dst + e1, x);
      } else {
        const uint2 cr = ld_cached8(cs + e1 / 2), sr = ld_cached8(sn + e1 / 2);
        st_vec(dst + e1, rotate_interleaved<T>(x, cr, sr));
      }
    } else {
      const uint4 x1 = ld_stream(src + e1), x2 = ld_stream(src + e2);
      if (which == 2) {
        st_vec(dst + e1, x1);
        st_vec(dst + e2, x2);
      } else {
        uint4 y1, y2;
        rotate_halfsplit<T>(x1, x2, ld_cached(cs + e1), ld_cached(sn + e1), y1, y2);
        st_vec(dst + e1, y1);
        st_vec(dst + e2, y2);
      }
    }
  } else {
    const float a = Elem<T>::to_f32(src[e1]), b = Elem<T>::to_f32(src[e2]);
    if (which == 2) {
      dst[e1] = src[e1];
      dst[e2] = src[e2];
    } else {
      const float cv = Elem<T>::to_f32(cs[c]), sv = Elem<T>::to_f32(sn[c]);
      const float y1 = __fsub_rn(Elem<T>::round(__fmul_rn(a, cv)), Elem<T>::round(__fmul_rn(b, sv)));
      const float y2 = __fadd_rn(Elem<T>::round(__fmul_rn(a, sv)), Elem<T>::round(__fmul_rn(b, cv)));
      dst[e1] = Elem<T>::from_f32(y1);
      dst[e2] = Elem<T>::from_f32(y2);
    }
  }
}

struct AttnParams {
  void *out;
  const void *q;
  const void *k_cache;
  const void *v_cache;
  int64_t b, h, t, total, cap, context;
  const int64_t *total_dev;
  int mask_mode;
  float scale;
  // Fused step only: the packed projection and the RoPE tables.
  const void *qkv;
  const void *cos;
  const void *sin;
  int64_t max_pos;
  int *err_flag;
};

// One 16-byte vector of a cached row: read-only path for caches written by
// an earlier launch, coherent loads where this launch wrote them.
template <typename T, bool kCoherent>
__device__ __forceinline__ uint4 ld_row_vec(const T *p) {
  if constexpr (kCoherent) {
    return ld_plain(p);
  } else {
    return ld_cached(p);
  }
}

// q . row over the D head dims (16-byte vector loads, f32 FMA in dim order).
template <typename T, int D, bool kCoherent>
__device__ __forceinline__ float dot_row(const T *row, const float *qs) {
  constexpr int V = Elem<T>::kVec;
  float acc = 0.f;
#pragma unroll
  for (int v = 0; v < D / V; ++v) {
    float x[V];
    unpack<T>(ld_row_vec<T, kCoherent>(row + v * V), x);
#pragma unroll
    for (int j = 0; j < V; ++j) acc = __fmaf_rn(qs[v * V + j], x[j], acc);
  }
  return acc;
}

// kFused: the block first does this head's part of xn_kv_append_rope (the t
// new k rows rotated and v rows copied into their ring slots, identical bytes
// from every block of the head) and rotates its own query into shared memory;
// then it attends as the plain kernel does, reading the caches with coherent
// loads. kInterleaved picks the RoPE form of the fused prologue.
template <typename T, int D, bool kFused, bool kInterleaved>
__global__ void __launch_bounds__(kAttnThreads) attention_decode_kernel(const AttnParams p) {
  griddep_wait();
  griddep_release();
  constexpr int V = Elem<T>::kVec;           // elements per 16-byte vector
  constexpr int kVpr = D / V;                // vectors per cached row
  constexpr int kGroups = kAttnThreads / kVpr;  // key groups in the weighted sum
  extern __shared__ float scores[];  // [kv_len]: scores, then probabilities
  __shared__ float qs[D];
  __shared__ float part[kGroups * D];
  __shared__ float red[32];
  const int64_t bh = blockIdx.x;  // bi * h + hh
  const int64_t i = blockIdx.y;   // query index within the step
  const int64_t bi = bh / p.h, hh = bh % p.h;
  const int64_t total = read_total(p.total, p.total_dev);
  const int64_t n = total + p.t;
  const int64_t kv_len = n < p.context ? n : p.context;
  const int64_t first = n - kv_len;  // position of logical key 0
  // XN_MASK_CACHE_LEN shows the keys of XN_MASK_ABSOLUTE: its offset
  // min(total, context) differs from total only when total >= context, and then
  // every one of the kv_len <= context keys is visible under either offset.
  const int64_t last_visible = p.mask_mode != XN_MASK_RELATIVE ? total + i : i + kv_len - p.t;
  // Position of query / new row i2 in the RoPE tables: total + i2, or the
  // cache's length before the step + i2 (XN_MASK_CACHE_LEN).
  const int64_t rope0 = p.mask_mode == XN_MASK_CACHE_LEN && total > p.context ? p.context : total;
  const int64_t nvis = last_visible + 1 < kv_len ? last_visible + 1 : kv_len;
  // Logical key j sits at slot (first + j) % cap; j < kv_len <= cap, so one
  // conditional subtraction replaces the per-key division.
  const int64_t slot0 = first % p.cap;
  auto slot_of = [&](int64_t j) -> int64_t {
    const int64_t s = slot0 + j;
    return s >= p.cap ? s - p.cap : s;
  };
  T *kw = static_cast<T *>(const_cast<void *>(p.k_cache)) + bh * p.cap * D;
  T *vw = static_cast<T *>(const_cast<void *>(p.v_cache)) + bh * p.cap * D;
  const T *kc = kw;
  const T *vc = vw;
  T *out = static_cast<T *>(p.out) + ((bi * p.t + i) * p.h + hh) * D;
  const int tid = threadIdx.x;

  if constexpr (kFused) {
    if (total < 0 || rope0 + p.t > p.max_pos) {  // device position past the tables
      if (tid == 0 && p.err_flag != nullptr) atomicOr(p.err_flag, 1);
      return;  // uniform over the block, before any barrier
    }
    constexpr int C = kInterleaved ? kVpr : kVpr / 2;  // work items per row
    const int64_t half = D / 2;
    const int64_t n_items = (2 * p.t + 1) * C;  // t k rows, t v rows, this block's q row
    for (int64_t it = tid; it < n_items; it += kAttnThreads) {
      const int64_t r = it / C;
      const int c = static_cast<int>(it % C);
      int which;
      int64_t i2;
      if (r < 2 * p.t) {
        which = 1 + static_cast<int>(r / p.t);
        i2 = r % p.t;
      } else {
        which = 0;
        i2 = i;
      }
      const int64_t pos = total + i2;  // ring position
      const T *src = static_cast<const T *>(p.qkv) + ((bi * p.t + i2) * 3 + which) * p.h * D + hh * D;
      T *dst = which == 1 ? kw + (pos % p.cap) * D : vw + (pos % p.cap) * D;
      const T *cs = static_cast<const T *>(p.cos) + (rope0 + i2) * half;
      const T *sn = static_cast<const T *>(p.sin) + (rope0 + i2) * half;
      if constexpr (kInterleaved) {
        const int e = c * V;
        uint4 y = ld_stream(src + e);
        if (which != 2) y = rotate_interleaved<T>(y, ld_cached8(cs + e / 2), ld_cached8(sn + e / 2));
        if (which == 0) {
          float f[V];
          unpack<T>(y, f);
#pragma unroll
          for (int k = 0; k < V; ++k) qs[e + k] = f[k];
        } else {
          st_vec(dst + e, y);
        }
      } else {
        const int e1 = c * V, e2 = c * V + static_cast<int>(half);
        uint4 y1 = ld_stream(src + e1), y2 = ld_stream(src + e2);
        if (which != 2) {
          const uint4 x1 = y1, x2 = y2;
          rotate_halfsplit<T>(x1, x2, ld_cached(cs + e1), ld_cached(sn + e1), y1, y2);
        }
        if (which == 0) {
          float f1[V], f2[V];
          unpack<T>(y1, f1);
          unpack<T>(y2, f2);
#pragma unroll
          for (int k = 0; k < V; ++k) {
            qs[e1 + k] = f1[k];
            qs[e2 + k] = f2[k];
          }
        } else {
          st_vec(dst + e1, y1);
          st_vec(dst + e2, y2);
        }
      }
    }
  } else {
    for (int k = tid; k < D; k += kAttnThreads)
      qs[k] = Elem<T>::to_f32(static_cast<const T *>(p.q)[(bh * p.t + i) * D + k]);
  }
  __syncthreads();

  // Phase 1: scores T(T(q.k) * T(scale)), -inf where masked.
  const float scale_t = Elem<T>::round(p.scale);
  float m = -INFINITY;
#pragma unroll 2
  for (int64_t j = tid; j < kv_len; j += kAttnThreads) {
    float s = -INFINITY;
    if (j < nvis) {
      s = Elem<T>::round(dot_row<T, D, kFused>(kc + slot_of(j) * D, qs));
      s = Elem<T>::round(__fmul_rn(s, scale_t));
    }
    scores[j] = s;
    m = fmaxf(m, s);
  }
  const float mx = group_max(m, kAttnThreads, red);

  // Softmax in T arithmetic: e = T(exp(T(s - max))), p = T(e / sum).
  float sum = 0.f;
  for (int64_t j = tid; j < kv_len; j += kAttnThreads) {
    const float e = Elem<T>::round(exp_t<T>(Elem<T>::round(__fsub_rn(scores[j], mx))));
    scores[j] = e;
    sum = __fadd_rn(sum, e);
  }
  sum = group_sum(sum, kAttnThreads, red);  // its barriers also publish scores[]
  const float rs = __frcp_rn(sum);
  for (int64_t j = tid; j < kv_len; j += kAttnThreads)
    scores[j] = Elem<T>::round(div_by(scores[j], sum, rs));
  __syncthreads();

  // Phase 2: out = T(sum_j p_j v_j). Thread = (key group g, vector c of the
  // row): it accumulates keys j = g, g + kGroups, ... for the V head dims of
  // vector c, with several 16-byte loads in flight; the group partials are
  // then added in group order. Masked keys (p = 0) are skipped.
  const int c = tid % kVpr, g = tid / kVpr;
  float acc[V];
#pragma unroll
  for (int k = 0; k < V; ++k) acc[k] = 0.f;
  const int64_t upto = nvis > 0 ? nvis : 0;
#pragma unroll 8
  for (int64_t j = g; j < upto; j += kGroups) {
    float x[V];
    unpack<T>(ld_row_vec<T, kFused>(vc + slot_of(j) * D + c * V), x);
    const float pj = scores[j];
#pragma unroll
    for (int k = 0; k < V; ++k) acc[k] = __fmaf_rn(pj, x[k], acc[k]);
  }
#pragma unroll
  for (int k = 0; k < V; ++k) part[g * D + c * V + k] = acc[k];
  __syncthreads();
  for (int k = tid; k < D; k += kAttnThreads) {
    float s = part[k];
#pragma unroll
    for (int w = 1; w < kGroups; ++w) s = __fadd_rn(s, part[w * D + k]);
    // No visible key: the reference's softmax of an all -inf row is NaN.
    out[k] = Elem<T>::from_f32(nvis > 0 ? s : __int_as_float(0x7fc00000));
  }
}

__global__ void position_advance_kernel(int64_t *total_dev, int64_t t) {
  griddep_wait();
  griddep_release(); *total_dev += t; }

template <typename T>
int launch_append(AppendParams p, int interleaved, cudaStream_t st) {
  constexpr int V = Elem<T>::kVec;
  const int64_t half = p.d / 2;
  const bool vec = is_aligned16(p.q_out) && is_aligned16(p.k_cache) && is_aligned16(p.v_cache) &&
                   is_aligned16(p.qkv) && is_aligned16(p.cos) && is_aligned16(p.sin) &&
                   (interleaved ? p.d % V == 0 : half % V == 0);
  p.chunks = vec ? (interleaved ? p.d / V : half / V) : half;
  const int64_t items = p.b * p.t * 3 * p.h * p.chunks;
  const int64_t grid = ceil_div(items, int64_t{256});
  if (grid > 0x7fffffffLL) return fail(XN_E_INVALID, "xn_kv_append_rope: too many elements");
  if (vec) {
    if (interleaved)
      launch_k(kv_append_rope_kernel<T, true, true>, dim3(grid), dim3(256), 0, st, p);
    else
      launch_k(kv_append_rope_kernel<T, false, true>, dim3(grid), dim3(256), 0, st, p);
  } else {
    if (interleaved)
      launch_k(kv_append_rope_kernel<T, true, false>, dim3(grid), dim3(256), 0, st, p);
    else
      launch_k(kv_append_rope_kernel<T, false, false>, dim3(grid), dim3(256), 0, st, p);
  }
  return check_launch("xn_kv_append_rope");
}

template <typename T, int D, bool kFused, bool kInterleaved>
void launch_attn_d(const AttnParams &p, cudaStream_t st) {
  const dim3 grid(static_cast<unsigned>(p.b * p.h), static_cast<unsigned>(p.t));
  const size_t smem = static_cast<size_t>(p.context) * sizeof(float);
  launch_k(attention_decode_kernel<T, D, kFused, kInterleaved>, dim3(grid), dim3(kAttnThreads), smem, st, p);
}

template <typename T, bool kFused, bool kInterleaved>
int launch_attn_f(const AttnParams &p, int64_t d, cudaStream_t st, const char *op) {
  switch (d) {
    case 32:
      launch_attn_d<T, 32, kFused, kInterleaved>(p, st);
      break;
    case 64:
      launch_attn_d<T, 64, kFused, kInterleaved>(p, st);
      break;
    case 128:
      launch_attn_d<T, 128, kFused, kInterleaved>(p, st);
      break;
    default:
      return fail(XN_E_INVALID, "%s: head dim %lld not in {32, 64, 128}", op, (long long)d);
  }
  return check_launch(op);
}

template <typename T>
int launch_attn(const AttnParams &p, int64_t d, int fused, int interleaved, cudaStream_t st, const char *op) {
  // Vector loads need 16-byte aligned rows: d * sizeof(T) is a multiple of 16
  // for every supported d, so aligned bases suffice.
  if (!is_aligned16(p.k_cache) || !is_aligned16(p.v_cache))
    return fail(XN_E_INVALID, "%s: k_cache and v_cache must be 16-byte aligned", op);
  if (!fused) return launch_attn_f<T, false, false>(p, d, st, op);
  if (!is_aligned16(p.qkv) || !is_aligned16(p.cos) || !is_aligned16(p.sin))
    return fail(XN_E_INVALID, "%s: qkv, cos and sin must be 16-byte aligned", op);
  return interleaved ? launch_attn_f<T, true, true>(p, d, st, op) : launch_attn_f<T, true, false>(p, d, st, op);
}

}  // namespace
}  // namespace xn

extern "C" {

int xn_kv_append_rope(void *q_out, void *k_cache, void *v_cache, const void *qkv, const void *cos,
                      const void *sin, int64_t b, int64_t h, int64_t t, int64_t d, int64_t total,
                      const int64_t *total_dev, int64_t max_pos, int64_t cap, int interleaved, int dtype,
                      int *err_flag, void *stream) {
  using namespace xn;
  const char *op = "xn_kv_append_rope";
  if (!is_float_dtype(dtype)) return fail(XN_E_DTYPE, "%s: unsupported dtype %d", op, dtype);
  if (b < 0 || h < 0 || t < 0 || d < 0) return fail(XN_E_INVALID, "%s: negative size", op);
  if (d % 2 != 0) return fail(XN_E_INVALID, "%s: head dim %lld is odd", op, (long long)d);
  if (cap <= 0 || t > cap) return fail(XN_E_INVALID, "%s: t=%lld new positions exceed cap=%lld", op, (long long)t, (long long)cap);
  if (total_dev == nullptr) {
    if (total < 0) return fail(XN_E_INVALID, "%s: negative position %lld", op, (long long)total);
    if (total + t > max_pos)
      return fail(XN_E_RANGE, "%s: pos %lld + t %lld exceeds the %lld rows of cos/sin", op, (long long)total,
                  (long long)t, (long long)max_pos);
  }
  if (b == 0 || h == 0 || t == 0 || d == 0) return ok();
  if (q_out == nullptr || k_cache == nullptr || v_cache == nullptr || qkv == nullptr || cos == nullptr ||
      sin == nullptr)
    return fail(XN_E_INVALID, "%s: null pointer", op);
  AppendParams p{q_out, k_cache, v_cache, qkv, cos, sin, b, h, t, d, total, max_pos, cap, total_dev, err_flag, 0};
  XN_DISPATCH_FLOAT(dtype, return launch_append<T>(p, interleaved, as_stream(stream)));
  return fail(XN_E_DTYPE, "%s: unsupported dtype %d", op, dtype);
}

int xn_attention_decode(void *out, const void *q, const void *k_cache, const void *v_cache, int64_t b, int64_t h,
                        int64_t t, int64_t d, int64_t total, const int64_t *total_dev, int64_t cap, int64_t context,
                        int mask_mode, float scale, int dtype, void *stream) {
  using namespace xn;
  const char *op = "xn_attention_decode";
  if (!is_float_dtype(dtype)) return fail(XN_E_DTYPE, "%s: unsupported dtype %d", op, dtype);
  if (b < 0 || h < 0 || t < 0) return fail(XN_E_INVALID, "%s: negative size", op);
  if (d != 32 && d != 64 && d != 128) return fail(XN_E_INVALID, "%s: head dim %lld not in {32, 64, 128}", op, (long long)d);
  if (context <= 0 || context > cap || context > kMaxContext)
    return fail(XN_E_INVALID, "%s: need 0 < context <= cap and context <= %d (context=%lld cap=%lld)", op,
                kMaxContext, (long long)context, (long long)cap);
  if (t > cap) return fail(XN_E_INVALID, "%s: t=%lld exceeds cap=%lld", op, (long long)t, (long long)cap);
  if (mask_mode != XN_MASK_RELATIVE && mask_mode != XN_MASK_ABSOLUTE && mask_mode != XN_MASK_CACHE_LEN)
    return fail(XN_E_INVALID, "%s: unknown mask mode %d", op, mask_mode);
  if (total_dev == nullptr && total < 0) return fail(XN_E_INVALID, "%s: negative position %lld", op, (long long)total);
  if (b * h > 0x7fffffffLL || t > 65535) return fail(XN_E_INVALID, "%s: grid too large (b*h=%lld, t=%lld)", op, (long long)(b * h), (long long)t);
  if (b == 0 || h == 0 || t == 0) return ok();
  if (out == nullptr || q == nullptr || k_cache == nullptr || v_cache == nullptr)
    return fail(XN_E_INVALID, "%s: null pointer", op);
  AttnParams p{out, q, k_cache, v_cache, b, h, t, total, cap, context, total_dev, mask_mode, scale,
               nullptr, nullptr, nullptr, 0, nullptr};
  XN_DISPATCH_FLOAT(dtype, return launch_attn<T>(p, d, 0, 0, as_stream(stream), op));
  return fail(XN_E_DTYPE, "%s: unsupported dtype %d", op, dtype);
}

int xn_decode_attention_step(void *out, void *k_cache, void *v_cache, const void *qkv, const void *cos,
                             const void *sin, int64_t b, int64_t h, int64_t t, int64_t d, int64_t total,
                             const int64_t *total_dev, int64_t max_pos, int64_t cap, int64_t context,
                             int mask_mode, float scale, int interleaved, int dtype, int *err_flag,
                             void *stream) {
  using namespace xn;
  const char *op = "xn_decode_attention_step";
  if (!is_float_dtype(dtype)) return fail(XN_E_DTYPE, "%s: unsupported dtype %d", op, dtype);
  if (b < 0 || h < 0 || t < 0) return fail(XN_E_INVALID, "%s: negative size", op);
  if (d != 32 && d != 64 && d != 128) return fail(XN_E_INVALID, "%s: head dim %lld not in {32, 64, 128}", op, (long long)d);
  if (context <= 0 || context > cap || context > kMaxContext)
    return fail(XN_E_INVALID, "%s: need 0 < context <= cap and context <= %d (context=%lld cap=%lld)", op,
                kMaxContext, (long long)context, (long long)cap);
  if (t > cap) return fail(XN_E_INVALID, "%s: t=%lld new positions exceed cap=%lld", op, (long long)t, (long long)cap);
  if (mask_mode != XN_MASK_RELATIVE && mask_mode != XN_MASK_ABSOLUTE && mask_mode != XN_MASK_CACHE_LEN)
    return fail(XN_E_INVALID, "%s: unknown mask mode %d", op, mask_mode);
  if (total_dev == nullptr) {
    if (total < 0) return fail(XN_E_INVALID, "%s: negative position %lld", op, (long long)total);
    // The rows rotate at total + i, or at min(total, context) + i (XN_MASK_CACHE_LEN).
    const int64_t rope0 = mask_mode == XN_MASK_CACHE_LEN && total > context ? context : total;
    if (rope0 + t > max_pos)
      return fail(XN_E_RANGE, "%s: pos %lld + t %lld exceeds the %lld rows of cos/sin", op, (long long)rope0,
                  (long long)t, (long long)max_pos);
  }
  if (b * h > 0x7fffffffLL || t > 65535) return fail(XN_E_INVALID, "%s: grid too large (b*h=%lld, t=%lld)", op, (long long)(b * h), (long long)t);
  if (b == 0 || h == 0 || t == 0) return ok();
  if (out == nullptr || k_cache == nullptr || v_cache == nullptr || qkv == nullptr || cos == nullptr ||
      sin == nullptr)
    return fail(XN_E_INVALID, "%s: null pointer", op);
  AttnParams p{out, nullptr, k_cache, v_cache, b, h, t, total, cap, context, total_dev, mask_mode, scale,
               qkv, cos, sin, max_pos, err_flag};
  XN_DISPATCH_FLOAT(dtype, return launch_attn<T>(p, d, 1, interleaved, as_stream(stream), op));
  return fail(XN_E_DTYPE, "%s: unsupported dtype %d", op, dtype);
}

int xn_position_advance(int64_t *total_dev, int64_t t, void *stream) {
  using namespace xn;
  if (total_dev == nullptr) return fail(XN_E_INVALID, "xn_position_advance: null pointer");
  if (t < 0) return fail(XN_E_INVALID, "xn_position_advance: negative t");
  launch_k(position_advance_kernel, dim3(1), dim3(1), 0, as_stream(stream), total_dev, t);
  return check_launch("xn_position_advance");
}

}  // extern "C"
