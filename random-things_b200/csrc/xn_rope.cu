// xn_rope.cu - rotary position embedding (half-split and interleaved) on
// [B,H,T,D] or [B,T,H,D] tensors, one or two tensors (Q and K) per launch.
//
// Reference semantics: mimi-rs/src/cpu_backend.rs:359-392 (rope) and
// :394-422 (rope_i). Each product and each sum is a T-typed operation there,
// so for bf16/f16 the kernel rounds after every multiply and add, which makes
// it bit-exact with the reference for every dtype:
//   y1 = T(T(x1*c) - T(x2*s)),  y2 = T(T(x1*s) + T(x2*c)).
//
// Design: a thread owns one 16-byte chunk of a row (or of each half of a row
// for the half-split form) at one time step and loops over `hpt` heads, so the
// cos/sin chunk is loaded once and reused for several heads. Lanes of a warp
// own consecutive chunks, so every global access is a full 16-byte vector and
// warps touch contiguous 128-byte segments.
#include <type_traits>

#include "xn_common.cuh"
#include "xn_internal.h"

namespace xn {
namespace {

struct RopeTensor {
  void *dst;
  const void *src;
  uint32_t heads;
  uint32_t items;  // work items of this tensor in this launch
  int64_t src_ts;  // [B,T,H,D] layout: elements between consecutive tokens
  int64_t dst_ts;  //   (H*D when contiguous; larger inside a packed QKV row)
};

struct RopeParams {
  RopeTensor ten[2];
  const void *cos;
  const void *sin;
  uint32_t t;       // time steps
  uint32_t d;       // head dim
  uint32_t chunks;  // work chunks per row (half-split: per half)
  uint32_t hpt;     // heads per thread
  int64_t pos;
  int layout;
};

constexpr int kMaxHpt = 4;  // heads per thread (cos/sin reuse, loads in flight)

template <typename T, bool kInterleaved, bool kVector>
__global__ void __launch_bounds__(256) rope_kernel(const RopeParams p) {
  griddep_wait();
  griddep_release();
  constexpr int V = Elem<T>::kVec;
  uint32_t item = blockIdx.x * blockDim.x + threadIdx.x;
  int which = 0;
  if (item >= p.ten[0].items) {
    item -= p.ten[0].items;
    which = 1;
    if (item >= p.ten[1].items) return;
  }
  const RopeTensor tn = p.ten[which];
  const uint32_t H = tn.heads;
  const uint32_t hg_count = (H + p.hpt - 1) / p.hpt;
  // Work order follows the memory order of the layout, so consecutive warps
  // stream consecutive bytes:
  //   [B,H,T,D]: item = ((bi * hg_count + hg) * T + ti) * chunks + c
  //   [B,T,H,D]: item = ((bi * T + ti) * hg_count + hg) * chunks + c
  const uint32_t c = item % p.chunks;
  uint32_t rest = item / p.chunks;
  uint32_t ti, hg;
  if (p.layout == XN_LAYOUT_BHTD) {
    ti = rest % p.t;
    rest /= p.t;
    hg = rest % hg_count;
    rest /= hg_count;
  } else {
    hg = rest % hg_count;
    rest /= hg_count;
    ti = rest % p.t;
    rest /= p.t;
  }
  const uint32_t bi = rest;

  const int64_t d = p.d;
  const int64_t half = d / 2;
  const int64_t trow = (p.pos + ti) * half;  // first table entry of this time step
  int64_t head_stride;
  const T *src = static_cast<const T *>(tn.src);
  T *dst = static_cast<T *>(tn.dst);
  if (p.layout == XN_LAYOUT_BHTD) {
    const int64_t row0 = ((static_cast<int64_t>(bi) * H) * p.t + ti) * d;
    src += row0;
    dst += row0;
    head_stride = static_cast<int64_t>(p.t) * d;
  } else {
    const int64_t tok = static_cast<int64_t>(bi) * p.t + ti;
    src += tok * tn.src_ts;
    dst += tok * tn.dst_ts;
    head_stride = d;
  }
  // src and dst now point at head 0 of this (b, t) row.
  const T *cs = static_cast<const T *>(p.cos);
  const T *sn = static_cast<const T *>(p.sin);

  if constexpr (kVector && !kInterleaved) {
    // chunk c: elements [c*V, c*V+V) of each half. All heads' loads first.
    uint4 r1[kMaxHpt], r2[kMaxHpt];
#pragma unroll
    for (int hh = 0; hh < kMaxHpt; ++hh) {
      const uint32_t h = hg * p.hpt + hh;
      if (hh < static_cast<int>(p.hpt) && h < H) {
        const int64_t e1 = h * head_stride + c * V;
        r1[hh] = ld_stream(src + e1);
        r2[hh] = ld_stream(src + e1 + half);
      }
    }
    const uint4 cr = ld_cached(cs + trow + c * V);
    const uint4 sr = ld_cached(sn + trow + c * V);
#pragma unroll
    for (int hh = 0; hh < kMaxHpt; ++hh) {
      const uint32_t h = hg * p.hpt + hh;
      if (hh < static_cast<int>(p.hpt) && h < H) {
        const int64_t e1 = h * head_stride + c * V;
        uint4 y1, y2;
        rotate_halfsplit<T>(r1[hh], r2[hh], cr, sr, y1, y2);
        st_vec(dst + e1, y1);
        st_vec(dst + e1 + half, y2);
      }
    }
  } else if constexpr (kVector && kInterleaved) {
    // chunk c: elements [c*V, c*V+V) = pairs [c*V/2, c*V/2 + V/2).
    constexpr int P = V / 2;
    uint4 rx[kMaxHpt];
#pragma unroll
    for (int hh = 0; hh < kMaxHpt; ++hh) {
      const uint32_t h = hg * p.hpt + hh;
      if (hh < static_cast<int>(p.hpt) && h < H) rx[hh] = ld_stream(src + h * head_stride + c * V);
    }
    const uint2 cr = ld_cached8(cs + trow + c * P), sr = ld_cached8(sn + trow + c * P);
#pragma unroll
    for (int hh = 0; hh < kMaxHpt; ++hh) {
      const uint32_t h = hg * p.hpt + hh;
      if (hh < static_cast<int>(p.hpt) && h < H)
        st_vec(dst + h * head_stride + c * V, rotate_interleaved<T>(rx[hh], cr, sr));
    }
  } else {
    // Scalar fallback: chunk c is one pair (element c of each half, or pair c).
    const float cv = Elem<T>::to_f32(cs[trow + c]);
    const float sv = Elem<T>::to_f32(sn[trow + c]);
    for (uint32_t hh = 0; hh < p.hpt; ++hh) {
      const uint32_t h = hg * p.hpt + hh;
      if (h >= H) break;
      const int64_t r = h * head_stride;
      const int64_t e1 = kInterleaved ? r + 2 * c : r + c;
      const int64_t e2 = kInterleaved ? e1 + 1 : e1 + half;
      const float a = Elem<T>::to_f32(src[e1]), b = Elem<T>::to_f32(src[e2]);
      const float y1 = __fsub_rn(Elem<T>::round(__fmul_rn(a, cv)), Elem<T>::round(__fmul_rn(b, sv)));
      const float y2 = __fadd_rn(Elem<T>::round(__fmul_rn(a, sv)), Elem<T>::round(__fmul_rn(b, cv)));
      dst[e1] = Elem<T>::from_f32(y1);
      dst[e2] = Elem<T>::from_f32(y2);
    }
  }
}

struct RopeJob {
  void *dst[2];
  const void *src[2];
  int64_t heads[2];
  int n;
  int64_t src_ts = 0;  // token strides for the [B,T,H,D] layout (0: contiguous)
  int64_t dst_ts = 0;
};

template <typename T>
int launch_rope(const RopeJob &job, const void *cos, const void *sin, int64_t b, int64_t t,
                int64_t d, int64_t pos, int interleaved, int layout, cudaStream_t st,
                const char *op) {
  constexpr int V = Elem<T>::kVec;
  const int64_t half = d / 2;
  bool vec = is_aligned16(cos) && is_aligned16(sin);
  for (int i = 0; i < job.n; ++i) vec = vec && is_aligned16(job.dst[i]) && is_aligned16(job.src[i]);
  // Token strides must keep every row start 16-byte aligned for the vector path.
  for (int i = 0; i < job.n; ++i) {
    const int64_t hd = job.heads[i] * d;
    const int64_t sts = job.src_ts ? job.src_ts : hd, dts = job.dst_ts ? job.dst_ts : hd;
    vec = vec && (sts * static_cast<int64_t>(sizeof(T))) % 16 == 0 && (dts * static_cast<int64_t>(sizeof(T))) % 16 == 0;
  }
  vec = vec && (interleaved ? (d % V == 0) : (half % V == 0));
  const int64_t chunks = vec ? (interleaved ? d / V : half / V) : half;
  int64_t max_heads = 0;
  for (int i = 0; i < job.n; ++i) max_heads = job.heads[i] > max_heads ? job.heads[i] : max_heads;
  const int64_t hpt = max_heads >= kMaxHpt ? kMaxHpt : (max_heads > 0 ? max_heads : 1);
  // Work items per batch element for each tensor; launch over batch slices so
  // each launch indexes its items with 32-bit integers.
  int64_t per_b = 0;
  for (int i = 0; i < job.n; ++i) per_b += ceil_div(job.heads[i], hpt) * t * chunks;
  if (per_b <= 0) return ok();
  const int64_t limit = 0x7fffff00LL;
  if (per_b > limit)
    return fail(XN_E_INVALID, "%s: one batch element is too large (%lld work items)", op, (long long)per_b);
  const int64_t b_step = limit / per_b;
  for (int64_t b0 = 0; b0 < b; b0 += b_step) {
    const int64_t nb = (b - b0) < b_step ? (b - b0) : b_step;
    RopeParams p{};
    int64_t total = 0;
    for (int i = 0; i < 2; ++i) {
      if (i < job.n) {
        const int64_t hd = job.heads[i] * d;
        const int64_t sts = job.src_ts ? job.src_ts : hd, dts = job.dst_ts ? job.dst_ts : hd;
        // Elements per batch element (BHTD is always contiguous).
        const int64_t sb = layout == XN_LAYOUT_BHTD ? hd * t : sts * t;
        const int64_t db = layout == XN_LAYOUT_BHTD ? hd * t : dts * t;
        p.ten[i].dst = static_cast<T *>(job.dst[i]) + b0 * db;
        p.ten[i].src = static_cast<const T *>(job.src[i]) + b0 * sb;
        p.ten[i].heads = static_cast<uint32_t>(job.heads[i]);
        p.ten[i].items = static_cast<uint32_t>(nb * ceil_div(job.heads[i], hpt) * t * chunks);
        p.ten[i].src_ts = sts;
        p.ten[i].dst_ts = dts;
      } else {
        p.ten[i] = RopeTensor{nullptr, nullptr, 1, 0, 0, 0};
      }
      total += p.ten[i].items;
    }
    p.cos = cos;
    p.sin = sin;
    p.t = static_cast<uint32_t>(t);
    p.d = static_cast<uint32_t>(d);
    p.chunks = static_cast<uint32_t>(chunks);
    p.hpt = static_cast<uint32_t>(hpt);
    p.pos = pos;
    p.layout = layout;
    const unsigned grid = static_cast<unsigned>(ceil_div(total, 256));
    if (interleaved) {
      if (vec)
        launch_k(rope_kernel<T, true, true>, dim3(grid), dim3(256), 0, st, p);
      else
        launch_k(rope_kernel<T, true, false>, dim3(grid), dim3(256), 0, st, p);
    } else {
      if (vec)
        launch_k(rope_kernel<T, false, true>, dim3(grid), dim3(256), 0, st, p);
      else
        launch_k(rope_kernel<T, false, false>, dim3(grid), dim3(256), 0, st, p);
    }
    const int rc = check_launch(op);
    if (rc != XN_OK) return rc;
  }
  return ok();
}

int rope_entry(const char *op, const RopeJob &job, const void *cos, const void *sin, int64_t b,
               int64_t t, int64_t d, int64_t pos, int64_t max_pos, int interleaved, int layout,
               int dtype, void *stream) {
  if (!is_float_dtype(dtype)) return fail(XN_E_DTYPE, "%s: unsupported dtype %d", op, dtype);
  if (b < 0 || t < 0 || d < 0 || pos < 0 || max_pos < 0)
    return fail(XN_E_INVALID, "%s: negative size or position", op);
  for (int i = 0; i < job.n; ++i)
    if (job.heads[i] < 0) return fail(XN_E_INVALID, "%s: negative head count", op);
  if (d % 2 != 0) return fail(XN_E_INVALID, "%s: requires even d dimension, got d=%lld", op, (long long)d);
  if (layout != XN_LAYOUT_BHTD && layout != XN_LAYOUT_BTHD)
    return fail(XN_E_INVALID, "%s: unknown layout %d", op, layout);
  if (pos + t > max_pos)
    return fail(XN_E_RANGE, "%s: position out of range, pos=%lld + t=%lld > max_pos=%lld", op,
                (long long)pos, (long long)t, (long long)max_pos);
  if (t > 0xffffffffLL || d > 0xffffffffLL || job.heads[0] > 0xffffffffLL)
    return fail(XN_E_INVALID, "%s: dimension too large", op);
  int64_t elems = 0;
  for (int i = 0; i < job.n; ++i) elems += b * job.heads[i] * t * d;
  if (elems == 0) return ok();
  if (cos == nullptr || sin == nullptr) return fail(XN_E_INVALID, "%s: null cos/sin table", op);
  for (int i = 0; i < job.n; ++i)
    if (job.heads[i] > 0 && (job.dst[i] == nullptr || job.src[i] == nullptr))
      return fail(XN_E_INVALID, "%s: null dst or src", op);
  XN_DISPATCH_FLOAT(dtype, return launch_rope<T>(job, cos, sin, b, t, d, pos, interleaved, layout,
                                                 as_stream(stream), op));
  return fail(XN_E_DTYPE, "%s: unsupported dtype %d", op, dtype);
}

}  // namespace
}  // namespace xn

extern "C" {

int xn_rope(void *dst, const void *src, const void *cos, const void *sin, int64_t b, int64_t h,
            int64_t t, int64_t d, int64_t pos, int64_t max_pos, int interleaved, int layout,
            int dtype, void *stream) {
  xn::RopeJob job{{dst, nullptr}, {src, nullptr}, {h, 0}, 1};
  return xn::rope_entry("xn_rope", job, cos, sin, b, t, d, pos, max_pos, interleaved, layout, dtype,
                        stream);
}

int xn_rope_qk(void *q_dst, const void *q_src, void *k_dst, const void *k_src, const void *cos,
               const void *sin, int64_t b, int64_t hq, int64_t hk, int64_t t, int64_t d,
               int64_t pos, int64_t max_pos, int interleaved, int layout, int dtype, void *stream) {
  xn::RopeJob job{{q_dst, k_dst}, {q_src, k_src}, {hq, hk}, 2};
  return xn::rope_entry("xn_rope_qk", job, cos, sin, b, t, d, pos, max_pos, interleaved, layout,
                        dtype, stream);
}

int xn_rope_qk_strided(void *q_dst, const void *q_src, void *k_dst, const void *k_src, const void *cos,
                       const void *sin, int64_t b, int64_t hq, int64_t hk, int64_t t, int64_t d, int64_t pos,
                       int64_t max_pos, int64_t src_tok_stride, int64_t dst_tok_stride, int interleaved,
                       int dtype, void *stream) {
  using namespace xn;
  const char *op = "xn_rope_qk_strided";
  const int64_t hmax = hq > hk ? hq : hk;
  if (src_tok_stride < hmax * d || dst_tok_stride < hmax * d)
    return fail(XN_E_INVALID, "%s: token stride smaller than heads * d (src %lld, dst %lld, need %lld)", op,
                (long long)src_tok_stride, (long long)dst_tok_stride, (long long)(hmax * d));
  RopeJob job{{q_dst, k_dst}, {q_src, k_src}, {hq, hk}, 2};
  job.src_ts = src_tok_stride;
  job.dst_ts = dst_tok_stride;
  return rope_entry(op, job, cos, sin, b, t, d, pos, max_pos, interleaved, XN_LAYOUT_BTHD, dtype, stream);
}

}  // extern "C"
