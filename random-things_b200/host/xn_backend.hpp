// xn_backend.hpp - C++ host-side mirror of the `xn` Backend trait for the
// fused layer-op path, on top of the C ABI in include/xn_fused.h.
//
// The reference's host code is Rust: `trait Backend` (mimi-rs/src/backend.rs)
// implemented for CUDA by `cuda_backend::Device` (mimi-rs/src/cuda_backend.rs)
// and called through the shape-checking tensor ops of
// mimi-rs/src/inplace_ops.rs. This header restates that interface in C++ for
// the ops on the path: same method names, same argument meaning
// (dim_m1 = last dimension, d = number of rows, b/h/t/d for rope), and the
// same error behaviour (a failed check throws xn::Error before any launch,
// with the reference's message text). Storage is a typed device pointer plus
// a length, the role CudaSlice<T> plays in the reference.
//
// Header-only; link libxn_fused.so and the CUDA runtime.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "xn_fused.h"

namespace xn {

// Element tags for the 16-bit float types (host code needs no CUDA half types).
struct bf16 {
  uint16_t bits;
};
struct f16 {
  uint16_t bits;
};

template <typename T>
struct DTypeOf;
template <>
struct DTypeOf<float> {
  static constexpr int value = XN_F32;
};
template <>
struct DTypeOf<bf16> {
  static constexpr int value = XN_BF16;
};
template <>
struct DTypeOf<f16> {
  static constexpr int value = XN_F16;
};
template <>
struct DTypeOf<int64_t> {
  static constexpr int value = XN_I64;
};
template <>
struct DTypeOf<uint8_t> {
  static constexpr int value = XN_U8;
};

// mimi-rs/src/error.rs: one error type; `code` carries the C ABI status.
class Error : public std::runtime_error {
 public:
  Error(const std::string &msg, int code = XN_E_INVALID) : std::runtime_error(msg), code(code) {}
  int code;
};

inline void check(int rc, const char *what) {
  if (rc != XN_OK) throw Error(std::string(what) + ": " + xn_last_error(), rc);
}

// Device buffer of `len` elements of T (the reference's Storage<T>).
template <typename T>
struct Storage {
  T *data = nullptr;
  size_t len = 0;
};

// inplace_ops.rs:172-473 use these unary ops on the path.
enum class UnaryOp { Silu, GeluErf };

// Per-layer streaming-decode state: k and v are [b, h, cap, d] ring buffers
// (position p in slot p % cap) and `total` counts the positions appended. It
// stands for the reference's KvCache (mimi.rs:1099-1153,
// pocket_tts/src/mimi_transformer.rs:10-61; cat then trim) and
// StreamingMHAState (pocket_tts/src/transformer.rs:5-33; slice_set into a
// preallocated buffer). The caller owns the two buffers.
template <typename T>
struct RingKvCache {
  Storage<T> k, v;
  size_t b = 0, h = 0, cap = 0, d = 0;
  size_t total = 0;
};

// Which causal mask / position bookkeeping the decode attention applies
// (xn_fused.h XN_MASK_*): CacheLen is mimi-rs's StreamingTransformer (offset =
// the cache's length before the step), Absolute Pocket's Mimi attention,
// Relative the flow LM's additive mask.
enum class DecodeMask { Relative = XN_MASK_RELATIVE, Absolute = XN_MASK_ABSOLUTE, CacheLen = XN_MASK_CACHE_LEN };

// The CUDA device of the reference (cuda_backend.rs:34-54): one stream on
// which every op is enqueued.
class CudaDevice {
 public:
  explicit CudaDevice(cudaStream_t stream = nullptr) : stream_(stream) {}
  cudaStream_t stream() const { return stream_; }

  void synchronize() const {
    if (cudaStreamSynchronize(stream_) != cudaSuccess) throw Error("synchronize failed", XN_E_CUDA);
  }

  // ---- Backend::rms_norm (backend.rs:165-172; checks inplace_ops.rs:259-273)
  template <typename T>
  void rms_norm(Storage<T> &dst, const Storage<T> &src, const Storage<T> &alpha, size_t dim_m1, size_t d,
                float eps) const {
    if (!(eps > 0.f)) throw Error("rms_norm_ eps must be positive");
    expect_len(src, dim_m1 * d, "rms_norm_ src");
    expect_len(dst, dim_m1 * d, "rms_norm_ dst");
    expect_len(alpha, dim_m1, "rms_norm_ alpha");
    check(xn_rms_norm(dst.data, src.data, alpha.data, nullptr, nullptr, nullptr, (int64_t)d, (int64_t)dim_m1, eps,
                      DTypeOf<T>::value, stream_),
          "rms_norm");
  }

  // Fused residual form: h = src + [ls *] branch -> residual_out; dst = rms_norm(h).
  template <typename T>
  void rms_norm_residual(Storage<T> &dst, Storage<T> &residual_out, const Storage<T> &src,
                         const Storage<T> &branch, const Storage<T> *layer_scale, const Storage<T> &alpha,
                         size_t dim_m1, size_t d, float eps) const {
    if (!(eps > 0.f)) throw Error("rms_norm_ eps must be positive");
    for (const Storage<T> *s : {&dst, &residual_out, &src, &branch}) expect_len(*s, dim_m1 * d, "rms_norm_residual");
    expect_len(alpha, dim_m1, "rms_norm_ alpha");
    if (layer_scale) expect_len(*layer_scale, dim_m1, "rms_norm_ layer_scale");
    check(xn_rms_norm(dst.data, src.data, alpha.data, branch.data, layer_scale ? layer_scale->data : nullptr,
                      residual_out.data, (int64_t)d, (int64_t)dim_m1, eps, DTypeOf<T>::value, stream_),
          "rms_norm_residual");
  }

  // ---- Backend::layer_norm (backend.rs:180-189; checks inplace_ops.rs:275-307)
  template <typename T>
  void layer_norm(Storage<T> &dst, const Storage<T> &src, const Storage<T> &weight, const Storage<T> &bias,
                  size_t dim_m1, size_t d, float eps, bool remove_mean) const {
    if (!(eps > 0.f)) throw Error("layer_norm_ eps must be positive");
    expect_len(src, dim_m1 * d, "layer_norm_ src");
    expect_len(dst, dim_m1 * d, "layer_norm_ dst");
    expect_len(weight, dim_m1, "layer_norm_ weight");
    expect_len(bias, dim_m1, "layer_norm_ bias");
    check(xn_layer_norm(dst.data, src.data, weight.data, bias.data, nullptr, nullptr, nullptr, (int64_t)d,
                        (int64_t)dim_m1, eps, remove_mean ? 1 : 0, DTypeOf<T>::value, stream_),
          "layer_norm");
  }

  template <typename T>
  void layer_norm_residual(Storage<T> &dst, Storage<T> &residual_out, const Storage<T> &src,
                           const Storage<T> &branch, const Storage<T> *layer_scale, const Storage<T> &weight,
                           const Storage<T> &bias, size_t dim_m1, size_t d, float eps, bool remove_mean) const {
    if (!(eps > 0.f)) throw Error("layer_norm_ eps must be positive");
    for (const Storage<T> *s : {&dst, &residual_out, &src, &branch})
      expect_len(*s, dim_m1 * d, "layer_norm_residual");
    expect_len(weight, dim_m1, "layer_norm_ weight");
    expect_len(bias, dim_m1, "layer_norm_ bias");
    if (layer_scale) expect_len(*layer_scale, dim_m1, "layer_norm_ layer_scale");
    check(xn_layer_norm(dst.data, src.data, weight.data, bias.data, branch.data,
                        layer_scale ? layer_scale->data : nullptr, residual_out.data, (int64_t)d, (int64_t)dim_m1,
                        eps, remove_mean ? 1 : 0, DTypeOf<T>::value, stream_),
          "layer_norm_residual");
  }

  // ---- Backend::rope / rope_i (backend.rs:101-124; cpu_backend.rs:370-375 size
  // bails; inplace_ops.rs:421-473 checks). cos/sin are [max_pos, d/2].
  template <typename T>
  void rope(Storage<T> &dst, const Storage<T> &src, const Storage<T> &cos, const Storage<T> &sin, size_t b,
            size_t h, size_t t, size_t d, size_t pos) const {
    rope_impl(dst, src, cos, sin, b, h, t, d, pos, false, "rope");
  }

  template <typename T>
  void rope_i(Storage<T> &dst, const Storage<T> &src, const Storage<T> &cos, const Storage<T> &sin, size_t b,
              size_t h, size_t t, size_t d, size_t pos) const {
    rope_impl(dst, src, cos, sin, b, h, t, d, pos, true, "rope-i");
  }

  // Q and K of a packed [B, T, (hq + 2*hk) * d] QKV projection, rotated without
  // the narrow / transpose / contiguous copies (mimi.rs:1332-1351); outputs are
  // contiguous [B, T, h, d] (hq == hk).
  template <typename T>
  void rope_qk_packed(Storage<T> &q_dst, Storage<T> &k_dst, const Storage<T> &qkv, const Storage<T> &cos,
                      const Storage<T> &sin, size_t b, size_t t, size_t heads, size_t d, size_t pos,
                      bool interleaved) const {
    const size_t row = 3 * heads * d;
    expect_at_least(qkv, b * t * row, "rope_qk_packed qkv");
    expect_at_least(q_dst, b * t * heads * d, "rope_qk_packed q");
    expect_at_least(k_dst, b * t * heads * d, "rope_qk_packed k");
    if (d % 2 != 0) throw Error("rope_qk_packed requires even d dimension, got d=" + std::to_string(d));
    const size_t max_pos = d ? cos.len / (d / 2) : 0;
    if (pos + t > max_pos)
      throw Error("rope_qk_packed position out of range, pos=" + std::to_string(pos) + " + t=" + std::to_string(t) +
                      " > max_pos=" + std::to_string(max_pos),
                  XN_E_RANGE);
    check(xn_rope_qk_strided(q_dst.data, qkv.data, k_dst.data, qkv.data + heads * d, cos.data, sin.data, (int64_t)b,
                             (int64_t)heads, (int64_t)heads, (int64_t)t, (int64_t)d, (int64_t)pos, (int64_t)max_pos,
                             (int64_t)row, (int64_t)(heads * d), interleaved ? 1 : 0, DTypeOf<T>::value, stream_),
          "rope_qk_packed");
  }

  // ---- Backend::unary for Silu / GeluErf (backend.rs:57-62)
  template <typename T>
  void unary(Storage<T> &dst, const Storage<T> &src, size_t len, UnaryOp op) const {
    expect_at_least(src, len, "unary src");
    expect_at_least(dst, len, "unary dst");
    check(xn_unary(dst.data, src.data, (int64_t)len, op == UnaryOp::Silu ? XN_UNARY_SILU : XN_UNARY_GELU_ERF,
                   DTypeOf<T>::value, stream_),
          "unary");
  }

  // dst = x + layer_scale * branch (LayerScale + add, mimi.rs:1441-1444);
  // layer_scale may be null.
  template <typename T>
  void residual_add(Storage<T> &dst, const Storage<T> &x, const Storage<T> &branch, const Storage<T> *layer_scale,
                    size_t dim_m1, size_t d) const {
    for (const Storage<T> *s : {&dst, &x, &branch}) expect_len(*s, dim_m1 * d, "residual_add");
    if (layer_scale) expect_len(*layer_scale, dim_m1, "residual_add layer_scale");
    check(xn_residual_add(dst.data, x.data, branch.data, layer_scale ? layer_scale->data : nullptr, (int64_t)d,
                          (int64_t)dim_m1, DTypeOf<T>::value, stream_),
          "residual_add");
  }

  // SwiGLU: dst = silu(gate) * up on [rows, cols] (llama.rs:256-263 composite).
  template <typename T>
  void swiglu(Storage<T> &dst, const Storage<T> &gate, const Storage<T> &up, size_t rows, size_t cols,
              size_t gate_stride, size_t up_stride) const {
    expect_at_least(dst, rows * cols, "swiglu dst");
    if (rows > 0) {
      expect_at_least(gate, (rows - 1) * gate_stride + cols, "swiglu gate");
      expect_at_least(up, (rows - 1) * up_stride + cols, "swiglu up");
    }
    check(xn_swiglu(dst.data, gate.data, up.data, (int64_t)rows, (int64_t)cols, (int64_t)gate_stride,
                    (int64_t)up_stride, DTypeOf<T>::value, stream_),
          "swiglu");
  }

  // ---- Backend::softmax (backend.rs:158-163)
  template <typename T>
  void softmax(Storage<T> &dst, const Storage<T> &src, size_t dim_m1, size_t d) const {
    expect_at_least(src, dim_m1 * d, "softmax src");
    expect_at_least(dst, dim_m1 * d, "softmax dst");
    check(xn_softmax(dst.data, src.data, (int64_t)d, (int64_t)dim_m1, 0, 1, 0, DTypeOf<T>::value, stream_),
          "softmax");
  }

  // Fused apply_causality_mask + softmax on [bh, t1, t2].
  template <typename T>
  void softmax_causal(Storage<T> &dst, const Storage<T> &src, size_t bh, size_t t1, size_t t2, size_t offset) const {
    expect_at_least(src, bh * t1 * t2, "softmax_causal src");
    expect_at_least(dst, bh * t1 * t2, "softmax_causal dst");
    check(xn_softmax(dst.data, src.data, (int64_t)(bh * t1), (int64_t)t2, 1, (int64_t)(t1 ? t1 : 1),
                     (int64_t)offset, DTypeOf<T>::value, stream_),
          "softmax_causal");
  }

  // T(scores * scale), optional causal mask, softmax in one launch
  // (mimi.rs:1361-1368); `scale` is the T-typed value.
  template <typename T>
  void attn_softmax(Storage<T> &dst, const Storage<T> &src, size_t bh, size_t t1, size_t t2, float scale,
                    bool causal, size_t offset) const {
    expect_at_least(src, bh * t1 * t2, "attn_softmax src");
    expect_at_least(dst, bh * t1 * t2, "attn_softmax dst");
    check(xn_softmax_scaled(dst.data, src.data, (int64_t)(bh * t1), (int64_t)t2, scale, causal ? 1 : 0,
                            (int64_t)(t1 ? t1 : 1), (int64_t)offset, DTypeOf<T>::value, stream_),
          "attn_softmax");
  }

  // ---- Backend::apply_causality_mask (backend.rs:150-156)
  template <typename T>
  void apply_causality_mask(Storage<T> &dst, size_t bh, size_t t1, size_t t2, size_t offset) const {
    expect_at_least(dst, bh * t1 * t2, "apply_causality_mask dst");
    check(xn_causality_mask(dst.data, (int64_t)bh, (int64_t)t1, (int64_t)t2, (int64_t)offset, DTypeOf<T>::value,
                            stream_),
          "apply_causality_mask");
  }

  // ---- Backend::index_select (backend.rs:142-148) with host ids, checked on
  // the host like Tensor::index_select (tensor.rs:170-176). The ids are
  // uploaded into `ids_dev` (caller-owned, >= ids.size() u32 elements) with an
  // async copy from `ids` (caller keeps it alive until the stream reaches it).
  template <typename T>
  void index_select(Storage<T> &dst, const Storage<T> &src, const std::vector<uint32_t> &ids,
                    Storage<uint32_t> &ids_dev, size_t dim, const std::vector<size_t> &dims) const {
    if (dim >= dims.size()) throw Error("index_select dim out of range");
    const size_t dim_size = dims[dim];
    for (size_t i = 0; i < ids.size(); ++i) {
      if (ids[i] >= dim_size)
        throw Error("index_select: index " + std::to_string(ids[i]) + " at position " + std::to_string(i) +
                    " is out of bounds for dimension " + std::to_string(dim) + " with size " +
                    std::to_string(dim_size));
    }
    size_t left = 1, right = 1;
    for (size_t i = 0; i < dim; ++i) left *= dims[i];
    for (size_t i = dim + 1; i < dims.size(); ++i) right *= dims[i];
    expect_at_least(ids_dev, ids.size(), "index_select ids buffer");
    expect_at_least(dst, left * ids.size() * right, "index_select dst");
    if (!ids.empty() &&
        cudaMemcpyAsync(ids_dev.data, ids.data(), ids.size() * sizeof(uint32_t), cudaMemcpyHostToDevice, stream_) !=
            cudaSuccess)
      throw Error("index_select: id upload failed", XN_E_CUDA);
    check(xn_index_select(dst.data, src.data, ids_dev.data, 0, (int64_t)ids.size(), (int64_t)left, (int64_t)dim_size,
                          (int64_t)right, DTypeOf<T>::value, nullptr, stream_),
          "index_select");
  }

  // Device-resident ids (u32 or i64): no host round trip; err_flag (device int,
  // may be null) is set to 1 for an out-of-range id, whose row is zeroed.
  template <typename T, typename I>
  void index_select_dev(Storage<T> &dst, const Storage<T> &src, const Storage<I> &ids, size_t left,
                        size_t src_dim, size_t right, int *err_flag) const {
    static_assert(sizeof(I) == 4 || sizeof(I) == 8, "ids are u32 or i64");
    check(xn_index_select(dst.data, src.data, ids.data, sizeof(I) == 8 ? 1 : 0, (int64_t)ids.len, (int64_t)left,
                          (int64_t)src_dim, (int64_t)right, DTypeOf<T>::value, err_flag, stream_),
          "index_select_dev");
  }

  // Fused RVQ decode (mimi.rs:1627-1744): codes [batch, n_q, frames] (device i64).
  template <typename T>
  void rvq_decode_sum(Storage<T> &dst, const std::vector<const T *> &codebooks, const Storage<int64_t> &codes,
                      size_t batch, size_t frames, size_t dim, size_t bins, bool out_bct, int *err_flag) const {
    expect_at_least(codes, batch * codebooks.size() * frames, "rvq codes");
    expect_at_least(dst, batch * frames * dim, "rvq dst");
    std::vector<const void *> tabs(codebooks.begin(), codebooks.end());
    check(xn_rvq_decode_sum(dst.data, tabs.data(), (int64_t)tabs.size(), codes.data, (int64_t)batch,
                            (int64_t)frames, (int64_t)dim, (int64_t)bins, out_bct ? 1 : 0, DTypeOf<T>::value,
                            err_flag, stream_),
          "rvq_decode_sum");
  }

  // ---- Streaming decode: append the step's k / v (rotated k) to the ring
  // cache and return the rotated q [b, h, t, d] (mimi.rs:1330-1354).
  template <typename T>
  void kv_append_rope(Storage<T> &q_out, RingKvCache<T> &cache, const Storage<T> &qkv, const Storage<T> &cos,
                      const Storage<T> &sin, size_t t, bool interleaved) const {
    const size_t b = cache.b, h = cache.h, d = cache.d;
    check_cache(cache, "kv_append_rope");
    expect_at_least(qkv, b * t * 3 * h * d, "kv_append_rope qkv");
    expect_at_least(q_out, b * h * t * d, "kv_append_rope q_out");
    const size_t max_pos = decode_max_pos(cos, sin, d, cache.total, t, "kv_append_rope");
    check(xn_kv_append_rope(q_out.data, cache.k.data, cache.v.data, qkv.data, cos.data, sin.data, (int64_t)b,
                            (int64_t)h, (int64_t)t, (int64_t)d, (int64_t)cache.total, nullptr, (int64_t)max_pos,
                            (int64_t)cache.cap, interleaved ? 1 : 0, DTypeOf<T>::value, nullptr, stream_),
          "kv_append_rope");
    cache.total += t;
  }

  // Attention of q [b, h, t, d] (the step's t queries, already appended) over
  // the last min(total, context) cached positions; out is [b, t, h * d]
  // (mimi.rs:1356-1374).
  template <typename T>
  void attention_decode(Storage<T> &out, const Storage<T> &q, const RingKvCache<T> &cache, size_t t,
                        size_t context, float scale, DecodeMask mask) const {
    check_cache(cache, "attention_decode");
    if (cache.total < t) throw Error("attention_decode: the step's positions are not in the cache");
    expect_at_least(q, cache.b * cache.h * t * cache.d, "attention_decode q");
    expect_at_least(out, cache.b * t * cache.h * cache.d, "attention_decode out");
    check(xn_attention_decode(out.data, q.data, cache.k.data, cache.v.data, (int64_t)cache.b, (int64_t)cache.h,
                              (int64_t)t, (int64_t)cache.d, (int64_t)(cache.total - t), nullptr, (int64_t)cache.cap,
                              (int64_t)context, static_cast<int>(mask), scale, DTypeOf<T>::value, stream_),
          "attention_decode");
  }

  // kv_append_rope + attention_decode in one launch.
  template <typename T>
  void decode_attention_step(Storage<T> &out, RingKvCache<T> &cache, const Storage<T> &qkv,
                             const Storage<T> &cos, const Storage<T> &sin, size_t t, size_t context, float scale,
                             DecodeMask mask, bool interleaved) const {
    const size_t b = cache.b, h = cache.h, d = cache.d;
    check_cache(cache, "decode_attention_step");
    expect_at_least(qkv, b * t * 3 * h * d, "decode_attention_step qkv");
    expect_at_least(out, b * t * h * d, "decode_attention_step out");
    const size_t max_pos = decode_max_pos(cos, sin, d, cache.total, t, "decode_attention_step");
    check(xn_decode_attention_step(out.data, cache.k.data, cache.v.data, qkv.data, cos.data, sin.data, (int64_t)b,
                                   (int64_t)h, (int64_t)t, (int64_t)d, (int64_t)cache.total, nullptr,
                                   (int64_t)max_pos, (int64_t)cache.cap, (int64_t)context, static_cast<int>(mask),
                                   scale, interleaved ? 1 : 0, DTypeOf<T>::value, nullptr, stream_),
          "decode_attention_step");
    cache.total += t;
  }

 private:
  template <typename T>
  static void check_cache(const RingKvCache<T> &c, const char *op) {
    expect_at_least(c.k, c.b * c.h * c.cap * c.d, op);
    expect_at_least(c.v, c.b * c.h * c.cap * c.d, op);
  }
  template <typename T>
  static size_t decode_max_pos(const Storage<T> &cos, const Storage<T> &sin, size_t d, size_t pos, size_t t,
                               const char *op) {
    if (d % 2 != 0) throw Error(std::string(op) + " requires even d dimension, got d=" + std::to_string(d));
    if (cos.len != sin.len) throw Error(std::string(op) + " cos/sin shape mismatch");
    const size_t max_pos = d ? cos.len / (d / 2) : 0;
    if (pos + t > max_pos)
      throw Error(std::string(op) + " position out of range, pos=" + std::to_string(pos) + " + t=" +
                      std::to_string(t) + " > max_pos=" + std::to_string(max_pos),
                  XN_E_RANGE);
    return max_pos;
  }
  template <typename T>
  static void expect_len(const Storage<T> &s, size_t n, const char *what) {
    if (s.len != n)
      throw Error(std::string("shape mismatch in ") + what + ", " + std::to_string(s.len) + " <> " + std::to_string(n));
  }
  template <typename T>
  static void expect_at_least(const Storage<T> &s, size_t n, const char *what) {
    if (s.len < n)
      throw Error(std::string(what) + ": storage of " + std::to_string(s.len) + " elements, need " +
                  std::to_string(n));
  }

  template <typename T>
  void rope_impl(Storage<T> &dst, const Storage<T> &src, const Storage<T> &cos, const Storage<T> &sin, size_t b,
                 size_t h, size_t t, size_t d, size_t pos, bool interleaved, const char *op) const {
    const size_t n = b * h * t * d;
    if (dst.len != n)
      throw Error(std::string(op) + " unexpected size for dst " + std::to_string(dst.len) + " " + std::to_string(b) +
                  " " + std::to_string(h) + " " + std::to_string(t) + " " + std::to_string(d));
    if (src.len != n)
      throw Error(std::string(op) + " unexpected size for src " + std::to_string(src.len) + " " + std::to_string(b) +
                  " " + std::to_string(h) + " " + std::to_string(t) + " " + std::to_string(d));
    if (d % 2 != 0) throw Error(std::string(op) + " requires even d dimension, got d=" + std::to_string(d));
    if (cos.len != sin.len) throw Error(std::string(op) + " cos/sin shape mismatch");
    const size_t max_pos = d ? cos.len / (d / 2) : 0;
    if (pos + t > max_pos)
      throw Error(std::string(op) + " position out of range, pos=" + std::to_string(pos) + " + t=" +
                      std::to_string(t) + " > max_pos=" + std::to_string(max_pos),
                  XN_E_RANGE);
    check(xn_rope(dst.data, src.data, cos.data, sin.data, (int64_t)b, (int64_t)h, (int64_t)t, (int64_t)d,
                  (int64_t)pos, (int64_t)max_pos, interleaved ? 1 : 0, XN_LAYOUT_BHTD, DTypeOf<T>::value, stream_),
          op);
  }

  cudaStream_t stream_;
};

}  // namespace xn
