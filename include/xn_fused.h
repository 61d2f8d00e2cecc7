/*
 * xn_fused.h - C ABI of the B200 (sm_100a) fused layer-op library.
 *
 * These entry points replace the CUDA kernels behind the `xn` tensor library's
 * `Backend` trait (mimi-rs/src/backend.rs:4-309, implemented for CUDA at
 * mimi-rs/src/cuda_backend.rs:414-1451) for the bandwidth-bound layer ops:
 * RMSNorm / LayerNorm (optionally fused with the residual add and the
 * layer-scale multiply), RoPE (half-split and interleaved), SiLU / GELU(erf) /
 * SwiGLU, row softmax (optionally fused with the causal mask), the causal
 * mask itself, embedding row gather and the fused RVQ codebook gather-sum.
 *
 * Conventions shared by every entry point:
 *   - Every pointer argument that names tensor data is a DEVICE pointer, except
 *     where a comment says otherwise. Tensors are contiguous, row-major.
 *   - Sizes are int64_t element counts (never bytes, except where stated).
 *   - `stream` is a cudaStream_t / CUstream passed as void*; NULL means the
 *     legacy default stream. Work is enqueued asynchronously on it.
 *   - No entry point allocates, frees or synchronises device memory. Each one
 *     is reentrant and may be called from several host threads at once.
 *   - The return value is XN_OK (0) or one of the XN_E_* codes below. On error
 *     nothing is launched and xn_last_error() returns a message describing
 *     the failure (thread-local, valid until the next call on that thread).
 *   - Zero-sized work (rows == 0, n == 0, ...) returns XN_OK without a launch.
 *   - Arithmetic follows the reference CPU backend (mimi-rs/src/cpu_backend.rs):
 *     reductions accumulate in f32; every operation the reference performs in
 *     the element type T (bf16/f16 rounding after each +,-,*,/,exp) is rounded
 *     to T at the same point here.
 */
#ifndef XN_FUSED_H
#define XN_FUSED_H

#include <stdint.h>

/* Exported symbols keep default visibility; the library hides everything else. */
#if defined(__GNUC__)
#define XN_API __attribute__((visibility("default")))
#else
#define XN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element types; same order as `enum DType` (mimi-rs/src/dtype.rs:4-10). */
typedef enum {
  XN_F16 = 0,
  XN_BF16 = 1,
  XN_F32 = 2,
  XN_I64 = 3,
  XN_U8 = 4
} xn_dtype_t;

/* Status codes. */
enum {
  XN_OK = 0,
  XN_E_INVALID = 1,   /* bad argument: null pointer, negative size, shape mismatch */
  XN_E_DTYPE = 2,     /* dtype not supported by this op */
  XN_E_RANGE = 3,     /* a position or size is out of the table's range */
  XN_E_CUDA = 4       /* the CUDA runtime reported an error while launching */
};

/* Bits a kernel sets in a caller's device error word (err_flag). */
enum {
  XN_DEVERR_RANGE = 1,  /* an id, code or device position outside its table: that part was skipped */
  XN_DEVERR_WAIT = 2    /* a bounded wait gave up (the rows that block had not finished are NaN) */
};

/* Unary ops handled by xn_unary; names follow `enum UnaryOp`
 * (mimi-rs/src/inplace_ops.rs:5-38). */
enum {
  XN_UNARY_SILU = 0,      /* s / (1 + exp(0 - s)), T arithmetic (cpu_backend.rs:213-215) */
  XN_UNARY_GELU_ERF = 1   /* x*0.5*(1+erf(x/sqrt2)) in f32, one rounding (cpu_backend.rs:197-204) */
};

/* RoPE memory layouts. */
enum {
  XN_LAYOUT_BHTD = 0,  /* [B, H, T, D], the layout of Backend::rope / rope_i */
  XN_LAYOUT_BTHD = 1   /* [B, T, H, D], e.g. the projection output before transpose */
};

/* Maximum number of codebooks accepted by xn_rvq_decode_sum. */
#define XN_RVQ_MAX_CODEBOOKS 32

/* Message for the last failing call on this thread ("" if none). */
XN_API const char *xn_last_error(void);

/* ABI version, bumped on any incompatible change of a signature below. */
XN_API int xn_abi_version(void);

/*
 * RMSNorm over the last dimension, optionally fused with the residual add.
 * Replaces Backend::rms_norm (mimi-rs/src/backend.rs:165-172; CUDA dispatch
 * mimi-rs/src/cuda_backend.rs:1005-1035; CPU semantics cpu_backend.rs:691-709).
 *
 *   h   = src                                    if branch == NULL
 *   h   = T(src + branch)                        if layer_scale == NULL
 *   h   = T(src + T(branch * layer_scale[col]))  otherwise
 *   residual_out = h                             if residual_out != NULL
 *   dst = T(h / sqrt(sum(h^2)/cols + eps) * alpha[col])
 *
 * With branch == NULL this is exactly Backend::rms_norm(dst, src, alpha,
 * dim_m1 = cols, d = rows, eps). The fused form replaces the composite
 * `residual.add(&branch)` + `rms_norm` of mimi-rs/src/models/llama.rs:310-313
 * (and LayerScale, mimi-rs/src/models/mimi.rs:1199-1201,1433-1439).
 * eps must be > 0 (mimi-rs/src/inplace_ops.rs:261). dst may alias src;
 * residual_out may alias src or branch.
 */
XN_API int xn_rms_norm(void *dst, const void *src, const void *alpha,
                const void *branch, const void *layer_scale, void *residual_out,
                int64_t rows, int64_t cols, float eps, int dtype, void *stream);

/*
 * LayerNorm over the last dimension (two-pass f32 mean / variance), with the
 * same optional residual / layer-scale prologue as xn_rms_norm.
 * Replaces Backend::layer_norm (mimi-rs/src/backend.rs:180-189; CUDA dispatch
 * mimi-rs/src/cuda_backend.rs:1037-1072; CPU semantics cpu_backend.rs:711-750).
 *
 *   mean = sum(h)/cols ; var = sum((h-mean)^2)/cols ; inv = 1/sqrt(var+eps)
 *   dst  = T(((remove_mean ? h-mean : h) * inv) * weight[col] + bias[col])
 *
 * weight == NULL acts as all ones and bias == NULL as all zeros. The fused
 * form replaces `layer_scale.forward` + `xs.add` + `norm2.forward` of
 * mimi-rs/src/models/mimi.rs:1433-1439.
 */
XN_API int xn_layer_norm(void *dst, const void *src, const void *weight, const void *bias,
                  const void *branch, const void *layer_scale, void *residual_out,
                  int64_t rows, int64_t cols, float eps, int remove_mean,
                  int dtype, void *stream);

/*
 * Rotary position embedding on one tensor of b*h*t rows of d elements.
 * Replaces Backend::rope (interleaved == 0; mimi-rs/src/backend.rs:101-111,
 * cuda_backend.rs:681-716, cpu_backend.rs:359-392) and Backend::rope_i
 * (interleaved != 0; backend.rs:114-124, cuda_backend.rs:718-751,
 * cpu_backend.rs:394-422).
 *
 * cos / sin are [max_pos, d/2] tables of the same dtype; row (pos + t) is used
 * for time step t. pos + t must be <= max_pos and d must be even
 * (mimi-rs/src/inplace_ops.rs:421-473). layout selects [B,H,T,D] (the
 * reference layout) or [B,T,H,D], which removes the transpose + contiguous
 * copies callers make around rope (pocket_tts/src/rope.rs:42-48,
 * mimi-rs/src/models/llama.rs:160-167). dst may alias src.
 */
XN_API int xn_rope(void *dst, const void *src, const void *cos, const void *sin,
            int64_t b, int64_t h, int64_t t, int64_t d, int64_t pos, int64_t max_pos,
            int interleaved, int layout, int dtype, void *stream);

/*
 * Q and K rotated in one launch (same b, t, d, pos, tables and layout;
 * hq and hk heads). Equivalent to two xn_rope calls
 * (mimi-rs/src/models/mimi.rs:1350-1351, llama.rs:171-172).
 */
XN_API int xn_rope_qk(void *q_dst, const void *q_src, void *k_dst, const void *k_src,
               const void *cos, const void *sin,
               int64_t b, int64_t hq, int64_t hk, int64_t t, int64_t d,
               int64_t pos, int64_t max_pos, int interleaved, int layout,
               int dtype, void *stream);

/*
 * Q and K rotated in place of the narrow + reshape + transpose + contiguous
 * copies the reference makes from the packed QKV projection
 * (mimi-rs/src/models/mimi.rs:1332-1351): both tensors are in [B, T, H, D]
 * layout with `src_tok_stride` elements between consecutive (b, t) tokens
 * (3 * H * D inside a packed [B, T, 3*H*D] projection, where k_src =
 * q_src + H * D) and outputs written with `dst_tok_stride` (H * D for
 * contiguous [B, T, H, D] outputs; equal to the source layout for in-place).
 * Arithmetic as xn_rope.
 */
XN_API int xn_rope_qk_strided(void *q_dst, const void *q_src, void *k_dst, const void *k_src,
                              const void *cos, const void *sin,
                              int64_t b, int64_t hq, int64_t hk, int64_t t, int64_t d,
                              int64_t pos, int64_t max_pos, int64_t src_tok_stride,
                              int64_t dst_tok_stride, int interleaved, int dtype, void *stream);

/*
 * Elementwise unary op on n elements (XN_UNARY_SILU or XN_UNARY_GELU_ERF).
 * Replaces Backend::unary for those ops (mimi-rs/src/backend.rs:57-62,
 * cuda_backend.rs:523-554, cpu_backend.rs:184-222). dst may alias src.
 */
XN_API int xn_unary(void *dst, const void *src, int64_t n, int op, int dtype, void *stream);

/*
 * Residual add with optional layer scale on [rows, cols]:
 *   dst = T(x + T(branch * layer_scale[col]))   (or T(x + branch))
 * Replaces LayerScale::forward (broadcast_mul, cpu_backend.rs:1379-1387) +
 * Tensor::add of mimi-rs/src/models/mimi.rs:1441-1444 where no norm follows
 * (the last layer of a stack); elsewhere the norms fuse it. dst may alias x.
 */
XN_API int xn_residual_add(void *dst, const void *x, const void *branch, const void *layer_scale,
                           int64_t rows, int64_t cols, int dtype, void *stream);

/*
 * SwiGLU: dst[r, c] = T(T(silu(gate[r, c])) * up[r, c]), silu in T arithmetic.
 * Replaces the composite `silu` + `mul` of mimi-rs/src/models/llama.rs:256-263
 * (Backend::unary then Backend::binary, cpu_backend.rs:213-215,224-258).
 * dst is contiguous [rows, cols]; gate / up rows start every gate_stride /
 * up_stride elements, so both may be halves of one fused projection output.
 */
XN_API int xn_swiglu(void *dst, const void *gate, const void *up, int64_t rows, int64_t cols,
              int64_t gate_stride, int64_t up_stride, int dtype, void *stream);

/*
 * Row softmax over the last dimension, optionally fused with the causal mask.
 * Replaces Backend::softmax (mimi-rs/src/backend.rs:158-163,
 * cuda_backend.rs:978-1003, cpu_backend.rs:667-689); with causal != 0 it also
 * replaces the Backend::apply_causality_mask that precedes it
 * (backend.rs:150-156, cpu_backend.rs:647-665; callers mimi.rs:1365-1368,
 * llama.rs:201-202). rows = bh * t1; row r is query (r % t1) and its columns
 * j > offset + (r % t1) give exactly 0 (they are not read). dst may equal src
 * (in place). Any width and alignment; 16-byte-aligned tensors run the vector
 * kernels, also for widths that are not a multiple of the vector.
 */
XN_API int xn_softmax(void *dst, const void *src, int64_t rows, int64_t cols,
               int causal, int64_t t1, int64_t offset, int dtype, void *stream);

/*
 * xn_softmax preceded by the attention-score scale: x = T(x * scale), then
 * the optional causal mask and the softmax. Replaces `scale` (Tensor::scale,
 * mimi-rs/src/ops.rs:101-105, cpu_backend.rs:260-276) + mask + softmax of
 * mimi-rs/src/models/mimi.rs:1361-1368 and llama.rs:192-202. `scale` is the
 * T-typed value the caller uses (T::from_f32(1 / sqrt(head_dim))).
 */
XN_API int xn_softmax_scaled(void *dst, const void *src, int64_t rows, int64_t cols, float scale,
                             int causal, int64_t t1, int64_t offset, int dtype, void *stream);

/*
 * xn_softmax (scaled == 0) or xn_softmax_scaled (scaled != 0) with a device
 * status word: err_flag (a device int, may be NULL) gets XN_DEVERR_WAIT when a
 * shared-memory stage of the wide-row kernel did not arrive within its bounded
 * wait; that kernel then waits (bounded) for its copies in flight, writes NaN
 * to the rows it had not finished and returns, so a lost copy shows as a
 * status instead of a hang. It cannot happen with valid arguments. The
 * environment variable XN_STAGE_WAIT_POLLS (read once per process) lowers the
 * number of polls before the wait gives up, for testing that path. No
 * reference counterpart: the reference's softmax has no waits
 * (mimi-rs/cuda-kernels/reduce.cu:178-220).
 */
XN_API int xn_softmax_status(void *dst, const void *src, int64_t rows, int64_t cols, int scaled, float scale,
                             int causal, int64_t t1, int64_t offset, int *err_flag, int dtype, void *stream);

/*
 * In-place causal mask on [bh, t1, t2]: x[b, i, j] = -inf where j > offset + i.
 * Replaces Backend::apply_causality_mask (mimi-rs/src/backend.rs:150-156,
 * cuda_backend.rs:951-976, cpu_backend.rs:647-665).
 */
XN_API int xn_causality_mask(void *dst, int64_t bh, int64_t t1, int64_t t2, int64_t offset,
                      int dtype, void *stream);

/*
 * Row gather: dst[l, i, :] = src[l, ids[i], :] for l < left, i < n_ids, with
 * rows of `right` elements and src_dim rows per l. ids are device u32
 * (ids_is_i64 == 0) or i64. Bit-exact copy for every dtype.
 * Replaces Backend::index_select (mimi-rs/src/backend.rs:142-148,
 * cuda_backend.rs:899-949, cpu_backend.rs:624-645) without its host upload of
 * the ids (cuda_backend.rs:911). An id outside [0, src_dim) gives a zero row
 * and sets *err_flag to 1 when err_flag (a device int) is not NULL: the
 * reference rejects such ids on the host (mimi-rs/src/tensor.rs:170-176).
 */
XN_API int xn_index_select(void *dst, const void *src, const void *ids, int ids_is_i64,
                    int64_t n_ids, int64_t left, int64_t src_dim, int64_t right,
                    int dtype, int *err_flag, void *stream);

/*
 * Fused RVQ decode: for codes [batch, n_q, frames] (device i64, the layout
 * ResidualVectorQuantizer::decode receives) and n_q codebooks of
 * [bins, dim] (`tables` is a HOST array of n_q device pointers),
 *   out[b, t, :] = (((E_0[c_0] + E_1[c_1]) + E_2[c_2]) + ...)   rounded to T per add
 * written as [batch, dim, frames] when out_bct != 0 (the `.t().contiguous()`
 * layout of VectorQuantization::decode) else [batch, frames, dim].
 * Replaces EuclideanCodebook::decode + VectorQuantization::decode +
 * ResidualVectorQuantization::decode (mimi-rs/src/models/mimi.rs:1627-1643,
 * 1683-1690, 1730-1744): one launch instead of n_q host syncs, uploads,
 * gathers, transposes and adds. A code outside [0, bins) contributes zeros and
 * sets *err_flag to 1 when err_flag is not NULL. n_q <= XN_RVQ_MAX_CODEBOOKS.
 */
XN_API int xn_rvq_decode_sum(void *dst, const void *const *tables, int64_t n_q,
                      const int64_t *codes, int64_t batch, int64_t frames,
                      int64_t dim, int64_t bins, int out_bct, int dtype,
                      int *err_flag, void *stream);

/*
 * Streaming decode, KV cache (next-step rows of the hot path).
 *
 * A layer's cache is a ring buffer per (batch, head): k_cache and v_cache are
 * [b, h, cap, d]. `total` counts the positions appended before the call; the
 * t new positions go to slots (total + i) % cap. After the append the cache
 * holds the n = total + t positions seen, of which the last
 * kv_len = min(n, context) (context <= cap) are attended, oldest first
 * (logical key j at slot (n - kv_len + j) % cap). This is the state of the
 * reference's cat-then-trim caches (mimi-rs/src/models/mimi.rs:1122-1153,
 * pocket_tts/src/mimi_transformer.rs:32-61; with context = cap = the
 * preallocated length it is the slice_set cache of
 * pocket_tts/src/transformer.rs:16-33) without their per-step copies.
 *
 * When total_dev is not NULL it points at the device copy of `total` (an
 * int64) and `total` is ignored, so one captured CUDA graph serves every step;
 * xn_position_advance then adds t on the device at the end of a step.
 */
enum {
  XN_MASK_RELATIVE = 0,  /* key j visible to query i iff j <= i + kv_len - t
                            (pocket_tts/src/transformer.rs:35-52) */
  XN_MASK_ABSOLUTE = 1,  /* iff j <= total + i: apply_causality_mask(offset) on
                            the trimmed cache with offset = the absolute position
                            (pocket_tts/src/mimi_transformer.rs:114-145) */
  XN_MASK_CACHE_LEN = 2  /* mimi-rs StreamingTransformer::forward
                            (mimi-rs/src/models/mimi.rs:1476-1487): offset = the
                            cache's length before the step, min(total, context),
                            used as the RoPE position of the new rows (rope_i at
                            offset, :1350-1351) and as the mask offset (:1364).
                            The visible keys are those of XN_MASK_ABSOLUTE; only
                            the rotation differs once the context is full. In
                            xn_attention_decode (no rotation) it equals
                            XN_MASK_ABSOLUTE; xn_kv_append_rope rotates at
                            `total`, so a caller of this mode uses the fused
                            xn_decode_attention_step. */
};

/*
 * KV-cache append fused with RoPE, reading the packed QKV projection
 * qkv [b, t, 3, h, d] (q | k | v, the in_proj output):
 *   q_out [b, h, t, d] = rope(q) at positions total + i
 *   k_cache slot (total + i) % cap = rope(k) ; v_cache slot = v
 * Replaces narrow/reshape/transpose/contiguous + rope_i on q and k +
 * KvCache::append (mimi-rs/src/models/mimi.rs:1330-1354;
 * pocket_tts/src/mimi_transformer.rs:122-137). RoPE arithmetic as xn_rope
 * (interleaved or half-split; cos/sin [max_pos, d/2]); requires
 * total + t <= max_pos and t <= cap. With total_dev, a position outside the
 * tables skips that step's writes and sets *err_flag (when not NULL) to 1.
 */
XN_API int xn_kv_append_rope(void *q_out, void *k_cache, void *v_cache, const void *qkv,
                      const void *cos, const void *sin, int64_t b, int64_t h, int64_t t,
                      int64_t d, int64_t total, const int64_t *total_dev, int64_t max_pos,
                      int64_t cap, int interleaved, int dtype, int *err_flag, void *stream);

/*
 * Decode attention over the ring cache, one launch for
 *   scores = T(T(q . k_j) * T(scale)), causal mask (mask_mode), softmax as
 *   xn_softmax, out = T(sum_j p_j v_j)
 * i.e. q.matmul_t(k).scale(scale), apply_causality_mask / mask add, softmax,
 * matmul(v) (mimi-rs/src/models/mimi.rs:1356-1371,
 * pocket_tts/src/transformer.rs:134-145). q [b, h, t, d] (xn_kv_append_rope's
 * q_out); out [b, t, h, d] = the [b, t, h*d] out_proj input (the reference's
 * transpose + reshape). The dot products and the weighted sum accumulate in
 * f32 in key order. d must be 32, 64 or 128; context <= 8192.
 */
XN_API int xn_attention_decode(void *out, const void *q, const void *k_cache, const void *v_cache,
                        int64_t b, int64_t h, int64_t t, int64_t d, int64_t total,
                        const int64_t *total_dev, int64_t cap, int64_t context, int mask_mode,
                        float scale, int dtype, void *stream);

/*
 * xn_kv_append_rope followed by xn_attention_decode in one launch: each
 * (batch, head, query) block writes its head's t new k (rotated) and v rows
 * into the ring caches and rotates its query on chip, then attends. Same
 * results as the two calls (q is not written out). qkv, cos and sin must be
 * 16-byte aligned. With total_dev, a position outside the tables skips the
 * step and sets *err_flag (when not NULL) to 1.
 */
XN_API int xn_decode_attention_step(void *out, void *k_cache, void *v_cache, const void *qkv,
                             const void *cos, const void *sin, int64_t b, int64_t h, int64_t t,
                             int64_t d, int64_t total, const int64_t *total_dev, int64_t max_pos,
                             int64_t cap, int64_t context, int mask_mode, float scale,
                             int interleaved, int dtype, int *err_flag, void *stream);

/* *total_dev += t on the device, ordered on `stream` (end of a decode step). */
XN_API int xn_position_advance(int64_t *total_dev, int64_t t, void *stream);

/*
 * Row-shard plan for splitting `rows` over `world` GPUs: contiguous blocks of
 * ceil(rows / world) rows; writes this rank's first row and row count (host
 * pointers). No reference counterpart: the reference is single-GPU.
 */
XN_API int xn_shard_rows(int64_t rows, int world, int rank, int64_t *begin, int64_t *count);

#ifdef __cplusplus
}
#endif

#endif /* XN_FUSED_H */
