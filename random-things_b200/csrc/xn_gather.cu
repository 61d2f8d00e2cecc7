// xn_gather.cu - embedding row gather (index_select) with device-resident ids,
// and the fused RVQ codebook gather-sum, for sm_100a.
//
// Reference semantics: mimi-rs/src/cpu_backend.rs:624-645 (index_select, a
// byte copy) and the RVQ decode chain mimi-rs/src/models/mimi.rs:1627-1744
// (per codebook: gather rows, transpose to [B, dim, T], add in codebook order
// with T rounding per add).
//
// Design: warps stride over (output row, 2 KB chunk) work items and copy each
// chunk with 16-byte vector loads, four in flight per lane before the stores;
// the grid is capped at 8 blocks per SM. Ids are read on the device
// (no host round trip); an out-of-range id yields a zero row and raises a
// device error flag instead of faulting. The RVQ kernel sums the n_q codebook
// rows of a frame in registers and, for the [B, dim, T] layout, transposes a
// tile of 32 frames through shared memory so the stores stay coalesced.
#include <type_traits>

#include "xn_common.cuh"
#include "xn_internal.h"

namespace xn {
namespace {

struct GatherParams {
  void *dst;
  const void *src;
  const void *ids;
  int *err;
  int64_t n_ids;
  int64_t out_rows;   // left * n_ids
  int64_t src_dim;
  int64_t row_units;  // row length in access units
  int ids_i64;
};

__device__ __forceinline__ int64_t load_id(const void *ids, int64_t i, int ids_i64) {
  return ids_i64 ? static_cast<const int64_t *>(ids)[i]
                 : static_cast<int64_t>(static_cast<const uint32_t *>(ids)[i]);
}

// U = access unit type (uint4 for 16-byte vectors, else the element type).
// Work items are (output row, chunk of 32 x kUnroll units); warps stride over
// them, so a grid of a few blocks per SM stays evenly loaded to the end (one
// warp per whole row would leave the last wave of rows half empty).
constexpr int kGatherUnroll = 4;

template <typename U>
__global__ void __launch_bounds__(256) gather_rows_kernel(const GatherParams p) {
  griddep_wait();
  griddep_release();
  const int lane = threadIdx.x & 31;
  const int64_t units_per_chunk = 32 * kGatherUnroll;
  const int64_t chunks = (p.row_units + units_per_chunk - 1) / units_per_chunk;
  const int64_t items = p.out_rows * chunks;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); item < items;
       item += warps) {
    const int64_t orow = item / chunks;
    const int64_t c = item - orow * chunks;
    const int64_t l = orow / p.n_ids;
    const int64_t i = orow - l * p.n_ids;
    const int64_t id = load_id(p.ids, i, p.ids_i64);
    U *d = static_cast<U *>(p.dst) + orow * p.row_units;
    const int64_t u_begin = c * units_per_chunk;
    if (id < 0 || id >= p.src_dim) {
      if (lane == 0 && p.err != nullptr) atomicOr(p.err, 1);
#pragma unroll
      for (int k = 0; k < kGatherUnroll; ++k) {
        const int64_t u = u_begin + lane + k * 32;
        if (u < p.row_units) d[u] = U{};
      }
      continue;
    }
    const U *s = static_cast<const U *>(p.src) + (l * p.src_dim + id) * p.row_units;
    U v[kGatherUnroll];
#pragma unroll
    for (int k = 0; k < kGatherUnroll; ++k) {
      const int64_t u = u_begin + lane + k * 32;
      if (u < p.row_units) {
        if constexpr (sizeof(U) == 16) {
          v[k] = ld_stream(s + u);
        } else {
          v[k] = s[u];
        }
      }
    }
#pragma unroll
    for (int k = 0; k < kGatherUnroll; ++k) {
      const int64_t u = u_begin + lane + k * 32;
      if (u < p.row_units) d[u] = v[k];
    }
  }
}

// Rows shorter than a warp's 32 x kUnroll units: a work item is `rpi`
// consecutive output rows, read as one flat span of rpi * row_units units, so
// every lane still has kUnroll accesses in flight and the stores of a warp are
// one contiguous run. Each lane looks up the id of the row its unit falls in.
template <typename U>
__global__ void __launch_bounds__(256) gather_short_rows_kernel(const GatherParams p, int rpi) {
  griddep_wait();
  griddep_release();
  const int lane = threadIdx.x & 31;
  const int ru = static_cast<int>(p.row_units);  // < 32 * kGatherUnroll
  const int span = rpi * ru;
  const int64_t items = (p.out_rows + rpi - 1) / rpi;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const bool one_slice = p.out_rows == p.n_ids;  // left == 1: no division by n_ids
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); item < items;
       item += warps) {
    const int64_t row0 = item * rpi;
    U v[kGatherUnroll];
    bool live[kGatherUnroll];
#pragma unroll
    for (int k = 0; k < kGatherUnroll; ++k) {
      const int f = lane + k * 32;
      const int r = f / ru;
      const int64_t orow = row0 + r;
      live[k] = f < span && orow < p.out_rows;
      v[k] = U{};
      if (live[k]) {
        const int64_t l = one_slice ? 0 : orow / p.n_ids;
        const int64_t i = orow - l * p.n_ids;
        const int64_t id = load_id(p.ids, i, p.ids_i64);
        if (id < 0 || id >= p.src_dim) {
          if (p.err != nullptr) atomicOr(p.err, 1);
        } else {
          const U *src = static_cast<const U *>(p.src) + (l * p.src_dim + id) * p.row_units + (f - r * ru);
          if constexpr (sizeof(U) == 16) {
            v[k] = ld_stream(src);
          } else {
            v[k] = *src;
          }
        }
      }
    }
    U *d = static_cast<U *>(p.dst) + row0 * p.row_units;
#pragma unroll
    for (int k = 0; k < kGatherUnroll; ++k)
      if (live[k]) d[lane + k * 32] = v[k];
  }
}

struct RvqTables {
  const void *p[XN_RVQ_MAX_CODEBOOKS];
};

struct RvqParams {
  RvqTables tab;
  void *dst;
  const int64_t *codes;  // [batch, nq, frames]
  int *err;
  int64_t batch, frames, dim, bins;
  int nq;
  int nvec;  // accesses per row
};

// Loads this frame's codes: lane q holds code q (nq <= 32), flags bad codes.
__device__ __forceinline__ int64_t frame_code(const RvqParams &p, int64_t b, int64_t t, int lane) {
  int64_t c = 0;
  if (lane < p.nq) {
    c = __ldg(p.codes + (b * p.nq + lane) * p.frames + t);
    if (c < 0 || c >= p.bins) {
      if (p.err != nullptr) atomicOr(p.err, 1);
      c = -1;
    }
  }
  return c;
}

// Lane q (< nq) holds the address of the row of codebook q that this frame's
// code selects, null for a bad code (its row adds +0.0). The other lanes read
// the addresses by shuffle, so each codebook pointer is fetched once per frame.
template <typename T>
__device__ __forceinline__ uintptr_t frame_row(const RvqParams &p, int64_t b, int64_t t, int lane) {
  const int64_t c = frame_code(p, b, t, lane);
  if (lane >= p.nq || c < 0) return 0;
  return reinterpret_cast<uintptr_t>(static_cast<const T *>(p.tab.p[lane]) + c * p.dim);
}

// Sum of the nq codebook rows for access unit u of the frame, in f32 values
// rounded to T after every add (the reference's T-typed adds in codebook
// order).
template <typename T, bool kVector>
__device__ __forceinline__ void frame_sum(const RvqParams &p, uintptr_t row_lane, int u,
                                          float (&acc)[kVector ? Elem<T>::kVec : 1]) {
  constexpr int N = kVector ? Elem<T>::kVec : 1;
  for (int q = 0; q < p.nq; ++q) {
    const T *row = reinterpret_cast<const T *>(__shfl_sync(0xffffffffu, row_lane, q));
    float v[N];
    if (row != nullptr) {
      if constexpr (kVector) {
        unpack<T>(ld_cached(row + static_cast<int64_t>(u) * N), v);
      } else {
        v[0] = Elem<T>::to_f32(__ldg(row + u));
      }
    } else {
#pragma unroll
      for (int j = 0; j < N; ++j) v[j] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < N; ++j) acc[j] = q == 0 ? v[j] : Elem<T>::round(__fadd_rn(acc[j], v[j]));
  }
}

// The same sum for 16-bit vector rows, kept packed: each add is one paired
// bf16x2 / f16x2 add, which rounds the exact sum of two T values once. That is
// the reference's f32 add followed by rounding to T: f32's 24 bits are at
// least 2p + 2 for T's p-bit significand (p = 8 or 11), so the double rounding
// is innocuous. Up to 8 codebook rows are loaded before they are added.
template <typename T>
__device__ __forceinline__ uint4 frame_sum_packed(const RvqParams &p, uintptr_t row_lane, int u) {
  uint4 acc = make_uint4(0u, 0u, 0u, 0u);
  for (int q0 = 0; q0 < p.nq; q0 += 8) {
    uint4 v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uintptr_t a = __shfl_sync(0xffffffffu, row_lane, (q0 + k) & 31);
      v[k] = make_uint4(0u, 0u, 0u, 0u);
      if (q0 + k < p.nq && a != 0) v[k] = ld_cached(reinterpret_cast<const T *>(a) + static_cast<int64_t>(u) * 8);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (q0 + k == 0) {
        acc = v[k];
      } else if (q0 + k < p.nq) {
        acc = make_uint4(t2_add<T>(acc.x, v[k].x), t2_add<T>(acc.y, v[k].y), t2_add<T>(acc.z, v[k].z),
                         t2_add<T>(acc.w, v[k].w));
      }
    }
  }
  return acc;
}

template <typename T, bool kVector>
constexpr bool kPackedSum = kVector && !std::is_same_v<T, float>;

// [batch, frames, dim] output: one warp per frame.
template <typename T, bool kVector>
__global__ void __launch_bounds__(256) rvq_btd_kernel(const RvqParams p) {
  griddep_wait();
  griddep_release();
  constexpr int N = kVector ? Elem<T>::kVec : 1;
  const int lane = threadIdx.x & 31;
  const int64_t frame = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (frame >= p.batch * p.frames) return;
  const int64_t b = frame / p.frames;
  const int64_t t = frame - b * p.frames;
  const uintptr_t row_lane = frame_row<T>(p, b, t, lane);
  T *out = static_cast<T *>(p.dst) + frame * p.dim;
  for (int u0 = 0; u0 < p.nvec; u0 += 32) {
    const int u = u0 + lane;
    // All lanes run the sum (it shuffles); only in-range units are stored.
    if constexpr (kPackedSum<T, kVector>) {
      const uint4 sum = frame_sum_packed<T>(p, row_lane, u < p.nvec ? u : 0);
      if (u < p.nvec) st_vec(out + static_cast<int64_t>(u) * N, sum);
    } else {
      float acc[N];
      frame_sum<T, kVector>(p, row_lane, u < p.nvec ? u : 0, acc);
      if (u < p.nvec) {
        if constexpr (kVector) {
          st_vec(out + static_cast<int64_t>(u) * N, pack<T>(acc));
        } else {
          out[u] = Elem<T>::from_f32(acc[0]);
        }
      }
    }
  }
}

// [batch, dim, frames] output: a block owns 32 frames of one batch element;
// warp w computes frames w, w+8, ... into a shared tile [32][dim+1] (f32),
// then each warp writes 32 consecutive frames of a channel per store.
template <typename T, bool kVector>
__global__ void __launch_bounds__(256) rvq_bct_kernel(const RvqParams p) {
  griddep_wait();
  griddep_release();
  constexpr int N = kVector ? Elem<T>::kVec : 1;
  extern __shared__ float tile[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t tiles_per_b = (p.frames + 31) / 32;
  const int64_t b = blockIdx.x / tiles_per_b;
  const int64_t t0 = (blockIdx.x - b * tiles_per_b) * 32;
  const int64_t ld = p.dim + 1;
  for (int f = warp; f < 32; f += 8) {
    const int64_t t = t0 + f;
    if (t >= p.frames) break;
    const uintptr_t row_lane = frame_row<T>(p, b, t, lane);
    for (int u0 = 0; u0 < p.nvec; u0 += 32) {
      const int u = u0 + lane;
      float acc[N];
      if constexpr (kPackedSum<T, kVector>) {
        unpack<T>(frame_sum_packed<T>(p, row_lane, u < p.nvec ? u : 0), acc);
      } else {
        frame_sum<T, kVector>(p, row_lane, u < p.nvec ? u : 0, acc);
      }
      if (u < p.nvec) {
#pragma unroll
        for (int j = 0; j < N; ++j) tile[f * ld + static_cast<int64_t>(u) * N + j] = acc[j];
      }
    }
  }
  __syncthreads();
  T *out = static_cast<T *>(p.dst) + b * p.dim * p.frames;
  const int64_t t = t0 + lane;
  if (t < p.frames) {
    for (int64_t c = warp; c < p.dim; c += 8) out[c * p.frames + t] = Elem<T>::from_f32(tile[lane * ld + c]);
  }
}

// Fallback for very wide codebook rows in [batch, dim, frames]: strided stores.
template <typename T>
__global__ void __launch_bounds__(256) rvq_bct_wide_kernel(const RvqParams p) {
  griddep_wait();
  griddep_release();
  const int lane = threadIdx.x & 31;
  const int64_t frame = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (frame >= p.batch * p.frames) return;
  const int64_t b = frame / p.frames;
  const int64_t t = frame - b * p.frames;
  const uintptr_t row_lane = frame_row<T>(p, b, t, lane);
  T *out = static_cast<T *>(p.dst) + b * p.dim * p.frames + t;
  for (int u0 = 0; u0 < p.nvec; u0 += 32) {
    const int u = u0 + lane;
    float acc[1];
    frame_sum<T, false>(p, row_lane, u < p.nvec ? u : 0, acc);
    if (u < p.nvec) out[static_cast<int64_t>(u) * p.frames] = Elem<T>::from_f32(acc[0]);
  }
}

constexpr int64_t kRvqTileMaxDim = 1024;

template <typename T>
int launch_rvq(RvqParams p, int out_bct, cudaStream_t st) {
  constexpr int V = Elem<T>::kVec;
  bool vec = p.dim % V == 0;
  for (int q = 0; q < p.nq; ++q) vec = vec && is_aligned16(p.tab.p[q]);
  vec = vec && (out_bct || is_aligned16(p.dst));
  p.nvec = static_cast<int>(vec ? p.dim / V : p.dim);
  const int64_t frames_total = p.batch * p.frames;
  if (!out_bct) {
    const int64_t grid = ceil_div(frames_total, 8);
    if (vec)
      launch_k(rvq_btd_kernel<T, true>, dim3(grid), dim3(256), 0, st, p);
    else
      launch_k(rvq_btd_kernel<T, false>, dim3(grid), dim3(256), 0, st, p);
  } else if (p.dim <= kRvqTileMaxDim) {
    const int64_t grid = p.batch * ((p.frames + 31) / 32);
    const size_t smem = static_cast<size_t>(32) * (p.dim + 1) * sizeof(float);
    if (vec) {
      if (smem > 48 * 1024) cudaFuncSetAttribute(rvq_bct_kernel<T, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      launch_k(rvq_bct_kernel<T, true>, dim3(grid), dim3(256), smem, st, p);
    } else {
      if (smem > 48 * 1024) cudaFuncSetAttribute(rvq_bct_kernel<T, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      launch_k(rvq_bct_kernel<T, false>, dim3(grid), dim3(256), smem, st, p);
    }
  } else {
    p.nvec = static_cast<int>(p.dim);
    launch_k(rvq_bct_wide_kernel<T>, dim3(ceil_div(frames_total, 8)), dim3(256), 0, st, p);
  }
  return check_launch("xn_rvq_decode_sum");
}

}  // namespace
}  // namespace xn

extern "C" {

int xn_index_select(void *dst, const void *src, const void *ids, int ids_is_i64, int64_t n_ids,
                    int64_t left, int64_t src_dim, int64_t right, int dtype, int *err_flag,
                    void *stream) {
  using namespace xn;
  const int eb = dtype_bytes(dtype);
  if (eb == 0) return fail(XN_E_DTYPE, "xn_index_select: unsupported dtype %d", dtype);
  if (n_ids < 0 || left < 0 || src_dim < 0 || right < 0)
    return fail(XN_E_INVALID, "xn_index_select: negative size");
  const int64_t out_rows = left * n_ids;
  if (out_rows == 0 || right == 0) return ok();
  if (dst == nullptr || ids == nullptr || (src == nullptr && src_dim > 0))
    return fail(XN_E_INVALID, "xn_index_select: null pointer");
  const int64_t row_bytes = right * eb;
  GatherParams p{dst, src, ids, err_flag, n_ids, out_rows, src_dim, 0, ids_is_i64 ? 1 : 0};
  cudaStream_t st = as_stream(stream);
  const bool vec = row_bytes % 16 == 0 && is_aligned16(dst) && is_aligned16(src);
  p.row_units = vec ? row_bytes / 16 : right;
  // Enough warps for every work item. Rows of at most half a warp's span are
  // packed several to a work item, and those grids (and the element-access
  // ones) are capped at 8 blocks of 8 warps per SM, the warps walking the
  // items. Longer 16-byte rows take one item per warp, all at once: no warp
  // waits on its next id behind its own row copies (bf16 rows of 4096-16384
  // columns: 0.96-0.98 -> 1.00-1.03 of the copy peak; short rows measured
  // faster with the cap, 262144 x 256 bf16 0.91 against 0.79).
  const int64_t span = 32 * kGatherUnroll;
  const int rpi = p.row_units > 0 && p.row_units * 2 <= span ? static_cast<int>(span / p.row_units) : 1;
  const int64_t items = rpi > 1 ? ceil_div(out_rows, static_cast<int64_t>(rpi)) : out_rows * ceil_div(p.row_units, span);
  int64_t grid = ceil_div(items, 8);
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (grid > cap && (!vec || rpi > 1)) grid = cap;
  if (grid > 0x7fffffffLL) grid = 0x7fffffffLL;
  if (vec && rpi > 1) {
    launch_k(gather_short_rows_kernel<uint4>, dim3(grid), dim3(256), 0, st, p, rpi);
  } else if (vec) {
    launch_k(gather_rows_kernel<uint4>, dim3(grid), dim3(256), 0, st, p);
  } else if (rpi > 1) {
    switch (eb) {
      case 1:
        launch_k(gather_short_rows_kernel<uint8_t>, dim3(grid), dim3(256), 0, st, p, rpi);
        break;
      case 2:
        launch_k(gather_short_rows_kernel<uint16_t>, dim3(grid), dim3(256), 0, st, p, rpi);
        break;
      case 4:
        launch_k(gather_short_rows_kernel<uint32_t>, dim3(grid), dim3(256), 0, st, p, rpi);
        break;
      default:
        launch_k(gather_short_rows_kernel<unsigned long long>, dim3(grid), dim3(256), 0, st, p, rpi);
        break;
    }
  } else {
    switch (eb) {
      case 1:
        launch_k(gather_rows_kernel<uint8_t>, dim3(grid), dim3(256), 0, st, p);
        break;
      case 2:
        launch_k(gather_rows_kernel<uint16_t>, dim3(grid), dim3(256), 0, st, p);
        break;
      case 4:
        launch_k(gather_rows_kernel<uint32_t>, dim3(grid), dim3(256), 0, st, p);
        break;
      default:
        launch_k(gather_rows_kernel<unsigned long long>, dim3(grid), dim3(256), 0, st, p);
        break;
    }
  }
  return check_launch("xn_index_select");
}

int xn_rvq_decode_sum(void *dst, const void *const *tables, int64_t n_q, const int64_t *codes,
                      int64_t batch, int64_t frames, int64_t dim, int64_t bins, int out_bct,
                      int dtype, int *err_flag, void *stream) {
  using namespace xn;
  if (!is_float_dtype(dtype)) return fail(XN_E_DTYPE, "xn_rvq_decode_sum: unsupported dtype %d", dtype);
  if (n_q <= 0 || n_q > XN_RVQ_MAX_CODEBOOKS)
    return fail(XN_E_INVALID, "xn_rvq_decode_sum: n_q=%lld outside [1, %d]", (long long)n_q, XN_RVQ_MAX_CODEBOOKS);
  if (batch < 0 || frames < 0 || dim < 0 || bins < 0) return fail(XN_E_INVALID, "xn_rvq_decode_sum: negative size");
  if (dim > 0x7fffffffLL) return fail(XN_E_INVALID, "xn_rvq_decode_sum: dim too large");
  if (batch * frames == 0 || dim == 0) return ok();
  if (dst == nullptr || codes == nullptr || tables == nullptr)
    return fail(XN_E_INVALID, "xn_rvq_decode_sum: null pointer");
  RvqParams p{};
  for (int64_t q = 0; q < n_q; ++q) {
    if (tables[q] == nullptr) return fail(XN_E_INVALID, "xn_rvq_decode_sum: codebook %lld is null", (long long)q);
    p.tab.p[q] = tables[q];
  }
  p.dst = dst;
  p.codes = codes;
  p.err = err_flag;
  p.batch = batch;
  p.frames = frames;
  p.dim = dim;
  p.bins = bins;
  p.nq = static_cast<int>(n_q);
  if (ceil_div(batch * frames, 8) > 0x7fffffffLL) return fail(XN_E_INVALID, "xn_rvq_decode_sum: too many frames");
  XN_DISPATCH_FLOAT(dtype, return launch_rvq<T>(p, out_bct, as_stream(stream)));
  return fail(XN_E_DTYPE, "xn_rvq_decode_sum: unsupported dtype %d", dtype);
}

}  // extern "C"
