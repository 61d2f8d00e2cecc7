// C++ port of the reference's CUDA known-answer tests for the fused-op path
// (mimi-rs/tests/cuda_tests.rs), written against the C++ Backend mirror
// (random-things_b200/host/xn_backend.hpp) so they read like the originals.
// Each test returns normally or throws; main() prints one line per test and
// exits non-zero if any failed. Built and run by tests/test_cpp_backend.py.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <functional>
#include <string>
#include <vector>

#include "xn_backend.hpp"

using xn::CudaDevice;
using xn::Storage;

namespace {

struct Failure : std::runtime_error {
  using std::runtime_error::runtime_error;
};

#define CHECK(cond)                                                                        \
  do {                                                                                     \
    if (!(cond)) throw Failure(std::string(__FILE__) + ":" + std::to_string(__LINE__) + ": " #cond); \
  } while (0)

template <typename T>
struct DeviceVec {
  Storage<T> s;
  explicit DeviceVec(const std::vector<T> &host) {
    s.len = host.size();
    if (cudaMalloc(&s.data, std::max<size_t>(1, host.size()) * sizeof(T)) != cudaSuccess) throw Failure("cudaMalloc");
    if (!host.empty()) cudaMemcpy(s.data, host.data(), host.size() * sizeof(T), cudaMemcpyHostToDevice);
  }
  explicit DeviceVec(size_t n) : DeviceVec(std::vector<T>(n)) {}
  ~DeviceVec() { cudaFree(s.data); }
  std::vector<T> to_vec() const {
    std::vector<T> h(s.len);
    cudaDeviceSynchronize();
    if (!h.empty()) cudaMemcpy(h.data(), s.data, s.len * sizeof(T), cudaMemcpyDeviceToHost);
    return h;
  }
};

// cuda_tests.rs:146-156
void test_silu(const CudaDevice &dev) {
  DeviceVec<float> x({0.0f, 1.0f, -1.0f}), y(3);
  dev.unary(y.s, x.s, 3, xn::UnaryOp::Silu);
  auto v = y.to_vec();
  CHECK(std::fabs(v[0] - 0.0f) < 1e-5f);
  CHECK(std::fabs(v[1] - 0.7310586f) < 1e-5f);
  CHECK(std::fabs(v[2] - (-0.26894143f)) < 1e-5f);
}

// cuda_tests.rs:323-342
void test_softmax(const CudaDevice &dev) {
  DeviceVec<float> x({1, 2, 3, 1, 2, 3}), y(6);
  dev.softmax(y.s, x.s, 3, 2);
  auto v = y.to_vec();
  CHECK(std::fabs(v[0] + v[1] + v[2] - 1.0f) < 1e-5f);
  CHECK(std::fabs(v[3] + v[4] + v[5] - 1.0f) < 1e-5f);
  CHECK(std::fabs(v[0] - 0.0900306f) < 1e-4f);
  CHECK(std::fabs(v[1] - 0.2447285f) < 1e-4f);
  CHECK(std::fabs(v[2] - 0.6652409f) < 1e-4f);
}

// cuda_tests.rs:344-355
void test_softmax_single_row(const CudaDevice &dev) {
  DeviceVec<float> x({0, 0, 0}), y(3);
  dev.softmax(y.s, x.s, 3, 1);
  for (float v : y.to_vec()) CHECK(std::fabs(v - 1.0f / 3.0f) < 1e-5f);
}

// cuda_tests.rs:361-384
void test_rms_norm(const CudaDevice &dev) {
  DeviceVec<float> x({1, 2, 3, 4, 5, 6}), alpha({1, 1, 1}), y(6);
  dev.rms_norm(y.s, x.s, alpha.s, 3, 2, 1e-5f);
  auto v = y.to_vec();
  const float s1 = 1.0f / std::sqrt((1.0f + 4.0f + 9.0f) / 3.0f + 1e-5f);
  const float s2 = 1.0f / std::sqrt((16.0f + 25.0f + 36.0f) / 3.0f + 1e-5f);
  for (int i = 0; i < 3; ++i) CHECK(std::fabs(v[i] - (i + 1) * s1) < 1e-4f);
  for (int i = 0; i < 3; ++i) CHECK(std::fabs(v[3 + i] - (i + 4) * s2) < 1e-4f);
}

// cuda_tests.rs:386-401
void test_rms_norm_with_scale(const CudaDevice &dev) {
  DeviceVec<float> x({1, 2, 3}), alpha({2, 2, 2}), y(3);
  dev.rms_norm(y.s, x.s, alpha.s, 3, 1, 1e-5f);
  auto v = y.to_vec();
  const float s = 1.0f / std::sqrt((1.0f + 4.0f + 9.0f) / 3.0f + 1e-5f);
  for (int i = 0; i < 3; ++i) CHECK(std::fabs(v[i] - (i + 1) * s * 2.0f) < 1e-4f);
}

// cuda_tests.rs:407-433
void test_layer_norm(const CudaDevice &dev) {
  DeviceVec<float> x({1, 2, 3, 4, 5, 6}), w({1, 1, 1}), b({0, 0, 0}), y(6);
  dev.layer_norm(y.s, x.s, w.s, b.s, 3, 2, 1e-5f, true);
  auto v = y.to_vec();
  const float inv = 1.0f / std::sqrt(2.0f / 3.0f + 1e-5f);
  for (int i = 0; i < 3; ++i) CHECK(std::fabs(v[i] - (i - 1) * inv) < 1e-4f);
  for (int i = 0; i < 3; ++i) CHECK(std::fabs(v[3 + i] - (i - 1) * inv) < 1e-4f);
}

// cuda_tests.rs:435-452
void test_layer_norm_with_affine(const CudaDevice &dev) {
  DeviceVec<float> x({1, 2, 3}), w({2, 2, 2}), b({1, 1, 1}), y(3);
  dev.layer_norm(y.s, x.s, w.s, b.s, 3, 1, 1e-5f, true);
  auto v = y.to_vec();
  const float inv = 1.0f / std::sqrt(2.0f / 3.0f + 1e-5f);
  for (int i = 0; i < 3; ++i) CHECK(std::fabs(v[i] - ((i - 1) * inv * 2.0f + 1.0f)) < 1e-4f);
}

// cuda_tests.rs:611-626 and :628-643 (index_select along dim 0 and dim 1)
void test_index_select(const CudaDevice &dev) {
  std::vector<float> data;
  for (int i = 1; i <= 12; ++i) data.push_back((float)i);
  DeviceVec<float> a(data), out0(9), out1(6);
  DeviceVec<uint32_t> ids(8);
  std::vector<uint32_t> ids0 = {0, 2, 3};
  dev.index_select(out0.s, a.s, ids0, ids.s, 0, {4, 3});
  CHECK((out0.to_vec() == std::vector<float>{1, 2, 3, 7, 8, 9, 10, 11, 12}));
  std::vector<uint32_t> ids1 = {1, 3};
  dev.index_select(out1.s, a.s, ids1, ids.s, 1, {3, 4});
  CHECK((out1.to_vec() == std::vector<float>{2, 4, 6, 8, 10, 12}));
  bool threw = false;
  try {
    std::vector<uint32_t> bad = {0, 4};
    dev.index_select(out1.s, a.s, bad, ids.s, 0, {4, 3});
  } catch (const xn::Error &e) {
    threw = std::string(e.what()).find("out of bounds") != std::string::npos;
  }
  CHECK(threw);
}

// cuda_tests.rs:756-790 and :792-818
void test_apply_causality_mask(const CudaDevice &dev) {
  DeviceVec<float> a(std::vector<float>(12, 1.0f));
  dev.apply_causality_mask(a.s, 1, 3, 4, 0);
  auto r = a.to_vec();
  const bool masked[12] = {0, 1, 1, 1, 0, 0, 1, 1, 0, 0, 0, 1};
  for (int i = 0; i < 12; ++i) CHECK(masked[i] ? (std::isinf(r[i]) && r[i] < 0) : r[i] == 1.0f);
  DeviceVec<float> b(std::vector<float>(8, 1.0f));
  dev.apply_causality_mask(b.s, 1, 2, 4, 2);
  auto rb = b.to_vec();
  for (int i = 0; i < 8; ++i) CHECK(i == 3 ? (std::isinf(rb[i]) && rb[i] < 0) : rb[i] == 1.0f);
}

// cuda_tests.rs:1109-1173
void test_rope_position_offset(const CudaDevice &dev) {
  DeviceVec<float> x({1, 2, 3, 4}), y(4);
  DeviceVec<float> cos({1, 1, 0, 0, -1, -1, 0, 0, 1, 1, 0.5f, 0.5f, 0, 0, 0, 0, 0, 0, 0, 0});
  DeviceVec<float> sin({0, 0, 1, 1, 0, 0, 0, 0, 0, 0, 0.866f, 0.866f, 0, 0, 0, 0, 0, 0, 0, 0});
  dev.rope(y.s, x.s, cos.s, sin.s, 1, 1, 1, 4, 0);
  auto y0 = y.to_vec();
  for (int i = 0; i < 4; ++i) CHECK(std::fabs(y0[i] - (i + 1)) < 1e-5f);
  dev.rope(y.s, x.s, cos.s, sin.s, 1, 1, 1, 4, 1);
  auto y1 = y.to_vec();
  CHECK(!(std::fabs(y1[0] - 1.0f) < 1e-5f && std::fabs(y1[1] - 2.0f) < 1e-5f));
  const float expect[4] = {-3, -4, 1, 2};
  for (int i = 0; i < 4; ++i) CHECK(std::fabs(y1[i] - expect[i]) < 1e-5f);
  bool threw = false;
  try {
    dev.rope(y.s, x.s, cos.s, sin.s, 1, 1, 1, 4, 10);  // pos + t > max_pos
  } catch (const xn::Error &e) {
    threw = e.code == XN_E_RANGE;
  }
  CHECK(threw);
}

// cuda_tests.rs:1059-1107 (rope with identity tables keeps the values)
void test_rope_identity(const CudaDevice &dev) {
  std::vector<float> k(1280);
  for (int i = 0; i < 1280; ++i) k[i] = i / 100.0f;
  DeviceVec<float> x(k), y(1280), cos(std::vector<float>(320, 1.0f)), sin(std::vector<float>(320, 0.0f));
  dev.rope(y.s, x.s, cos.s, sin.s, 1, 4, 5, 64, 0);
  auto v = y.to_vec();
  for (int i = 0; i < 1280; ++i) CHECK(std::fabs(v[i] - k[i]) < 1e-5f);
}

// Streaming decode on the ring cache (mimi.rs:1317-1384 op sequence): with
// identity RoPE tables and a zero query every visible key scores 0, so each
// step's output is the mean of the visible value rows. Values of step s are
// all s + 1; context 2 keeps the last two positions.
void test_decode_attention_mean_of_visible_values(const CudaDevice &dev) {
  const size_t b = 1, h = 1, d = 32, cap = 2, context = 2, steps = 4;
  for (int fused = 0; fused < 2; ++fused) {
    DeviceVec<float> k(b * h * cap * d), v(b * h * cap * d);
    xn::RingKvCache<float> cache;
    cache.k = k.s;
    cache.v = v.s;
    cache.b = b, cache.h = h, cache.cap = cap, cache.d = d;
    DeviceVec<float> cos(std::vector<float>(8 * d / 2, 1.0f)), sin(std::vector<float>(8 * d / 2, 0.0f));
    DeviceVec<float> q(b * h * d), out(b * h * d);
    const float expect[steps] = {1.0f, 1.5f, 2.5f, 3.5f};
    for (size_t s = 0; s < steps; ++s) {
      std::vector<float> qkv(3 * d, 0.0f);
      for (size_t i = 0; i < d; ++i) {
        qkv[d + i] = 0.25f * i;               // k (scores stay 0: q = 0)
        qkv[2 * d + i] = static_cast<float>(s + 1);  // v
      }
      DeviceVec<float> qkv_d(qkv);
      if (fused) {
        dev.decode_attention_step(out.s, cache, qkv_d.s, cos.s, sin.s, 1, context, 0.125f, xn::DecodeMask::Relative,
                                  true);
      } else {
        dev.kv_append_rope(q.s, cache, qkv_d.s, cos.s, sin.s, 1, true);
        dev.attention_decode(out.s, q.s, cache, 1, context, 0.125f, xn::DecodeMask::Relative);
      }
      auto o = out.to_vec();
      for (size_t i = 0; i < d; ++i) CHECK(std::fabs(o[i] - expect[s]) < 1e-6f);
    }
    CHECK(cache.total == steps);
    bool threw = false;
    DeviceVec<float> qkv_last(3 * d);
    try {
      cache.total = 8;  // past the 8 rows of the tables
      dev.decode_attention_step(out.s, cache, qkv_last.s, cos.s, sin.s, 1, context, 0.125f, xn::DecodeMask::Relative,
                                true);
    } catch (const xn::Error &e) {
      threw = e.code == XN_E_RANGE;
    }
    CHECK(threw);
  }
}

}  // namespace

int main() {
  CudaDevice dev;
  const std::vector<std::pair<const char *, std::function<void(const CudaDevice &)>>> tests = {
      {"test_silu", test_silu},
      {"test_softmax", test_softmax},
      {"test_softmax_single_row", test_softmax_single_row},
      {"test_rms_norm", test_rms_norm},
      {"test_rms_norm_with_scale", test_rms_norm_with_scale},
      {"test_layer_norm", test_layer_norm},
      {"test_layer_norm_with_affine", test_layer_norm_with_affine},
      {"test_index_select", test_index_select},
      {"test_apply_causality_mask", test_apply_causality_mask},
      {"test_rope_position_offset", test_rope_position_offset},
      {"test_rope_identity", test_rope_identity},
      {"test_decode_attention_mean_of_visible_values", test_decode_attention_mean_of_visible_values},
  };
  int failed = 0;
  for (const auto &t : tests) {
    try {
      t.second(dev);
      std::printf("PASS %s\n", t.first);
    } catch (const std::exception &e) {
      ++failed;
      std::printf("FAIL %s: %s\n", t.first, e.what());
    }
  }
  std::printf("%d failed of %zu\n", failed, tests.size());
  return failed == 0 ? 0 : 1;
}
