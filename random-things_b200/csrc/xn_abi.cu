// xn_abi.cu - error reporting and small host utilities of the C ABI.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "xn_internal.h"

namespace {
thread_local char g_last_error[1024] = {0};
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};
}  // namespace

namespace xn {

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int ok() {
  g_last_error[0] = '\0';
  return XN_OK;
}

int check_launch(const char *op) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(XN_E_CUDA, "%s: kernel launch failed: %s", op, cudaGetErrorString(e));
  return ok();
}

int dtype_bytes(int dtype) {
  switch (dtype) {
    case XN_F16:
    case XN_BF16:
      return 2;
    case XN_F32:
      return 4;
    case XN_I64:
      return 8;
    case XN_U8:
      return 1;
    default:
      return 0;
  }
}

bool pdl_enabled() {
  static const bool enabled = [] {
    const char *v = std::getenv("XN_PDL");
    return !(v != nullptr && v[0] == '0');
  }();
  return enabled;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

}  // namespace xn

extern "C" {

const char *xn_last_error(void) { return g_last_error; }

int xn_abi_version(void) { return 1; }

int xn_shard_rows(int64_t rows, int world, int rank, int64_t *begin, int64_t *count) {
  if (!begin || !count) return xn::fail(XN_E_INVALID, "xn_shard_rows: null output pointer");
  if (rows < 0 || world <= 0 || rank < 0 || rank >= world)
    return xn::fail(XN_E_INVALID, "xn_shard_rows: bad arguments rows=%lld world=%d rank=%d",
                    (long long)rows, world, rank);
  const int64_t per = (rows + world - 1) / world;
  int64_t b = per * rank;
  if (b > rows) b = rows;
  int64_t e = b + per;
  if (e > rows) e = rows;
  *begin = b;
  *count = e - b;
  return xn::ok();
}

}  // extern "C"
