// Library-level entry points: ABI version, status strings, per-thread last error.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"

namespace b2 {

static thread_local std::string g_last_error;

int fail(int status, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace b2

extern "C" {

int b2_abi_version(void) { return 1; }

const char* b2_status_name(int status) {
  switch (status) {
    case B2_OK: return "B2_OK";
    case B2_EINVAL: return "B2_EINVAL";
    case B2_ETIMEOUT: return "B2_ETIMEOUT";
    case B2_ECUDA: return "B2_ECUDA";
    case B2_ENOTSUP: return "B2_ENOTSUP";
    case B2_ERANGE: return "B2_ERANGE";
    default: return "B2_UNKNOWN";
  }
}

int b2_last_error(char* buf, size_t len) {
  if (!buf || len == 0) return B2_EINVAL;
  const std::string& e = b2::g_last_error;
  size_t n = e.size() < len - 1 ? e.size() : len - 1;
  memcpy(buf, e.data(), n);
  buf[n] = 0;
  return B2_OK;
}

}  // extern "C"
