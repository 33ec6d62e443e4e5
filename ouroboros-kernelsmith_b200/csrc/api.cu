// Library-wide host helpers: error reporting, device attributes, version.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"
#include "tma.cuh"

namespace b2k {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

// Streaming multiprocessors of the current device (148 on B200), cached per
// device ordinal.
int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    return B2K_ELAUNCH;
  }
  return B2K_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static TimeoutReader g_readers[64];
static int g_nreaders = 0;

void register_timeout_reader(TimeoutReader f) {
  if (g_nreaders < 64) g_readers[g_nreaders++] = f;
}

int dtype_size(int dtype) {
  switch (dtype) {
    case B2K_F32: return 4;
    case B2K_F16: return 2;
    case B2K_BF16: return 2;
    case B2K_I8: return 1;
    case B2K_I64: return 8;
    default: return 0;
  }
}

}  // namespace b2k

extern "C" int b2k_version(void) { return 100; }  // 0.1.0

extern "C" const char* b2k_last_error(void) { return b2k::g_err; }

extern "C" unsigned b2k_pipeline_timeouts(int reset) {
  unsigned total = 0;
  for (int i = 0; i < b2k::g_nreaders; ++i) total += b2k::g_readers[i](reset != 0);
  return total;
}
