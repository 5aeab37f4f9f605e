// Library-level entry points: version, thread-local error reporting, device info.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>

#include "common.cuh"

static thread_local char g_err[512] = {0};

int iron_set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

static std::atomic<long long> g_launches{0};

void iron_count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

// every kernel launch site of the library calls this right after its launch
int iron_check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return iron_set_error(IRON_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  iron_count_launch();
  return IRON_OK;
}

extern "C" int64_t iron_launch_count(void) { return (int64_t)g_launches.load(std::memory_order_relaxed); }

int iron_num_sms() {
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

extern "C" const char* iron_version(void) { return "iron_b200 0.1.0 (sm_100a)"; }

extern "C" int iron_last_error(char* buf, int buflen) {
  int n = (int)strlen(g_err);
  if (buf && buflen > 0) {
    int c = n < buflen - 1 ? n : buflen - 1;
    memcpy(buf, g_err, c);
    buf[c] = 0;
  }
  return n;
}
