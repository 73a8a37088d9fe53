// Library-level C ABI: version, error strings, device error word.
#include <stdarg.h>

#include <atomic>
#include <mutex>

#include "common.cuh"

namespace q3 {

static thread_local char g_last_error[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// The error word is a static device variable (one per device that loads the
// library, zero-initialised at module load); host code looks its address up
// once per device, so no entry point ever allocates device memory for it.
static __device__ int g_error_word = 0;

int* device_error_word() {
  static int* words[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!words[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_error_word) != cudaSuccess) return nullptr;
    words[dev] = static_cast<int*>(p);
  }
  return words[dev];
}

static std::atomic<uint64_t> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("Q3VL_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

}  // namespace q3

extern "C" int q3_version(void) { return 100; }

extern "C" uint64_t q3_launch_count(void) {
  return q3::g_launches.load(std::memory_order_relaxed);
}

extern "C" const char* q3_last_error(void) { return q3::g_last_error; }

extern "C" int q3_device_error(int clear) {
  int* w = q3::device_error_word();
  if (!w) return -1;
  int v = 0;
  if (cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  if (clear && v != 0) cudaMemset(w, 0, sizeof(int));
  return v;
}
