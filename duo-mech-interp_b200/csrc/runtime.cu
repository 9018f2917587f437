// Error plumbing and device queries shared by every C entry point.
#include <cstdlib>
#include <atomic>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace duo {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

static std::atomic<unsigned long long> g_launches{0};

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("DUO_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int sm_count() {
  static int cached = 0;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (cached == 0) {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
      cached = n;
    else
      cached = 148;
  }
  return cached;
}

}  // namespace duo

extern "C" const char* duo_last_error(void) { return duo::g_last_error.c_str(); }

extern "C" int duo_abi_version(void) { return 1; }

extern "C" unsigned long long duo_launch_count(void) { return duo::g_launches.load(std::memory_order_relaxed); }
