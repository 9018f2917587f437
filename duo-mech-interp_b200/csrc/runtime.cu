// Error plumbing and device queries shared by every C entry point.
#include <cstdlib>
#include <atomic>
#include <cstring>
#include <mutex>
#include <map>
#include <set>
#include <tuple>

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
void count_launches(long long delta) {
  g_launches.fetch_add(static_cast<unsigned long long>(delta), std::memory_order_relaxed);
}
unsigned long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("DUO_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int sm_count() {
  constexpr int kMaxDev = 64;
  static int cached[kMaxDev] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) {
    cudaGetLastError();
    return 148;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == 0) {
    int n = 0;
    cached[dev] = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0 ? n : 148;
  }
  return cached[dev];
}

int ensure_smem_attr_fn(const void* func, int bytes) {
  int dev = 0;
  DUO_CUDA_TRY(cudaGetDevice(&dev));
  static std::mutex mu;
  // the largest size set so far per (device, kernel): the attribute is a maximum, so it is only ever raised (a
  // kernel launched with several sizes would otherwise be left at a smaller one than a size recorded as done)
  static std::map<std::pair<int, const void*>, int> set_to;
  const auto key = std::make_pair(dev, func);
  std::lock_guard<std::mutex> lock(mu);
  const auto it = set_to.find(key);
  if (it != set_to.end() && it->second >= bytes) return DUO_OK;
  DUO_CUDA_TRY(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  set_to[key] = bytes;
  return DUO_OK;
}

}  // namespace duo

extern "C" const char* duo_last_error(void) { return duo::g_last_error.c_str(); }

extern "C" int duo_abi_version(void) { return 1; }

extern "C" unsigned long long duo_launch_count(void) { return duo::g_launches.load(std::memory_order_relaxed); }
