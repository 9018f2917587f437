// The fault word of the bounded-wait kernels, its host-visible mirror and the engine's gate on it.
//
// Every kernel that waits on an mbarrier (TMA loads, tcgen05 commits) bounds the wait to 2 s of %globaltimer.  A wait
// that gives up ORs a code into the device word g_tc_fault and the kernel unwinds instead of hanging the GPU.  Codes:
// 1 a producer waited for a free ring slot, 2 the MMA issuer waited for a filled slot, 4 the epilogue waited for the
// accumulator, 8 the persistent MMA issuer waited for a drained accumulator, 16 the conv prologue waited for a tile,
// 32 / 64 the tcgen05 chunked scan waited for its TMA tiles / its MMAs, 128 the tcgen05 attention prefill gave up a
// pipeline wait, 256 that kernel found its shared memory misaligned (it then does nothing).
//
// A give-up is not allowed to turn into a long stall.  Two mechanisms keep it short:
//   - device side: the tensor-core kernels that run without a cluster read the word when they start and, if it is
//     set, skip their work (after the programmatic-launch wait, so stream order holds).  One give-up therefore costs
//     one bounded wait, not one more 2 s give-up per later launch;
//   - host side: the engine's last kernel of every forward copies the word into a host-mapped word of the device
//     (plain stores to pinned memory, no atomics), and every engine call reads that word before it launches anything.
//     Once a fault is visible the engine refuses further work with DUO_ECUDA.  The host notices the fault within the
//     calls it had already queued; duo_fault_status synchronises, reads and clears both words.
#include <atomic>
#include <mutex>

#include "kernels.cuh"
#include "tc.cuh"

namespace duo {

__device__ unsigned g_tc_fault;

namespace {

constexpr int kMaxDev = 64;

struct FaultSlots {
  unsigned* dev = nullptr;          // device address of g_tc_fault on this device
  unsigned* mirror_host = nullptr;  // host-mapped word (host view)
  unsigned* mirror_dev = nullptr;   // the same word as the device addresses it
  bool dev_tried = false, mirror_tried = false;
};

std::mutex g_mu;
FaultSlots g_slots[kMaxDev];
std::atomic<unsigned> g_raised{0};  // set by duo_fault_raise (host only)

int current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) {
    cudaGetLastError();
    return -1;
  }
  return dev;
}

}  // namespace

unsigned* tc_fault_ptr() {
  const int dev = current_device();
  if (dev < 0) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  FaultSlots& s = g_slots[dev];
  if (!s.dev_tried) {
    s.dev_tried = true;
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_tc_fault) == cudaSuccess) s.dev = static_cast<unsigned*>(p);
    else cudaGetLastError();
  }
  return s.dev;
}

int fault_mirror_init() {
  const int dev = current_device();
  if (dev < 0) return fail(DUO_ECUDA, "fault word: no usable current CUDA device");
  std::lock_guard<std::mutex> lock(g_mu);
  FaultSlots& s = g_slots[dev];
  if (s.mirror_host) return DUO_OK;
  if (s.mirror_tried) return fail(DUO_ECUDA, "fault word: the host-mapped mirror could not be allocated");
  s.mirror_tried = true;
  void* h = nullptr;
  cudaError_t e = cudaHostAlloc(&h, 64, cudaHostAllocMapped | cudaHostAllocPortable);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(DUO_ENOMEM, std::string("fault word: cudaHostAlloc of the host-mapped mirror failed: ") +
                                cudaGetErrorString(e));
  }
  *static_cast<volatile unsigned*>(h) = 0u;
  void* d = nullptr;
  e = cudaHostGetDevicePointer(&d, h, 0);
  if (e != cudaSuccess) {
    cudaGetLastError();
    cudaFreeHost(h);
    return fail(DUO_ECUDA, std::string("fault word: cudaHostGetDevicePointer failed: ") + cudaGetErrorString(e));
  }
  s.mirror_host = static_cast<unsigned*>(h);
  s.mirror_dev = static_cast<unsigned*>(d);
  return DUO_OK;
}

unsigned* fault_mirror_dev() {
  const int dev = current_device();
  if (dev < 0) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  return g_slots[dev].mirror_dev;
}

int fault_gate(const char* where) {
  unsigned v = g_raised.load(std::memory_order_relaxed);
  const int dev = current_device();
  if (dev >= 0) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_slots[dev].mirror_host) v |= *static_cast<volatile unsigned*>(g_slots[dev].mirror_host);
  }
  if (v == 0) return DUO_OK;
  return fail(DUO_ECUDA, std::string(where) + ": a bounded wait inside an earlier kernel gave up (fault code " +
                             std::to_string(v) + "); nothing was launched.  duo_fault_status reads and clears it");
}

}  // namespace duo

using namespace duo;

extern "C" int duo_fault_status(unsigned* out) {
  DUO_CHECK_ARG(out, "fault_status: null pointer");
  unsigned v = g_raised.exchange(0u);
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {  // no device: only the host-side word exists
    cudaGetLastError();
    *out = v;
    return DUO_OK;
  }
  DUO_CUDA_TRY(cudaDeviceSynchronize());
  unsigned d = 0, zero = 0;
  DUO_CUDA_TRY(cudaMemcpyFromSymbol(&d, g_tc_fault, sizeof(d)));
  DUO_CUDA_TRY(cudaMemcpyToSymbol(g_tc_fault, &zero, sizeof(zero)));
  const int dev = current_device();
  if (dev >= 0) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_slots[dev].mirror_host) {
      volatile unsigned* h = g_slots[dev].mirror_host;
      d |= *h;
      *h = 0u;
    }
  }
  *out = v | d;
  return DUO_OK;
}

extern "C" int duo_fault_raise(unsigned code) {
  g_raised.fetch_or(code, std::memory_order_relaxed);
  return DUO_OK;
}
