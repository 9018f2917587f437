// duo_attention_noalloc: the attention entry point for callers that must not allocate device memory.
//
// duo_attention keeps its split-K decode partials in a workspace that the library allocates with cudaMalloc the
// first time a call needs it (and grows later).  Some callers cannot accept that: a serving stack whose pooled
// allocator owns every byte of device memory, or a latency-critical decode loop in which an allocation (and the
// device-wide synchronisation that cudaMalloc implies) is not allowed.  This entry point runs the same kernels with the
// same split plan, but its scratch is one file-scope device array of fixed size, so a call allocates nothing.
//
// Limits and rules of use:
//   - the array holds kScratchFloats = 262,144 floats (1 MiB).  A decode call (t == 1) needs
//     b * nh * splits * (hd + 2) floats, with the split count chosen as duo_attention chooses it; a call that needs
//     more is rejected with DUO_EINVAL before anything is launched.  Prefill calls (t > 1) use no scratch;
//   - every GPU that loads the library holds the array until the process exits;
//   - the first call on a device looks up the array's device address (cudaGetSymbolAddress) with that device
//     current, and caches it; make that first call before any stream capture;
//   - all calls share the one array and it keeps the last call's contents.  Nothing in it needs to start at zero:
//     the decode kernel writes every partial it later reads.  Calls whose work overlaps on the GPU (two streams, or
//     two threads) race on the array: order them on one stream.
#include <mutex>

#include "kernels.cuh"

namespace duo {
namespace {

constexpr long kScratchFloats = 1L << 18;
static __device__ __align__(256) float g_attn_scratch[kScratchFloats];

// Device address of g_attn_scratch for the current device (looked up once per device); null and a status on error.
float* scratch_on_current_device(int* status) {
  static std::mutex mu;
  static float* addr[64] = {};
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    *status = fail(DUO_ECUDA, "attention_noalloc: no usable current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess || !p) {
      *status = fail(DUO_ECUDA, std::string("attention_noalloc: cudaGetSymbolAddress of the static scratch failed: ") +
                                    cudaGetErrorString(e));
      return nullptr;
    }
    addr[dev] = static_cast<float*>(p);
  }
  *status = DUO_OK;
  return addr[dev];
}

}  // namespace
}  // namespace duo

using namespace duo;

extern "C" int duo_attention_noalloc(const void* q, const void* kc, const void* vc, const int32_t* start,
                                     const void* gate, int gate_stride, void* o, int dtype, int b, int t, int nh,
                                     int nkv, int hd, int max_len, float scale, duo_stream stream) {
  DUO_CHECK_ARG(b >= 0 && t >= 0 && nh > 0 && nkv > 0 && max_len > 0, "attention_noalloc: bad shape");
  DUO_CHECK_ARG(valid_act(dtype), "attention_noalloc: dtype must be f32, bf16 or f16");
  DUO_CHECK_ARG(b == 0 || t == 0 || (q && kc && vc && start && o), "attention_noalloc: null pointer");
  AttnArgs a{};
  a.q = q; a.kc = kc; a.vc = vc; a.cache_row0 = 0; a.start = start; a.len = nullptr;
  a.gate = gate; a.gate_stride = gate_stride; a.gate_hstride = hd; a.o = o;
  a.b = b; a.t = t; a.nh = nh; a.nkv = nkv; a.hd = hd; a.max_len = max_len; a.scale = scale;
  if (t == 1 && b > 0) {
    const long need = attn_decode_scratch_floats(b, nh, nkv, max_len, dtype);
    if (need > kScratchFloats)
      return fail(DUO_EINVAL, "attention_noalloc: this decode call needs " + std::to_string(need) +
                                  " floats of split-K scratch (b * nh * splits * (hd + 2)) but the static array holds " +
                                  std::to_string(kScratchFloats) + "; use duo_attention or split the batch");
    if (need > 0) {
      int status = DUO_OK;
      a.work = scratch_on_current_device(&status);
      if (!a.work) return status;
      a.work_floats = kScratchFloats;
    }
  }
  return launch_attention(a, dtype, as_stream(stream));
}
