// Shared helpers for the duo mixer kernels (sm_100a only).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string>
#include <type_traits>
#include <utility>

#include "../../include/duo_mixer.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ != 1000)
#error "duo mixer kernels are written for sm_100a only"
#endif

namespace duo {

// ---------------------------------------------------------------------------------------------------------------
// host-side error plumbing: every C entry point returns a duo status and records a message for duo_last_error()

void set_error(const std::string& msg);
int fail(int code, const std::string& msg);

#define DUO_CHECK_ARG(cond, msg)                                    \
  do {                                                              \
    if (!(cond)) return ::duo::fail(DUO_EINVAL, std::string(msg));  \
  } while (0)

#define DUO_CUDA_TRY(expr)                                                                                \
  do {                                                                                                    \
    cudaError_t _e = (expr);                                                                              \
    if (_e != cudaSuccess)                                                                                \
      return ::duo::fail(DUO_ECUDA, std::string(#expr) + ": " + cudaGetErrorString(_e));                 \
  } while (0)

// after every kernel launch: count it (duo_launch_count) and turn a launch error into a status
#define DUO_LAUNCH_CHECK(what)                                                                             \
  do {                                                                                                    \
    ::duo::count_launch();                                                                                \
    cudaError_t _e = cudaGetLastError();                                                                  \
    if (_e != cudaSuccess) return ::duo::fail(DUO_ECUDA, std::string(what) + ": " + cudaGetErrorString(_e)); \
  } while (0)

void count_launch();
// launches executed by graph replays: the capture counted one step's kernels, each replay runs them again
void count_launches(long long delta);
unsigned long long launch_count();

// ---------------------------------------------------------------------------------------------------------------
// Programmatic dependent launch.  Kernels are launched with programmatic stream serialisation, so the CTAs of a kernel
// may become resident while its predecessor in the stream is still running.  Every kernel calls pdl_wait()
// (griddepcontrol.wait: returns once the preceding grid has completed and its writes are visible) before its first
// access to memory that another kernel writes or reads, and only after that pdl_trigger()
// (griddepcontrol.launch_dependents), which lets the successor's CTAs launch and run their prologue meanwhile.
// Because no kernel triggers before its own wait, a kernel that starts early overlaps only its immediate predecessor:
// every earlier kernel has completed.  A prologue may therefore read data that the immediate predecessor does not
// write (the GEMMs prefetch constant weight tiles).  A grid launched without the attribute passes both at once.
// DUO_PDL=0 in the environment launches without the attribute.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                          Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}


#define DUO_TRY(expr)              \
  do {                             \
    int _s = (expr);               \
    if (_s != DUO_OK) return _s;   \
  } while (0)

inline cudaStream_t as_stream(duo_stream s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool valid_act(int dt) { return dt == DUO_F32 || dt == DUO_BF16 || dt == DUO_F16; }
inline size_t act_bytes(int dt) { return dt == DUO_F32 ? 4 : 2; }

inline int cdiv(long a, long b) { return (int)((a + b - 1) / b); }

// Run f(tag) with tag a value of the C++ type of activation dtype `dt` (float, __nv_bfloat16 or __half):
//   with_act(dt, [&](auto tag) { using T = decltype(tag); ... });
template <typename F> int with_act(int dt, F&& f) {
  switch (dt) {
    case DUO_F32: return f(float{});
    case DUO_BF16: return f(__nv_bfloat16{});
    case DUO_F16: return f(__half{});
    default: return fail(DUO_EINVAL, "unsupported activation dtype " + std::to_string(dt));
  }
}

// number of SMs of the current device (looked up once per device)
int sm_count();

// cudaFuncAttributeMaxDynamicSharedMemorySize = bytes for `func` on the current device, set once per (device, func)
int ensure_smem_attr_fn(const void* func, int bytes);
template <typename K> int ensure_smem_attr(K* kernel, int bytes) {
  return ensure_smem_attr_fn(reinterpret_cast<const void*>(kernel), bytes);
}

// ---------------------------------------------------------------------------------------------------------------
// device helpers

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// load 8 consecutive values of T as floats (16-byte aligned for bf16, 32 for f32)
__device__ __forceinline__ void load8(const float* p, float* o) {
  float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* o) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    float2 f = __bfloat1622float2(h[i]);
    o[2 * i] = f.x; o[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load8(const __half* p, float* o) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    float2 f = __half22float2(h[i]);
    o[2 * i] = f.x; o[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void store8(__half* p, const float* v) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; i++) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ void store8(float* p, const float* v) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* v) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; i++) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// block-wide sum for blockDim.x a multiple of 32, <= 1024; `red` needs 32 floats of shared memory
__device__ __forceinline__ float block_sum(float v, float* red) {
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  return warp_sum(t);
}

// 16-byte global -> shared copy through L2 only (cp.async.cg); an invalid source zero-fills the 16 bytes
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid = true) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// wait until at most N of this thread's committed groups are still in flight
template <int N> __device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// the common prologue: wait for the predecessor, then let the successor launch
__device__ __forceinline__ void pdl_enter() {
  pdl_wait();
  pdl_trigger();
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }
__device__ __forceinline__ float siluf_(float x) { return x / (1.f + expf(-x)); }
// SiLU on the hardware exponential and the approximate divide (a few ulp; x -> -inf gives -0), for the SwiGLU
// epilogues of the 16-bit GEMMs, whose result is rounded to bf16 / f16 right after
__device__ __forceinline__ float silu16_(float x) { return __fdividef(x, 1.f + __expf(-x)); }
// SiLU for a result stored as T: the fast form when T is 16-bit, the accurate one for f32 (the f32 engine)
template <typename T> __device__ __forceinline__ float silu_t(float x) {
  if constexpr (sizeof(T) == 2) return silu16_(x);
  else return siluf_(x);
}
// SiLU as x sigmoid(x) = x (1 + tanh(x / 2)) / 2 on one hardware tanh (tanh.approx.f32, about 2^-11 relative error,
// one special-function op where silu16_ takes two): for values rounded to bf16 right after
__device__ __forceinline__ float silu_tanh(float x) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * x));
  return 0.5f * x * (1.f + t);
}
// the bf16 engine's SiLU where the special-function pipe bounds the kernel; f16 and f32 keep silu_t
template <typename T> __device__ __forceinline__ float silu_bf(float x) {
  if constexpr (sizeof(T) == 2 && !std::is_same<T, __half>::value) return silu_tanh(x);
  else return silu_t<T>(x);
}
// torch's softplus (beta 1, threshold 20) and the reference WGSL's (kernels_qwen35.js:11)
__device__ __forceinline__ float softplusf_(float x) { return x > 20.f ? x : log1pf(expf(x)); }

// int8 -> f32 for four packed bytes without the I2F pipe: bias each byte to unsigned, place it in the mantissa of
// 2^23, subtract 2^23 + 128.  Exact for every int8 value.
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float* o) {
  uint32_t u = w ^ 0x80808080u;
  const float bias = 8388736.f;  // 2^23 + 128
  o[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - bias;
  o[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - bias;
  o[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - bias;
  o[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - bias;
}

}  // namespace duo
