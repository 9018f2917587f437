// Row-wise and elementwise kernels of the forward: RMSNorm, SwiGLU with the neuron-push hook, the residual vector
// add, per-row argmax, and the small bookkeeping kernels (last-token copy, row lengths).
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "tc.cuh"

namespace duo {

// ---------------------------------------------------------------------------------------------------------------
// RMSNorm (engine/kernels.js:226-246): one block per row, 8 values per thread per step

template <typename TY>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* __restrict__ x, int d, const float* __restrict__ w,
                                                      float eps, int offset, TY* __restrict__ y) {
  pdl_enter();
  __shared__ float red[32];
  const float* xr = x + (long)blockIdx.x * d;
  float ss = 0.f;
  for (int c = threadIdx.x * 8; c < d; c += blockDim.x * 8) {
    float v[8];
    load8(xr + c, v);
#pragma unroll
    for (int j = 0; j < 8; j++) ss = fmaf(v[j], v[j], ss);
  }
  const float r = rsqrtf(block_sum(ss, red) / (float)d + eps);
  TY* yr = y + (long)blockIdx.x * d;
  for (int c = threadIdx.x * 8; c < d; c += blockDim.x * 8) {
    float v[8], g[8];
    load8(xr + c, v);
    load8(w + c, g);
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = v[j] * r * (offset ? 1.f + g[j] : g[j]);
    store8(yr + c, v);
  }
}

int launch_rmsnorm(const float* x, int m, int d, const float* w, float eps, int offset, void* y, int y_dtype,
                   cudaStream_t st) {
  if (m == 0) return DUO_OK;
  const int threads = std::min(256, std::max(32, ((d / 8 + 31) / 32) * 32));
  return with_act(y_dtype, [&](auto yt) -> int {
    using TY = decltype(yt);
    DUO_CUDA_TRY(::duo::launch_kernel(rmsnorm_kernel<TY>, m, threads, 0, st, x, d, w, eps, offset, static_cast<TY*>(y)));
    DUO_LAUNCH_CHECK("rmsnorm_kernel");
    return DUO_OK;
  });
}

// ---------------------------------------------------------------------------------------------------------------
// SwiGLU + neuron pushes (engine/kernels_qwen35.js:254-279): a = silu(gate) * up from gu[M, 2I] = [gate | up], then
// the layer's push records in order: neuron n (or every neuron), add or multiply a per-row value.

template <typename T>
__global__ void __launch_bounds__(256) swiglu_push_kernel(const T* __restrict__ gu, int inter, int t, int row_base,
                                                          PushTable pt, T* __restrict__ a) {
  pdl_enter();
  const int m = blockIdx.y;
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c0 >= inter) return;
  const T* gr = gu + (long)m * 2 * inter;
  float g[8], u[8], v[8];
  load8(gr + c0, g);
  load8(gr + inter + c0, u);
#pragma unroll
  for (int j = 0; j < 8; j++) v[j] = silu_t<T>(g[j]) * u[j];
  const int r = row_base + m / t;
  for (int i = 0; i < pt.count; i++) {
    const int n = pt.neuron[i];
    const float val = pt.vals[(long)i * pt.rows + r];
    const bool mul = pt.mode[i] == DUO_PUSH_MUL;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      if (n == DUO_ALL_NEURONS || n == c0 + j) v[j] = mul ? v[j] * val : v[j] + val;
    }
  }
  store8(a + (long)m * inter + c0, v);
}

int launch_swiglu_push(const void* gu, int m, int inter, int t, int row_base, const PushTable& pt, void* a,
                       int dtype, cudaStream_t st) {
  if (m == 0) return DUO_OK;
  dim3 grid(cdiv(inter / 8, 256), m);
  return with_act(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    DUO_CUDA_TRY(::duo::launch_kernel(swiglu_push_kernel<T>, grid, 256, 0, st, static_cast<const T*>(gu), inter, t, row_base, pt, static_cast<T*>(a)));
    DUO_LAUNCH_CHECK("swiglu_push_kernel");
    return DUO_OK;
  });
}

// ---------------------------------------------------------------------------------------------------------------
// residual vector add (engine/kernels.js:190-203): x[m, :] += vec[row_base + m / t, :]

__global__ void vec_add_kernel(float* __restrict__ x, int h, int t, int row_base, const float* __restrict__ vec) {
  pdl_enter();
  const int m = blockIdx.y;
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (c >= h) return;
  const int r = row_base + m / t;
  float4* xp = reinterpret_cast<float4*>(x + (long)m * h + c);
  const float4 v = *reinterpret_cast<const float4*>(vec + (long)r * h + c);
  float4 o = *xp;
  o.x += v.x; o.y += v.y; o.z += v.z; o.w += v.w;
  *xp = o;
}

int launch_vec_add(float* x, int m, int h, int t, int row_base, const float* vec, cudaStream_t st) {
  if (m == 0) return DUO_OK;
  DUO_CUDA_TRY(::duo::launch_kernel(vec_add_kernel, dim3(cdiv(h / 4, 256), m), 256, 0, st, x, h, t, row_base, vec));
  DUO_LAUNCH_CHECK("vec_add_kernel");
  return DUO_OK;
}

// ---------------------------------------------------------------------------------------------------------------
// per-row argmax over the vocabulary (engine/kernels.js:261-284): ties go to the lower index

__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ logits, int v, int32_t* __restrict__ out) {
  pdl_enter();
  const float* row = logits + (long)blockIdx.x * v;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = threadIdx.x; i < v; i += blockDim.x) {
    const float x = row[i];
    if (x > best) { best = x; idx = i; }  // ascending i per thread: the first maximum is kept
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) { sb[w] = best; si[w] = idx; }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sb[lane] : -INFINITY;
    idx = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
    }
    if (lane == 0) out[blockIdx.x] = idx == 0x7fffffff ? 0 : idx;
  }
}

int launch_argmax(const float* logits, int m, int v, int32_t* out, cudaStream_t st) {
  if (m == 0) return DUO_OK;
  DUO_CUDA_TRY(::duo::launch_kernel(argmax_kernel, m, 1024, 0, st, logits, v, out));
  DUO_LAUNCH_CHECK("argmax_kernel");
  return DUO_OK;
}

// ---------------------------------------------------------------------------------------------------------------
// bookkeeping: last token of each row -> last[row], row lengths += t

// The last kernel of a forward also copies the fault word of the bounded-wait kernels into its host-mapped mirror
// (plain stores to pinned memory), where the engine's next call sees it without synchronising.
__global__ void copy_last_kernel(const float* __restrict__ x, int h, int t, int row_base, float* __restrict__ last,
                                 const unsigned* fault, unsigned* mirror) {
  pdl_enter();
  if (blockIdx.x == 0 && threadIdx.x == 0 && fault && mirror) {
    const unsigned f = *reinterpret_cast<const volatile unsigned*>(fault);
    if (f) *reinterpret_cast<volatile unsigned*>(mirror) = f;
  }
  const int r = blockIdx.x;
  const float* src = x + ((long)r * t + t - 1) * h;
  float* dst = last + (long)(row_base + r) * h;
  for (int c = threadIdx.x * 4; c < h; c += blockDim.x * 4)
    *reinterpret_cast<float4*>(dst + c) = *reinterpret_cast<const float4*>(src + c);
}

__global__ void advance_len_kernel(int32_t* len, int row_base, int rows, int t) {
  pdl_enter();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < rows) len[row_base + i] += t;
}

int launch_finish_rows(const float* x, int h, int t, int row_base, int rows, float* last, int32_t* len,
                       cudaStream_t st) {
  if (rows == 0) return DUO_OK;
  const unsigned* fault = tc_fault_ptr();
  unsigned* mirror = fault_mirror_dev();
  DUO_CUDA_TRY(::duo::launch_kernel(copy_last_kernel, rows, 256, 0, st, x, h, t, row_base, last, fault, mirror));
  DUO_LAUNCH_CHECK("copy_last_kernel");
  DUO_CUDA_TRY(::duo::launch_kernel(advance_len_kernel, cdiv(rows, 256), 256, 0, st, len, row_base, rows, t));
  DUO_LAUNCH_CHECK("advance_len_kernel");
  return DUO_OK;
}

// ids for the next decode step from the argmax of the previous one, and the token log
// One block: the step index is the host's `step`, or (step_ctr != nullptr, a graph-replayed step) read from the
// device counter, which the block advances once every thread has read it.
__global__ void feed_tokens_kernel(const int32_t* __restrict__ am, int rows, int32_t* __restrict__ ids,
                                   int32_t* __restrict__ log, int n_steps, int step, int32_t* step_ctr) {
  pdl_enter();
  if (step_ctr) step = *step_ctr;
  __syncthreads();
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    const int tok = am[r];
    ids[r] = tok;
    if (step < n_steps) log[(long)r * n_steps + step] = tok;
  }
  __syncthreads();
  if (step_ctr && threadIdx.x == 0) *step_ctr = step + 1;
}

int launch_feed_tokens(const int32_t* am, int rows, int32_t* ids, int32_t* log, int n_steps, int step,
                       int32_t* step_ctr, cudaStream_t st) {
  DUO_CUDA_TRY(::duo::launch_kernel(feed_tokens_kernel, 1, 256, 0, st, am, rows, ids, log, n_steps, step, step_ctr));
  DUO_LAUNCH_CHECK("feed_tokens_kernel");
  return DUO_OK;
}

// 16-bit -> f32 copy (the capture hooks of the 16-bit engines), 8 values per thread
template <typename T>
__global__ void to_f32_kernel(const T* __restrict__ src, long n8, float* __restrict__ dst) {
  pdl_enter();
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    float v[8];
    load8(src + 8 * i, v);
    store8(dst + 8 * i, v);
  }
}

int launch_to_f32(const void* src, int dtype, long n, float* dst, cudaStream_t st) {
  if (n == 0) return DUO_OK;
  if (n % 8 || (reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(dst) & 31))
    return fail(DUO_EINVAL, "to_f32: n must be a multiple of 8 and the buffers 16 / 32-byte aligned");
  const int grid = (int)std::min<long>((n / 8 + 255) / 256, (long)sm_count() * 8);
  if (dtype == DUO_BF16)
    DUO_CUDA_TRY(::duo::launch_kernel(to_f32_kernel<__nv_bfloat16>, grid, 256, 0, st,
                                      static_cast<const __nv_bfloat16*>(src), n / 8, dst));
  else if (dtype == DUO_F16)
    DUO_CUDA_TRY(::duo::launch_kernel(to_f32_kernel<__half>, grid, 256, 0, st, static_cast<const __half*>(src), n / 8, dst));
  else
    return fail(DUO_EINVAL, "to_f32: source must be bf16 or f16");
  DUO_LAUNCH_CHECK("to_f32_kernel");
  return DUO_OK;
}

// Per (layer, neuron) of a capture [L, T, I] over tokens t0 .. T-1: max, its first token, min, its first token
// (engine/kernels.js:288-306).  Thread per neuron, consecutive threads on consecutive neurons (coalesced rows).
__global__ void token_extremes_kernel(const float* __restrict__ cap, int L, int T, int I, int t0,
                                      float* __restrict__ out) {
  pdl_enter();
  const int n = blockIdx.x * blockDim.x + threadIdx.x, l = blockIdx.y;
  if (n >= I || l >= L) return;
  float mx = -3.4e38f, mn = 3.4e38f;
  int amx = 0, amn = 0;
  const float* c = cap + (long)l * T * I + n;
  for (int t = t0; t < T; t++) {
    const float v = c[(long)t * I];
    if (v > mx) { mx = v; amx = t; }
    if (v < mn) { mn = v; amn = t; }
  }
  float4* o = reinterpret_cast<float4*>(out + ((long)l * I + n) * 4);
  *o = make_float4(mx, (float)amx, mn, (float)amn);
}

}  // namespace duo

using namespace duo;

extern "C" int duo_rmsnorm(const float* x, int m, int d, const float* w, float eps, int offset, void* y, int y_dtype,
                           duo_stream stream) {
  DUO_CHECK_ARG(m >= 0 && d > 0 && d % 8 == 0, "rmsnorm: d must be a positive multiple of 8");
  DUO_CHECK_ARG(m == 0 || (x && w && y), "rmsnorm: null pointer");
  DUO_CHECK_ARG(valid_act(y_dtype), "rmsnorm: y dtype must be f32, bf16 or f16");
  return launch_rmsnorm(x, m, d, w, eps, offset, y, y_dtype, as_stream(stream));
}

extern "C" int duo_token_extremes(const float* cap, int layers, int t, int inter, int t0, float* out,
                                  duo_stream stream) {
  DUO_CHECK_ARG(layers >= 0 && t >= 0 && inter >= 0 && t0 >= 0, "token_extremes: bad sizes");
  if (layers == 0 || inter == 0) return DUO_OK;
  DUO_CHECK_ARG(cap && out, "token_extremes: null pointer");
  DUO_CHECK_ARG((reinterpret_cast<uintptr_t>(out) & 15) == 0, "token_extremes: out must be 16-byte aligned");
  DUO_CUDA_TRY(::duo::launch_kernel(token_extremes_kernel, dim3(cdiv(inter, 256), layers), 256, 0, as_stream(stream),
                                    cap, layers, t, inter, t0, out));
  DUO_LAUNCH_CHECK("token_extremes_kernel");
  return DUO_OK;
}
