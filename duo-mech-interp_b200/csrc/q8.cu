// int8 "q8" weights: quantiser, dequantiser, embedding gather and the decode GEMV.
//
// Format (engine/kernels.js:1-47 of the reference): symmetric int8 with one f32 scale per group of `group` values
// along a row; scale = absmax / 127 (1 for an all-zero group); q = round(v / scale), half to even.  A row-major
// int8[n, k] array is byte-for-byte the reference's packing of four values per little-endian u32.
#include <algorithm>

#include "common.cuh"

namespace duo {

// ---------------------------------------------------------------------------------------------------------------
// quantise: one 128-thread block per group; IEEE division and round-half-even make it bit-exact

template <typename T> __device__ __forceinline__ float ld_src(const T* p, long i);
template <> __device__ __forceinline__ float ld_src<float>(const float* p, long i) { return p[i]; }
template <> __device__ __forceinline__ float ld_src<__nv_bfloat16>(const __nv_bfloat16* p, long i) {
  return __bfloat162float(p[i]);
}
template <> __device__ __forceinline__ float ld_src<__half>(const __half* p, long i) { return __half2float(p[i]); }

template <typename T>
__global__ void __launch_bounds__(128) q8_quantize_kernel(const T* __restrict__ w, long groups, int group,
                                                          int8_t* __restrict__ q, float* __restrict__ s) {
  pdl_enter();
  __shared__ float red[32];
  for (long g = blockIdx.x; g < groups; g += gridDim.x) {
    const long base = g * (long)group;
    float m = 0.f;
    for (int i = threadIdx.x; i < group; i += blockDim.x) m = fmaxf(m, fabsf(ld_src(w, base + i)));
    m = warp_max(m);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float scale = (m == 0.f) ? 1.f : __fdiv_rn(m, 127.f);
    for (int i = threadIdx.x; i < group; i += blockDim.x) {
      const float v = ld_src(w, base + i);
      q[base + i] = (int8_t)__float2int_rn(__fdiv_rn(v, scale));
    }
    if (threadIdx.x == 0) s[g] = scale;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// dequantise: 16 values per thread

template <typename TO>
__global__ void q8_dequant_kernel(const int8_t* __restrict__ q, const float* __restrict__ s, long total16, int k,
                                  int group, TO* __restrict__ out) {
  pdl_enter();
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total16; i += (long)gridDim.x * blockDim.x) {
    const long e = i * 16;
    const long row = e / k;
    const int col = (int)(e - row * k);
    const float sc = s[row * (k / group) + col / group];
    uint4 u = *reinterpret_cast<const uint4*>(q + e);
    float f[16];
    i8x4_to_f32(u.x, f);
    i8x4_to_f32(u.y, f + 4);
    i8x4_to_f32(u.z, f + 8);
    i8x4_to_f32(u.w, f + 12);
#pragma unroll
    for (int j = 0; j < 16; j++) f[j] *= sc;
    store8(out + e, f);
    store8(out + e + 8, f + 8);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// gather: one 128-thread block per token, 8 values per thread per step

__global__ void q8_gather_kernel(const int32_t* __restrict__ ids, const int8_t* __restrict__ q,
                                 const float* __restrict__ s, int k, int group, int vocab, float* __restrict__ y) {
  pdl_enter();
  const int t = blockIdx.x;
  const int id = ids[t];
  float* yr = y + (long)t * k;
  const bool ok = id >= 0 && id < vocab;
  for (int c = threadIdx.x * 8; c < k; c += blockDim.x * 8) {
    float f[8];
    if (ok) {
      uint2 u = *reinterpret_cast<const uint2*>(q + (long)id * k + c);
      i8x4_to_f32(u.x, f);
      i8x4_to_f32(u.y, f + 4);
      const float sc = s[(long)id * (k / group) + c / group];
#pragma unroll
      for (int j = 0; j < 8; j++) f[j] *= sc;
    } else {
#pragma unroll
      for (int j = 0; j < 8; j++) f[j] = 0.f;
    }
    store8(yr + c, f);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// GEMV for m <= 8 rows of activations: 16 int8 weights per lane per step (one 128-bit streaming load), f32 FMAs,
// per-16 partial sums scaled by the group scale, warp-shuffle reduction per output.

__device__ __forceinline__ uint4 ld_stream16(const int8_t* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

template <typename TX> __device__ __forceinline__ void ld_x16(const TX* p, float* o) {
  load8(p, o);
  load8(p + 8, o + 8);
}

// Each warp owns R consecutive weight rows at a time and issues the 16-byte loads of all of them before using any,
// so R KiB-rows are in flight per warp; blocks of 8 warps stride over the row groups (a grid sized to the SMs).  Per
// row the arithmetic is the one-warp-per-row order: lane l takes bytes 16 l + 512 j of the row, 16 products summed in
// f32, times the group scale, accumulated over j, then a warp butterfly.
template <int M, int R, typename TX, typename TY>
__global__ void __launch_bounds__(256) q8_gemv_kernel(const TX* __restrict__ x, int k, const int8_t* __restrict__ q,
                                                      const float* __restrict__ s, int group, int n,
                                                      TY* __restrict__ y, int accumulate) {
  pdl_enter();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ng = k / group;
  for (int r0 = (blockIdx.x * 8 + warp) * R; r0 < n; r0 += gridDim.x * 8 * R) {
    float acc[M][R];
#pragma unroll
    for (int i = 0; i < M; i++)
#pragma unroll
      for (int r = 0; r < R; r++) acc[i][r] = 0.f;
#pragma unroll 2
    for (int c = lane * 16; c < k; c += 512) {
      uint4 u[R];
      float sc[R];
#pragma unroll
      for (int r = 0; r < R; r++) {
        const int row = min(r0 + r, n - 1);
        u[r] = ld_stream16(q + (long)row * k + c);
        sc[r] = s[(long)row * ng + c / group];
      }
#pragma unroll
      for (int i = 0; i < M; i++) {
        float xv[16];
        ld_x16(x + (long)i * k + c, xv);
#pragma unroll
        for (int r = 0; r < R; r++) {
          float w[16];
          i8x4_to_f32(u[r].x, w);
          i8x4_to_f32(u[r].y, w + 4);
          i8x4_to_f32(u[r].z, w + 8);
          i8x4_to_f32(u[r].w, w + 12);
          float d = 0.f;
#pragma unroll
          for (int j = 0; j < 16; j++) d = fmaf(w[j], xv[j], d);
          acc[i][r] = fmaf(d, sc[r], acc[i][r]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < M; i++)
#pragma unroll
      for (int r = 0; r < R; r++) acc[i][r] = warp_sum(acc[i][r]);
    // lane i * R + r writes y[i][r0 + r]
#pragma unroll
    for (int i = 0; i < M; i++)
#pragma unroll
      for (int r = 0; r < R; r++)
        if (lane == i * R + r && r0 + r < n) {
          TY* yp = y + (long)i * n + r0 + r;
          float v = acc[i][r];
          if (accumulate) v += to_f(*yp);
          *yp = from_f<TY>(v);
        }
  }
}

template <int M> constexpr int gemv_rows() { return M <= 2 ? 8 : M <= 4 ? 4 : 2; }

template <typename TX, typename TY>
int launch_gemv_t(const void* x, int m, int k, const int8_t* q, const float* s, int group, int n, void* y,
                  int accumulate, cudaStream_t st) {
  const TX* xp = static_cast<const TX*>(x);
  TY* yp = static_cast<TY*>(y);
  auto grid_for = [&](int rows_per_warp) { return std::max(1, std::min(cdiv(n, 8 * rows_per_warp), 4 * sm_count())); };
  switch (m) {
#define DUO_GEMV_CASE(MM)                                                                                          \
  case MM:                                                                                                         \
    DUO_CUDA_TRY(::duo::launch_kernel(q8_gemv_kernel<MM, gemv_rows<MM>(), TX, TY>, grid_for(gemv_rows<MM>()), 256, 0, \
                                      st, xp, k, q, s, group, n, yp, accumulate));                                 \
    break;
    DUO_GEMV_CASE(1) DUO_GEMV_CASE(2) DUO_GEMV_CASE(3) DUO_GEMV_CASE(4)
    DUO_GEMV_CASE(5) DUO_GEMV_CASE(6) DUO_GEMV_CASE(7) DUO_GEMV_CASE(8)
#undef DUO_GEMV_CASE
    default: return fail(DUO_EINVAL, "gemv: m must be 1..8");
  }
  DUO_LAUNCH_CHECK("q8_gemv_kernel");
  return DUO_OK;
}

int launch_gemv(const void* x, int x_dtype, int m, int k, const int8_t* q, const float* s, int group, int n, void* y,
                int y_dtype, int accumulate, cudaStream_t st) {
  return with_act(x_dtype, [&](auto xt) -> int {
    return with_act(y_dtype, [&](auto yt) -> int {
      return launch_gemv_t<decltype(xt), decltype(yt)>(x, m, k, q, s, group, n, y, accumulate, st);
    });
  });
}

int launch_gather(const int32_t* ids, int t, const int8_t* q, const float* s, int group, int k, int vocab, float* y,
                  cudaStream_t st) {
  if (t == 0) return DUO_OK;
  DUO_CUDA_TRY(::duo::launch_kernel(q8_gather_kernel, t, 128, 0, st, ids, q, s, k, group, vocab, y));
  DUO_LAUNCH_CHECK("q8_gather_kernel");
  return DUO_OK;
}

int launch_dequant(const int8_t* q, const float* s, int n, int k, int group, void* out, int out_dtype,
                   cudaStream_t st) {
  const long total16 = (long)n * k / 16;
  if (total16 == 0) return DUO_OK;
  const int grid = (int)std::min<long>((total16 + 255) / 256, (long)sm_count() * 16);
  return with_act(out_dtype, [&](auto ot) -> int {
    using TO = decltype(ot);
    DUO_CUDA_TRY(::duo::launch_kernel(q8_dequant_kernel<TO>, grid, 256, 0, st, q, s, total16, k, group, static_cast<TO*>(out)));
    DUO_LAUNCH_CHECK("q8_dequant_kernel");
    return DUO_OK;
  });
}

// ---------------------------------------------------------------------------------------------------------------
// 16-bit (bf16 or f16) pack of an int8 matrix for the tensor-core GEMM (one 128-thread block per row, 8 values per thread)

__device__ __forceinline__ int pack_dst_row(int n, int interleave) {
  if (interleave <= 0) return n;
  const int half = n >= interleave;            // 0: gate row, 1: up row
  const int r = n - half * interleave;
  return (r / 64) * 128 + half * 64 + (r % 64);
}

template <typename TO>
__global__ void q8_pack16_kernel(const int8_t* __restrict__ q, const float* __restrict__ s, int k, int group,
                                    int interleave, int apply_scale, TO* __restrict__ out,
                                    float* __restrict__ colscale) {
  pdl_enter();
  const int n = blockIdx.x;
  const int dn = pack_dst_row(n, interleave);
  const int8_t* qr = q + (long)n * k;
  TO* orow = out + (long)dn * k;
  for (int c = threadIdx.x * 8; c < k; c += blockDim.x * 8) {
    const uint2 u = *reinterpret_cast<const uint2*>(qr + c);
    float f[8];
    i8x4_to_f32(u.x, f);
    i8x4_to_f32(u.y, f + 4);
    if (apply_scale) {
      const float sc = s[(long)n * (k / group) + c / group];
#pragma unroll
      for (int j = 0; j < 8; j++) f[j] *= sc;
    }
    store8(orow + c, f);
  }
  if (colscale && threadIdx.x == 0) colscale[dn] = s[(long)n * (k / group)];
}

int launch_pack16(const int8_t* q, const float* s, int n, int k, int group, int interleave, int apply_scale,
                  int out_dtype, void* out, float* colscale_out, cudaStream_t st) {
  if (n == 0) return DUO_OK;
  if (interleave > 0 && (interleave % 64 || n != 2 * interleave))
    return fail(DUO_EINVAL, "pack: interleave needs n = 2 * interleave, a multiple of 64");
  if (out_dtype == DUO_F16)
    DUO_CUDA_TRY(::duo::launch_kernel(q8_pack16_kernel<__half>, n, 128, 0, st, q, s, k, group, interleave, apply_scale, static_cast<__half*>(out),
                                                colscale_out));
  else
    DUO_CUDA_TRY(::duo::launch_kernel(q8_pack16_kernel<__nv_bfloat16>, n, 128, 0, st, q, s, k, group, interleave, apply_scale,
                                                       static_cast<__nv_bfloat16*>(out), colscale_out));
  DUO_LAUNCH_CHECK("q8_pack16_kernel");
  return DUO_OK;
}

static int check_q8_shape(int n, int k, int group) {
  DUO_CHECK_ARG(n >= 0 && k > 0, "q8: bad shape");
  DUO_CHECK_ARG(group > 0 && k % group == 0, "q8: k must be a multiple of the group size");
  DUO_CHECK_ARG(k % 16 == 0 && group % 16 == 0, "q8: k and the group size must be multiples of 16");
  return DUO_OK;
}

}  // namespace duo

using namespace duo;

extern "C" int duo_q8_quantize(const void* w, int w_dtype, int n, int k, int group, int8_t* q, float* s,
                               duo_stream stream) {
  DUO_TRY(check_q8_shape(n, k, group));
  DUO_CHECK_ARG(w && q && s, "q8_quantize: null pointer");
  const long groups = (long)n * (k / group);
  if (groups == 0) return DUO_OK;
  const int grid = (int)std::min<long>(groups, (long)sm_count() * 32);
  cudaStream_t st = as_stream(stream);
  if (w_dtype == DUO_F32)
    DUO_CUDA_TRY(::duo::launch_kernel(q8_quantize_kernel<float>, grid, 128, 0, st, static_cast<const float*>(w), groups, group, q, s));
  else if (w_dtype == DUO_BF16)
    DUO_CUDA_TRY(::duo::launch_kernel(q8_quantize_kernel<__nv_bfloat16>, grid, 128, 0, st, static_cast<const __nv_bfloat16*>(w), groups, group, q, s));
  else if (w_dtype == DUO_F16)
    DUO_CUDA_TRY(::duo::launch_kernel(q8_quantize_kernel<__half>, grid, 128, 0, st, static_cast<const __half*>(w), groups, group, q, s));
  else
    return fail(DUO_EINVAL, "q8_quantize: w_dtype must be f32, bf16 or f16");
  DUO_LAUNCH_CHECK("q8_quantize_kernel");
  return DUO_OK;
}

extern "C" int duo_q8_dequantize(const int8_t* q, const float* s, int n, int k, int group, void* out, int out_dtype,
                                 duo_stream stream) {
  DUO_TRY(check_q8_shape(n, k, group));
  DUO_CHECK_ARG(q && s && out, "q8_dequantize: null pointer");
  DUO_CHECK_ARG(valid_act(out_dtype), "q8_dequantize: out dtype must be f32, bf16 or f16");
  return launch_dequant(q, s, n, k, group, out, out_dtype, as_stream(stream));
}

extern "C" int duo_q8_gemv(const void* x, int x_dtype, int m, int k, const int8_t* q, const float* s, int group,
                           int n, void* y, int y_dtype, int accumulate, duo_stream stream) {
  DUO_TRY(check_q8_shape(n, k, group));
  DUO_CHECK_ARG(x && q && s && y, "q8_gemv: null pointer");
  DUO_CHECK_ARG(m >= 1 && m <= 8, "q8_gemv: m must be 1..8");
  if (n == 0) return DUO_OK;
  return launch_gemv(x, x_dtype, m, k, q, s, group, n, y, y_dtype, accumulate, as_stream(stream));
}

extern "C" int duo_q8_gather(const int32_t* ids, int t, const int8_t* q, const float* s, int group, int k, int vocab,
                             float* y, duo_stream stream) {
  DUO_TRY(check_q8_shape(vocab, k, group));
  DUO_CHECK_ARG(t >= 0 && (t == 0 || (ids && q && s && y)), "q8_gather: null pointer");
  DUO_CHECK_ARG(k % 8 == 0, "q8_gather: k must be a multiple of 8");
  return launch_gather(ids, t, q, s, group, k, vocab, y, as_stream(stream));
}
