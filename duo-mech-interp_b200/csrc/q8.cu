// int8 "q8" weights: quantiser, dequantiser, embedding gather and the decode GEMV.
//
// Format (engine/kernels.js:1-47 of the reference): symmetric int8 with one f32 scale per group of `group` values
// along a row; scale = absmax / 127 (1 for an all-zero group); q = round(v / scale), half to even.  A row-major
// int8[n, k] array is byte-for-byte the reference's packing of four values per little-endian u32.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "tc.cuh"

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

// The same GEMV with the weights streamed through shared memory: a persistent grid (one CTA per SM), whose producer
// thread copies blocks of CW RPW consecutive weight rows (contiguous bytes of the row-major [n, k] matrix) and their
// group scales into a ring of `nst` slots with 1D bulk copies (cp.async.bulk, completion on a per-slot mbarrier), so
// ~200 KB per SM are in flight however long the consumers take; CW consumer warps take RPW rows of each block
// (16 for one activation row, whose ~3 instructions per weight byte need the warps to hide latency).
// CTA b handles blocks b, b + grid, ..., so neighbouring CTAs stream neighbouring memory.  Per row the arithmetic is
// exactly the register kernel's (lane l takes bytes 16 l + 512 j, 16 products in f32 times the group scale,
// accumulated over j, then the same butterfly), so the two give identical outputs.  Waits are bounded (fault code
// 1024 when one gives up).
constexpr int GS_RING = 210 * 1024;
template <int M> constexpr int gemv_stream_warps() { return M == 1 ? 16 : 8; }

template <int M, int RPW, bool XPRE, typename TX, typename TY>
__global__ void __launch_bounds__(32 * gemv_stream_warps<M>() + 32, 1)
    q8_gemv_stream_kernel(const TX* __restrict__ x, int k, const int8_t* __restrict__ q, const float* __restrict__ s,
                          int group, int n, TY* __restrict__ y, int accumulate, int nst, unsigned* fault) {
  constexpr int CW = gemv_stream_warps<M>(), RS = CW * RPW;  // consumer warps, rows per block
  if (tc::fault_pending(fault)) {
    pdl_wait();
    return;
  }
  extern __shared__ __align__(128) uint8_t gsm[];
  const int ng = k / group;
  const uint32_t wb = (uint32_t)(RS * k), sbytes = (uint32_t)(RS * ng * 4);
  uint8_t* wring = gsm;
  float* sring = reinterpret_cast<float*>(gsm + (size_t)nst * wb);
  uint64_t* full = reinterpret_cast<uint64_t*>(gsm + (size_t)nst * (wb + sbytes));
  uint64_t* empty = full + nst;
  volatile int* abort = reinterpret_cast<volatile int*>(empty + nst);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int i = 0; i < nst; i++) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], CW);
    }
    *abort = 0;
    tc::fence_mbar_init();
  }
  __syncthreads();
  pdl_enter();
  const int nblk = (n + RS - 1) / RS;
  if (warp == CW) {
    if (lane == 0) {  // producer
      int issued = 0;
      for (int bk = blockIdx.x, li = 0; bk < nblk && !*abort; bk += gridDim.x, li++) {
        const int sl = li % nst;
        if (li >= nst && !tc::mbar_wait(&empty[sl], (uint32_t)((li / nst - 1) & 1))) {
          atomicOr(fault, 1024u);
          *abort = 1;
          break;
        }
        const int rows = min(RS, n - bk * RS);  // n % 4 == 0: the scale bytes stay a multiple of 16
        tc::mbar_arrive_expect_tx(&full[sl], (uint32_t)(rows * k + rows * ng * 4));
        tc::bulk_g2s(wring + (size_t)sl * wb, q + (long)bk * RS * k, (uint32_t)(rows * k), &full[sl]);
        tc::bulk_g2s(sring + (size_t)sl * (sbytes / 4), s + (long)bk * RS * ng, (uint32_t)(rows * ng * 4), &full[sl]);
        issued = li + 1;
      }
      // no copy may still be landing when the CTA exits (the consumers wait for every block unless aborted)
      for (int li = max(0, issued - nst); li < issued; li++) tc::mbar_wait(&full[li % nst], (uint32_t)((li / nst) & 1));
    }
  } else {  // consumers: warp w takes rows w RPW .. of each block
    // XPRE (one activation row, k <= 1024): this lane's 32 activations stay in registers for the whole call
    float xr[XPRE ? 2 : 1][16];
    if constexpr (XPRE) {
#pragma unroll
      for (int j = 0; j < 2; j++) {
        const int c = lane * 16 + 512 * j;
        if (c < k) ld_x16(x + c, xr[j]);
      }
    }
    for (int bk = blockIdx.x, li = 0; bk < nblk; bk += gridDim.x, li++) {
      const int sl = li % nst;
      if (*abort || !tc::mbar_wait(&full[sl], (uint32_t)((li / nst) & 1))) {
        if (lane == 0) {
          atomicOr(fault, 1024u);
          *abort = 1;
        }
        break;
      }
      const int r0 = bk * RS + warp * RPW;
      const uint8_t* wr = wring + (size_t)sl * wb + (size_t)warp * RPW * k;
      const float* sr = sring + (size_t)sl * (sbytes / 4) + warp * RPW * ng;
      float acc[M][RPW];
#pragma unroll
      for (int i = 0; i < M; i++)
#pragma unroll
        for (int r = 0; r < RPW; r++) acc[i][r] = 0.f;
#pragma unroll 2
      for (int c = lane * 16, j = 0; c < k; c += 512, j++) {
        uint4 u[RPW];
        float sc[RPW];
#pragma unroll
        for (int r = 0; r < RPW; r++) {  // rows past n hold stale bytes: computed, never stored
          u[r] = *reinterpret_cast<const uint4*>(wr + (size_t)r * k + c);
          sc[r] = sr[r * ng + c / group];
        }
#pragma unroll
        for (int i = 0; i < M; i++) {
          float xv[16];
          if constexpr (XPRE) {
#pragma unroll
            for (int e = 0; e < 16; e++) xv[e] = xr[j & 1][e];
          } else {
            ld_x16(x + (long)i * k + c, xv);
          }
#pragma unroll
          for (int r = 0; r < RPW; r++) {
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
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&empty[sl]);  // this warp is done with the slot's bytes
#pragma unroll
      for (int i = 0; i < M; i++)
#pragma unroll
        for (int r = 0; r < RPW; r++) acc[i][r] = warp_sum(acc[i][r]);
#pragma unroll
      for (int i = 0; i < M; i++)
#pragma unroll
        for (int r = 0; r < RPW; r++)
          if (lane == i * RPW + r && r0 + r < n) {
            TY* yp = y + (long)i * n + r0 + r;
            float v = acc[i][r];
            if (accumulate) v += to_f(*yp);
            *yp = from_f<TY>(v);
          }
    }
  }
  __syncthreads();
}

template <int M, int RPW, bool XPRE, typename TX, typename TY>
int run_gemv_stream(const TX* x, int k, const int8_t* q, const float* s, int group, int n, TY* y, int accumulate,
                    cudaStream_t st) {
  constexpr int RS = gemv_stream_warps<M>() * RPW;
  const long slot = (long)RS * k + (long)RS * (k / group) * 4;
  const int nst = (int)std::min<long>(8, GS_RING / slot);
  const int smem = (int)(nst * slot + 16 * nst + 16);
  unsigned* fault = tc_fault_ptr();
  if (!fault) return fail(DUO_ECUDA, "tensor-core fault word is not addressable");
  auto kern = q8_gemv_stream_kernel<M, RPW, XPRE, TX, TY>;
  DUO_TRY(ensure_smem_attr(kern, smem));
  const int grid = std::min(cdiv(n, RS), sm_count());
  DUO_CUDA_TRY(::duo::launch_kernel(kern, grid, 32 * gemv_stream_warps<M>() + 32, smem, st, x, k, q, s, group, n, y,
                                    accumulate, nst, fault));
  DUO_LAUNCH_CHECK("q8_gemv_stream_kernel");
  return DUO_OK;
}

// Streaming form for matrices large enough to be bandwidth-bound: 16-byte aligned weights and scales, k a multiple
// of 16 and of the group, n a multiple of 4 (whole 16-byte scale copies), and at least two ring slots.
// Rows per consumer warp and block: ~4 KB of a block per warp, at most 2 rows when m > 4 (registers).
static int gemv_stream_rpw(int m, int k) {
  const int r = k <= 1024 ? 4 : k <= 2048 ? 2 : 1;
  return m > 4 ? std::min(r, 2) : r;
}
static bool gemv_stream_ok(int m, int k, const int8_t* q, const float* s, int group, int n) {
  if (n < 2048 || n % 4 || k % 16 || group <= 0 || k % group) return false;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(s)) & 15) return false;
  const int rpw = gemv_stream_rpw(m, k);
  const long rs = (m == 1 ? 16L : 8L) * rpw;
  const long slot = rs * k + rs * (k / group) * 4;
  return GS_RING / slot >= 2;
}

template <typename TX, typename TY>
int launch_gemv_t(const void* x, int m, int k, const int8_t* q, const float* s, int group, int n, void* y,
                  int accumulate, cudaStream_t st) {
  const TX* xp = static_cast<const TX*>(x);
  TY* yp = static_cast<TY*>(y);
  if (m >= 1 && m <= 8 && gemv_stream_ok(m, k, q, s, group, n)) {
    const int rpw = gemv_stream_rpw(m, k);
    auto pick = [&](auto mm) -> int {
      constexpr int MM = decltype(mm)::value;
      if constexpr (MM == 1)
        if (rpw == 4) return run_gemv_stream<1, 4, true>(xp, k, q, s, group, n, yp, accumulate, st);  // k <= 1024
      if constexpr (MM <= 4)
        if (rpw == 4) return run_gemv_stream<MM, 4, false>(xp, k, q, s, group, n, yp, accumulate, st);
      if (rpw == 2) return run_gemv_stream<MM, 2, false>(xp, k, q, s, group, n, yp, accumulate, st);
      return run_gemv_stream<MM, 1, false>(xp, k, q, s, group, n, yp, accumulate, st);
    };
    switch (m) {
      case 1: return pick(std::integral_constant<int, 1>{});
      case 2: return pick(std::integral_constant<int, 2>{});
      case 3: return pick(std::integral_constant<int, 3>{});
      case 4: return pick(std::integral_constant<int, 4>{});
      case 5: return pick(std::integral_constant<int, 5>{});
      case 6: return pick(std::integral_constant<int, 6>{});
      case 7: return pick(std::integral_constant<int, 7>{});
      default: return pick(std::integral_constant<int, 8>{});
    }
  }
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
