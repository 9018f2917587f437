// Projections of the forward: the bf16 tensor-core GEMM (tcgen05 + TMA + TMEM) and the f32 CUDA-core GEMM on int8
// weights used by the f32 engine.  Both compute acc[m, n] = sum_k A[m, k] W[n, k] and hand it to one of the
// epilogues of GemmEpi (plain store, residual add with the optional steering vector, SwiGLU with neuron pushes).
//
// The reference computes these products with `matvec` / `matmul` (engine/kernels.js:55-151) in f32 on int8 weights
// dequantised per 128-group; model.js:382-396 picks between them by row count.
#include <cooperative_groups.h>

#include <algorithm>
#include <mutex>

#include "kernels.cuh"
#include "tc.cuh"

namespace duo {

namespace cg = cooperative_groups;

// ---------------------------------------------------------------------------------------------------------------
// tcgen05 GEMM for small grids with more than 256 rows (decode-sized row counts go to gemm_dec.cu): one CTA per
// 128 x BN tile (x a K range), K step 64 (one 128-byte swizzle row of 16-bit values), a ~96 KB TMA ring so that two
// CTAs share an SM.  Large grids go to the persistent kernel (gemm_persist.cu).  Warp 0: TMA producer (one lane).  Warp 1: TMEM allocator and MMA issuer (one lane).
// Warps 2-5: epilogue, one accumulator row (TMEM lane) per thread, read 32 columns at a time.

constexpr int TC_BM = 128, TC_BK = 64, TC_THREADS = 192;

// the f32 epilogue tile reuses the pipeline buffers (idle once every MMA has completed)
__device__ __forceinline__ float* stile_of(uint8_t* smem) { return reinterpret_cast<float*>(smem); }

template <int BN> struct TcCfg {
  static constexpr int A_BYTES = TC_BM * TC_BK * 2;
  static constexpr int B_BYTES = BN * TC_BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (96 * 1024) / STAGE_BYTES;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

template <int BN, int EPI, bool F16>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b, int M, int N,
                   int K, int kper, GemmEpiArgs ep, unsigned* fault) {
  using C = TcCfg<BN>;
  static_assert(C::STAGES >= 2, "ring too small");
  static_assert(TC_BM * ((EPI == EPI_SWIGLU ? BN / 2 : BN) + 4) * 4 <= C::STAGES * C::STAGE_BYTES,
                "the epilogue tile must fit in the ring");
  if (gridDim.z == 1 && tc::fault_pending(fault)) {  // an earlier kernel gave up a wait (no cluster when z == 1)
    pdl_wait();
    return;
  }
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + C::STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tmem_full = empty + C::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile_n = blockIdx.x * BN, tile_m = blockIdx.y * TC_BM;
  // split-K (residual-add epilogue only): this CTA reduces k blocks [kb0, kb0 + num_k)
  const int kb0 = blockIdx.z * kper;
  const int num_k = min(kper, K / TC_BK - kb0);
  const bool split = gridDim.z > 1;  // launched as a cluster of gridDim.z CTAs along z (residual add only)
  bool epi_ok = false;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; s++) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(tmem_full, 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tma_a);
    tc::prefetch_tmap(&tma_b);
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, BN);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  // Programmatic launch: constant weight tiles of the first stages stream in while the preceding kernel finishes;
  // everything else waits for it.
  const int pre = ep.b_const ? min(num_k, C::STAGES) : 0;
  if (warp == 0 && lane == 0) {
    for (int kb = 0; kb < pre; kb++) {
      tc::mbar_arrive_expect_tx(&full[kb], C::STAGE_BYTES);
      tc::tma_load_2d(sb + kb * C::B_BYTES, &tma_b, (kb0 + kb) * TC_BK, tile_n, &full[kb]);
    }
  }
  pdl_wait();
  pdl_trigger();

  if (warp == 0 && lane == 0) {
    for (int kb = 0; kb < num_k; kb++) {
      const int s = kb % C::STAGES;
      const uint32_t ph = (kb / C::STAGES) & 1;
      if (kb < pre) {  // its B tile is already on the way
        tc::tma_load_2d(sa + s * C::A_BYTES, &tma_a, (kb0 + kb) * TC_BK, tile_m, &full[s]);
        continue;
      }
      if (kb >= C::STAGES && !tc::mbar_wait(&empty[s], ph ^ 1)) {
        atomicOr(fault, 1u);
        break;
      }
      tc::mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
      tc::tma_load_2d(sa + s * C::A_BYTES, &tma_a, (kb0 + kb) * TC_BK, tile_m, &full[s]);
      tc::tma_load_2d(sb + s * C::B_BYTES, &tma_b, (kb0 + kb) * TC_BK, tile_n, &full[s]);
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = tc::idesc_16_f32(TC_BM, BN, F16);
    const uint64_t da0 = tc::desc_kmajor_sw128(tc::smem_u32(sa)), db0 = tc::desc_kmajor_sw128(tc::smem_u32(sb));
    bool ok = true;
    for (int kb = 0; kb < num_k; kb++) {
      const int s = kb % C::STAGES;
      const uint32_t ph = (kb / C::STAGES) & 1;
      if (!tc::mbar_wait(&full[s], ph)) {
        atomicOr(fault, 2u);
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const uint64_t da = tc::desc_add(da0, s * C::A_BYTES), db = tc::desc_add(db0, s * C::B_BYTES);
#pragma unroll
      for (int k = 0; k < TC_BK / 16; k++)  // 16 k = 32 bytes along the swizzled rows
        tc::mma_bf16(tmem, tc::desc_add(da, 32 * k), tc::desc_add(db, 32 * k), idesc, (kb | k) != 0);
      tc::mma_commit(&empty[s]);
    }
    if (ok) tc::mma_commit(tmem_full);
  } else if (warp >= 2) {
    // Epilogue in two passes.  (1) Each warp moves its 32 accumulator rows TMEM -> registers -> (scaled, and for
    // SwiGLU combined) f32 rows of a shared-memory tile that reuses the pipeline buffers, idle once every MMA has
    // completed.  (2) The four warps sweep the tile row by row with consecutive lanes on consecutive columns, so every
    // global load / store of the output (and the residual read-modify-write) is coalesced.
    constexpr int NC = (EPI == EPI_SWIGLU) ? BN / 2 : BN;  // output columns of this tile
    constexpr int P = NC + 4;                               // row pitch: rows start 4 banks apart
    float* stile = stile_of(smem);
    const int quad = warp & 3;  // TMEM lanes 32*quad .. 32*quad+31 belong to this warp
    const int row = quad * 32 + lane;
    const bool ok = tc::mbar_wait(tmem_full, 0);
    epi_ok = ok;
    if (!ok) {
      if (lane == 0) atomicOr(fault, 4u);
    } else {
      tc::fence_after_sync();
      const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
      float* srow = stile + row * P;
#pragma unroll 1
      for (int c0 = 0; c0 < NC; c0 += 32) {
        float v[32];
        if (EPI != EPI_SWIGLU) tc::tmem_ld32(trow + c0, v);
        if (EPI == EPI_SWIGLU) {
          // the tile's columns come in 128-wide groups [64 gate rows | the matching 64 up rows]; output columns
          // c0 .. c0 + 31 take gate column gc and up column gc + 64
          const int gc = (c0 / 64) * 128 + (c0 % 64);
          tc::tmem_ld32(trow + gc, v);
          float u[32];
          tc::tmem_ld32(trow + gc + 64, u);
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const float gs = ep.colscale ? v[j] * ep.colscale[tile_n + gc + j] : v[j];
            const float us = ep.colscale ? u[j] * ep.colscale[tile_n + gc + 64 + j] : u[j];
            v[j] = silu16_(gs) * us;
          }
        } else if (ep.colscale) {
#pragma unroll
          for (int j = 0; j < 32; j++) v[j] *= (tile_n + c0 + j < N) ? ep.colscale[tile_n + c0 + j] : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(srow + c0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      }
    }
    if (!split) asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
    if (ok && !split) {
      const int ew = warp - 2;
      const int n0 = (EPI == EPI_SWIGLU) ? tile_n / 2 : tile_n;  // first output column of the tile
      const int ncols = (EPI == EPI_SWIGLU) ? N / 2 : N;          // output width
      const bool al = ((reinterpret_cast<uintptr_t>(ep.c) & 15) == 0) && (ep.ldc % 4 == 0);
      for (int rr = ew; rr < TC_BM; rr += 4) {
        const int m = tile_m + rr;
        if (m >= M) break;
        const int r = ep.row_base + m / ep.t;
        const float* srow = stile + rr * P;
        for (int c = lane * 4; c < NC; c += 128) {
          const int n = n0 + c;
          if (n >= ncols) break;
          float4 v = *reinterpret_cast<const float4*>(srow + c);
          float x[4] = {v.x, v.y, v.z, v.w};
          const long off = (long)m * ep.ldc + n;
          const bool vec4 = al && n + 4 <= ncols;
          if (EPI == EPI_SWIGLU && ep.push.count) {
            const unsigned pm = push_mask(ep.push, n, 4);
            if (pm) {
#pragma unroll
              for (int i = 0; i < 4; i++) x[i] = push_apply_masked(ep.push, pm, r, n + i, x[i]);
            }
          }
          if (EPI == EPI_ADD_F32) {
            float* X = static_cast<float*>(ep.c) + off;
            const float* vr = ep.vec ? ep.vec + (long)r * ep.ldc + n : nullptr;
            if (vec4) {
              float4 o = *reinterpret_cast<float4*>(X);
              o.x += x[0]; o.y += x[1]; o.z += x[2]; o.w += x[3];
              if (vr) {
                const float4 a = *reinterpret_cast<const float4*>(vr);
                o.x += a.x; o.y += a.y; o.z += a.z; o.w += a.w;
              }
              *reinterpret_cast<float4*>(X) = o;
            } else {
              for (int i = 0; i < 4 && n + i < ncols; i++) X[i] += x[i] + (vr ? vr[i] : 0.f);
            }
          } else if (ep.c_dtype == DUO_F16) {
            __half* C = static_cast<__half*>(ep.c) + off;
            if (vec4) {
              __half2 lo = __floats2half2_rn(x[0], x[1]), hi = __floats2half2_rn(x[2], x[3]);
              uint2 u;
              u.x = *reinterpret_cast<uint32_t*>(&lo);
              u.y = *reinterpret_cast<uint32_t*>(&hi);
              *reinterpret_cast<uint2*>(C) = u;
            } else {
              for (int i = 0; i < 4 && n + i < ncols; i++) C[i] = __float2half_rn(x[i]);
            }
          } else if (ep.c_dtype == DUO_BF16) {
            __nv_bfloat16* C = static_cast<__nv_bfloat16*>(ep.c) + off;
            if (vec4) {
              __nv_bfloat162 lo = __floats2bfloat162_rn(x[0], x[1]), hi = __floats2bfloat162_rn(x[2], x[3]);
              uint2 u;
              u.x = *reinterpret_cast<uint32_t*>(&lo);
              u.y = *reinterpret_cast<uint32_t*>(&hi);
              *reinterpret_cast<uint2*>(C) = u;
            } else {
              for (int i = 0; i < 4 && n + i < ncols; i++) C[i] = __float2bfloat16_rn(x[i]);
            }
          } else {
            float* C = static_cast<float*>(ep.c) + off;
            if (vec4) *reinterpret_cast<float4*>(C) = make_float4(x[0], x[1], x[2], x[3]);
            else for (int i = 0; i < 4 && n + i < ncols; i++) C[i] = x[i];
          }
        }
      }
    }
  }
  if (split) {
    // K split across the CTAs of this cluster (blockIdx.z = cluster rank): once every partial tile is in its CTA's
    // shared memory, CTA z sums rows [z rpc, z rpc + rpc) of all of them over distributed shared memory, in rank
    // order (deterministic), and does the residual read-modify-write for those rows.
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (warp >= 2 && epi_ok) {
      constexpr int P = BN + 4;
      const int ks = gridDim.z, z = blockIdx.z;
      const int rpc = (TC_BM + ks - 1) / ks;
      const int r_hi = min(TC_BM, (z + 1) * rpc);
      const bool al = ((reinterpret_cast<uintptr_t>(ep.c) & 15) == 0) && (ep.ldc % 4 == 0) &&
                      (ep.vec == nullptr || (reinterpret_cast<uintptr_t>(ep.vec) & 15) == 0);
      for (int rr = z * rpc + (warp - 2); rr < r_hi; rr += 4) {
        const int m = tile_m + rr;
        if (m >= M) break;
        const int r = ep.row_base + m / ep.t;
        for (int c = lane * 4; c < BN; c += 128) {
          const int n = tile_n + c;
          if (n >= N) break;
          float x[4] = {0.f, 0.f, 0.f, 0.f};
          for (int q = 0; q < ks; q++) {
            const float4 v = *reinterpret_cast<const float4*>(cluster.map_shared_rank(stile_of(smem), q) + rr * P + c);
            x[0] += v.x; x[1] += v.y; x[2] += v.z; x[3] += v.w;
          }
          float* X = static_cast<float*>(ep.c) + (long)m * ep.ldc + n;
          const float* vr = ep.vec ? ep.vec + (long)r * ep.ldc + n : nullptr;
          if (al && n + 4 <= N) {
            float4 o = *reinterpret_cast<float4*>(X);
            o.x += x[0]; o.y += x[1]; o.z += x[2]; o.w += x[3];
            if (vr) {
              const float4 a = *reinterpret_cast<const float4*>(vr);
              o.x += a.x; o.y += a.y; o.z += a.z; o.w += a.w;
            }
            *reinterpret_cast<float4*>(X) = o;
          } else {
            for (int i = 0; i < 4 && n + i < N; i++) X[i] += x[i] + (vr ? vr[i] : 0.f);
          }
        }
      }
    }
    cluster.sync();  // no CTA leaves while a peer may still read its tile
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, BN);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// host side

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  });
  return fn;
}

int make_tmap_16(CUtensorMap* map, const void* base, int dtype, long rows, long cols, long ld, int box_rows,
                int box_cols) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return fail(DUO_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld * 2) % 16)
    return fail(DUO_EINVAL, "tensor map: base must be 16-byte aligned and rows a multiple of 16 bytes");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = dtype == DUO_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DUO_ECUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
  return DUO_OK;
}

int make_tmap_nd_16(CUtensorMap* map, const void* base, int dtype, int rank, const long* dims, const long* strides,
                    const int* box) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return fail(DUO_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (rank < 2 || rank > 5) return fail(DUO_EINVAL, "tensor map: rank must be 2..5");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (box[0] * 2) % 16 || box[0] * 2 > 128)
    return fail(DUO_EINVAL, "tensor map: base 16-byte aligned, box row a multiple of 16 bytes and at most 128");
  cuuint64_t d[5], s[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; i++) {
    d[i] = (cuuint64_t)dims[i];
    bx[i] = (cuuint32_t)box[i];
    es[i] = 1;
    if (i + 1 < rank) {
      if (strides[i] % 16) return fail(DUO_EINVAL, "tensor map: strides must be multiples of 16 bytes");
      s[i] = (cuuint64_t)strides[i];
    }
  }
  const CUtensorMapDataType dt = dtype == DUO_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUresult r = enc(map, dt, (cuuint32_t)rank, const_cast<void*>(base), d, s, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DUO_ECUDA, "cuTensorMapEncodeTiled (N-d) failed with code " + std::to_string((int)r));
  return DUO_OK;
}

int make_tmap_3d_16(CUtensorMap* map, const void* base, int dtype, long d0, long d1, long d2, long s1, long s2,
                    int box0, int box1) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return fail(DUO_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || s1 % 16 || s2 % 16 || (box0 * 2) % 16)
    return fail(DUO_EINVAL, "tensor map: base, strides and the box row must be multiples of 16 bytes");
  cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2};
  cuuint64_t strides[2] = {(cuuint64_t)s1, (cuuint64_t)s2};
  cuuint32_t box[3] = {(cuuint32_t)box0, (cuuint32_t)box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt = dtype == DUO_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUresult r = enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DUO_ECUDA, "cuTensorMapEncodeTiled (3D) failed with code " + std::to_string((int)r));
  return DUO_OK;
}

int make_tmap_plain(CUtensorMap* map, const void* base, int dtype, long rows, long cols, long ld, int box_rows,
                    int box_cols) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return fail(DUO_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const int es = dtype == DUO_F32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld * es) % 16 || (box_cols * es) % 16)
    return fail(DUO_EINVAL, "tensor map: base, rows and box rows must be multiples of 16 bytes");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * es)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = dtype == DUO_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == DUO_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DUO_ECUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
  return DUO_OK;
}

template <int BN, int EPI, bool F16>
static int run_tc(const CUtensorMap& ta, const CUtensorMap& tb, int m, int n, int k, int ksplit,
                  const GemmEpiArgs& ep, cudaStream_t st) {
  using C = TcCfg<BN>;
  DUO_TRY(ensure_smem_attr(gemm_tc_kernel<BN, EPI, F16>, C::SMEM));
  unsigned* fault = tc_fault_ptr();
  if (!fault) return fail(DUO_ECUDA, "tensor-core fault word is not addressable");
  const int num_k = k / TC_BK;
  const int kper = cdiv(num_k, ksplit);
  dim3 grid(cdiv(n, BN), cdiv(m, TC_BM), cdiv(num_k, kper));
  if (grid.z == 1) {
    DUO_CUDA_TRY(::duo::launch_kernel(gemm_tc_kernel<BN, EPI, F16>, grid, TC_THREADS, C::SMEM, st, ta, tb, m, n, k, kper, ep, fault));
  } else {
    // K split: the grid.z CTAs of one output tile form a cluster and reduce their partial tiles on chip
    DUO_CHECK_ARG(EPI == EPI_ADD_F32 && grid.z <= 8, "gemm_tc: K split only for the residual add, at most 8 ways");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = grid.z;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    DUO_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BN, EPI, F16>, ta, tb, m, n, k, kper, ep, fault));
  }
  DUO_LAUNCH_CHECK("gemm_tc_kernel");
  return DUO_OK;
}

template <bool F16>
static int dispatch_tc(const CUtensorMap& ta, const CUtensorMap& tb, int bn, int ksplit, int m, int n, int k,
                       const GemmEpiArgs& ep, cudaStream_t st) {
  if (ep.epi == EPI_SWIGLU) return run_tc<128, EPI_SWIGLU, F16>(ta, tb, m, n, k, 1, ep, st);
  if (ep.epi == EPI_ADD_F32)
    return bn == 128 ? run_tc<128, EPI_ADD_F32, F16>(ta, tb, m, n, k, ksplit, ep, st)
                     : run_tc<64, EPI_ADD_F32, F16>(ta, tb, m, n, k, ksplit, ep, st);
  return bn == 128 ? run_tc<128, EPI_STORE, F16>(ta, tb, m, n, k, 1, ep, st)
                   : run_tc<64, EPI_STORE, F16>(ta, tb, m, n, k, 1, ep, st);
}

int launch_gemm_tc(const void* a, int m, int k, const void* b, int n, int ab_dtype, const GemmEpiArgs& ep,
                   cudaStream_t st) {
  if (m == 0 || n == 0) return DUO_OK;
  DUO_CHECK_ARG(k % TC_BK == 0, "gemm_tc: k must be a multiple of 64");
  DUO_CHECK_ARG(ab_dtype == DUO_BF16 || ab_dtype == DUO_F16, "gemm_tc: operands must be bf16 or f16");
  // decode-sized row counts: the weights-on-M kernel (row groups x weight blocks x K slices)
  if (m <= 256 && ep.epi != EPI_ARGMAX) return launch_gemm_dec(a, m, k, b, n, ab_dtype, ep, st);
  // the fused RMSNorm (producer partials per 256 columns, consumer row factors) is an epilogue of the persistent
  // kernel with 256-wide tiles, whatever the grid
  const bool fused_norm = ep.nrm_out || ep.row_part;
  if (ep.nrm_out) {
    const bool al = ((reinterpret_cast<uintptr_t>(ep.nrm_out) | reinterpret_cast<uintptr_t>(ep.c) |
                      reinterpret_cast<uintptr_t>(ep.nrm_w)) & 15) == 0 && ep.ldc % 8 == 0;
    DUO_CHECK_ARG(ep.epi == EPI_ADD_F32 && n % 256 == 0 && al && ep.nrm_w && ep.nrm_part,
                  "gemm_tc: the fused norm needs the residual add, n a multiple of 256 and 16-byte aligned rows");
  }
  if (ep.row_part)
    DUO_CHECK_ARG((ep.epi == EPI_STORE || ep.epi == EPI_SWIGLU) && ep.row_blocks > 0 && ep.row_d > 0,
                  "gemm_tc: row factors apply to the store and SwiGLU epilogues");
  const int sms = sm_count();
  const long tiles_m = cdiv(m, TC_BM);
  // the widest N tile that still gives every SM work (SwiGLU: gate / up interleaved per 64 rows, tiles >= 128)
  if (ep.epi == EPI_SWIGLU) DUO_CHECK_ARG(n % 128 == 0, "gemm_tc: SwiGLU epilogue needs n a multiple of 128");
  int bn = 256;
  if (!fused_norm && tiles_m * cdiv(n, 256) < sms) bn = 128;
  if (!fused_norm && ep.epi != EPI_SWIGLU && tiles_m * cdiv(n, 128) < sms) bn = 64;
  const long tiles = tiles_m * cdiv(n, bn);
  // small grid: per-tile kernel, two CTAs per SM; otherwise the persistent kernel
  const bool small = bn == 64 || (bn == 128 && tiles < 2L * sms);
  CUtensorMap ta, tb;
  DUO_TRY(make_tmap_16(&ta, a, ab_dtype, m, k, k, TC_BM, TC_BK));
  DUO_TRY(make_tmap_16(&tb, b, ab_dtype, n, k, k, bn, TC_BK));
  if (!small) return launch_gemm_persist(ta, tb, bn, m, n, k, ab_dtype, ep, st);
  int ksplit = 1;
  if (ep.epi == EPI_ADD_F32) {  // still too few CTAs: split K over a cluster, partial tiles summed on chip
    const int num_k = k / TC_BK;
    ksplit = (int)std::max<long>(1, std::min<long>({2L * sms / tiles, 8, num_k / 4}));
  }
  return ab_dtype == DUO_F16 ? dispatch_tc<true>(ta, tb, bn, ksplit, m, n, k, ep, st)
                             : dispatch_tc<false>(ta, tb, bn, ksplit, m, n, k, ep, st);
}

// ---------------------------------------------------------------------------------------------------------------
// f32 CUDA-core GEMM on int8 weights (the f32 engine; the reference's precision).  64 x 64 tiles, K step 32,
// 256 threads with 4 x 4 outputs each; weights dequantised (f32(q) * scale) while staging into shared memory.

__global__ void __launch_bounds__(256) gemm_f32_q8_kernel(const float* __restrict__ A, int M, int K,
                                                           const int8_t* __restrict__ W, const float* __restrict__ S,
                                                           int group, int N, GemmEpiArgs ep) {
  pdl_enter();
  __shared__ float As[32][64 + 4];
  __shared__ float Ws[32][64 + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  const int groups = K / group;
  for (int k0 = 0; k0 < K; k0 += 32) {
    for (int e = threadIdx.x; e < 64 * 32; e += 256) {
      const int r = e >> 5, kk = e & 31;
      const int gm = m0 + r, gn = n0 + r;
      As[kk][r] = gm < M ? A[(long)gm * K + k0 + kk] : 0.f;
      Ws[kk][r] = gn < N ? (float)W[(long)gn * K + k0 + kk] * S[(long)gn * groups + (k0 + kk) / group] : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < 32; kk++) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; i++) { a[i] = As[kk][ty * 4 + i]; b[i] = Ws[kk][tx * 4 + i]; }
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int n = n0 + tx * 4 + j;
      if (n >= N) continue;
      float v = acc[i][j] * (ep.colscale ? ep.colscale[n] : 1.f);
      const long off = (long)m * ep.ldc + n;
      if (ep.epi == EPI_STORE) {
        if (ep.c_dtype == DUO_F32) static_cast<float*>(ep.c)[off] = v;
        else static_cast<__nv_bfloat16*>(ep.c)[off] = __float2bfloat16_rn(v);
      } else {
        float* x = static_cast<float*>(ep.c);
        if (ep.vec) v += ep.vec[(long)(ep.row_base + m / ep.t) * ep.ldc + n];
        x[off] += v;
      }
    }
  }
}

int launch_gemm_f32_q8(const float* a, int m, int k, const int8_t* q, const float* s, int group, int n,
                       const GemmEpiArgs& ep, cudaStream_t st) {
  if (m == 0 || n == 0) return DUO_OK;
  DUO_CHECK_ARG(k % 32 == 0, "gemm_f32: k must be a multiple of 32");
  DUO_CHECK_ARG(ep.epi == EPI_STORE || ep.epi == EPI_ADD_F32, "gemm_f32: store or add epilogue only");
  DUO_CUDA_TRY(::duo::launch_kernel(gemm_f32_q8_kernel, dim3(cdiv(n, 64), cdiv(m, 64)), 256, 0, st, a, m, k, q, s, group, n, ep));
  DUO_LAUNCH_CHECK("gemm_f32_q8_kernel");
  return DUO_OK;
}

}  // namespace duo

using namespace duo;

extern "C" int duo_gemm_bf16(const void* a, int m, int k, const void* b, int n, const float* col_scale, void* c,
                             int c_dtype, int ldc, int accumulate, duo_stream stream) {
  DUO_CHECK_ARG(m >= 0 && n >= 0 && k > 0, "gemm_bf16: bad shape");
  DUO_CHECK_ARG(k % 64 == 0, "gemm_bf16: k must be a multiple of 64");
  DUO_CHECK_ARG(m == 0 || n == 0 || (a && b && c), "gemm_bf16: null pointer");
  DUO_CHECK_ARG(valid_act(c_dtype), "gemm_bf16: c dtype must be f32, bf16 or f16");
  DUO_CHECK_ARG(ldc >= n, "gemm_bf16: ldc < n");
  DUO_CHECK_ARG(!accumulate || c_dtype == DUO_F32, "gemm_bf16: accumulate needs an f32 C");
  GemmEpiArgs ep;
  ep.epi = accumulate ? EPI_ADD_F32 : EPI_STORE;
  ep.c = c;
  ep.c_dtype = c_dtype;
  ep.ldc = ldc;
  ep.colscale = col_scale;
  return launch_gemm_tc(a, m, k, b, n, DUO_BF16, ep, as_stream(stream));
}

extern "C" int duo_q8_gemm(const void* x, int x_dtype, int m, int k, const int8_t* q, const float* s, int group,
                           int n, int swiglu, void* y, int y_dtype, int ldy, int accumulate, duo_stream stream) {
  DUO_CHECK_ARG(m >= 0 && m <= 256 && n >= 0 && k > 0, "q8_gemm: 0 <= m <= 256 rows, n >= 0, k > 0");
  DUO_CHECK_ARG(x_dtype == DUO_BF16 || x_dtype == DUO_F16, "q8_gemm: x must be bf16 or f16");
  DUO_CHECK_ARG(k % 64 == 0 && group > 0 && group % 64 == 0 && k % group == 0,
                "q8_gemm: k and the group size multiples of 64, the group dividing k");
  DUO_CHECK_ARG(valid_act(y_dtype), "q8_gemm: y dtype must be f32, bf16 or f16");
  DUO_CHECK_ARG(m == 0 || n == 0 || (x && q && s && y), "q8_gemm: null pointer");
  DUO_CHECK_ARG(!accumulate || y_dtype == DUO_F32, "q8_gemm: accumulate needs an f32 y");
  DUO_CHECK_ARG(!swiglu || (n % 128 == 0 && y_dtype == x_dtype && !accumulate),
                "q8_gemm: SwiGLU needs n a multiple of 128 and y in x's dtype");
  DUO_CHECK_ARG(ldy >= (swiglu ? n / 2 : n), "q8_gemm: ldy too small");
  GemmEpiArgs ep;
  ep.epi = swiglu ? EPI_SWIGLU : accumulate ? EPI_ADD_F32 : EPI_STORE;
  ep.c = y;
  ep.c_dtype = y_dtype;
  ep.ldc = ldy;
  if (group == k) ep.colscale = s;  // one scale per row: the epilogue's column scale
  if (swiglu) ep.cs_inter = n / 2;
  return launch_gemm_dec_q8(x, m, k, q, s, group, swiglu ? n / 2 : 0, n, x_dtype, ep, as_stream(stream));
}

extern "C" int duo_gemm_swiglu(const void* a, int m, int k, const void* b, int inter, int ab_dtype,
                               const float* col_scale, void* out, int ldo, const int32_t* push_neurons,
                               const int32_t* push_modes, const float* push_vals, int push_count, int push_rows, int t,
                               int row_base, duo_stream stream) {
  DUO_CHECK_ARG(m >= 0 && inter >= 0 && k > 0 && t > 0 && row_base >= 0, "gemm_swiglu: bad shape");
  DUO_CHECK_ARG(k % 64 == 0 && inter % 64 == 0, "gemm_swiglu: k and inter must be multiples of 64");
  DUO_CHECK_ARG(ab_dtype == DUO_BF16 || ab_dtype == DUO_F16, "gemm_swiglu: operands must be bf16 or f16");
  DUO_CHECK_ARG(m == 0 || inter == 0 || (a && b && out), "gemm_swiglu: null pointer");
  DUO_CHECK_ARG(ldo >= inter, "gemm_swiglu: ldo < inter");
  DUO_CHECK_ARG(push_count >= 0 && (push_count == 0 || (push_neurons && push_modes && push_vals)),
                "gemm_swiglu: null push table");
  DUO_CHECK_ARG(push_count <= 32, "gemm_swiglu: at most 32 push records");
  DUO_CHECK_ARG(push_count == 0 || row_base + (m > 0 ? (m - 1) / t : 0) < push_rows,
                "gemm_swiglu: rows beyond the push table");
  GemmEpiArgs ep;
  ep.epi = EPI_SWIGLU;
  ep.c = out;
  ep.c_dtype = ab_dtype;
  ep.ldc = ldo;
  ep.colscale = col_scale;
  ep.t = t;
  ep.row_base = row_base;
  ep.push = PushTable{push_neurons, push_modes, push_vals, push_count, push_rows};
  return launch_gemm_tc(a, m, k, b, 2 * inter, ab_dtype, ep, as_stream(stream));
}

