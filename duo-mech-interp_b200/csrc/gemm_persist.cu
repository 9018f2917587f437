// Persistent tcgen05 GEMM for the large projections (prefill, lm_head): one CTA per SM walks the 128 x BN output tiles
// t = blockIdx.x, blockIdx.x + gridDim.x, ...  The TMA ring runs continuously across tile boundaries and the
// accumulator is double-buffered in TMEM (2 x BN columns), so the MMA of tile i + 1 proceeds while the epilogue warps
// drain tile i: a CTA pays the pipeline fill once and no epilogue sits on the critical path.
//
// Warp 0: TMA producer (one lane).  Warp 1: TMEM allocator and MMA issuer (one lane).  Warps 2-5: epilogue; warp w
// owns accumulator rows 32 (w % 4) .. + 31 (its TMEM lane quarter) and moves them out 32 columns at a time through a
// 32 x 36 float transpose buffer of its own, so each global row segment is written (and, for the residual add, read)
// by consecutive lanes with 16-byte accesses.
//
// The arithmetic is that of gemm.cu's tile kernel (the reference's matmul, engine/kernels.js:55-151, f32 accumulate
// over bf16 / f16 operands) with the same three epilogues.
#include "kernels.cuh"
#include "tc.cuh"

namespace duo {

namespace {

// PEPI_PITCH: transpose-buffer row pitch in floats; 36 keeps rows 16-byte aligned and float4 accesses conflict-free
constexpr int PBM = 128, PBK = 64, PTHREADS = 192, PEPI_PITCH = 36;

template <int BN> struct PCfg {
  static constexpr int A_BYTES = PBM * PBK * 2;
  static constexpr int B_BYTES = BN * PBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES;
  static constexpr int EPI_BYTES = 4 * 32 * PEPI_PITCH * 4;
  static constexpr int BAR_OFF = STAGES * STAGE_BYTES + EPI_BYTES;
  static constexpr int SMEM = 1024 /*align*/ + BAR_OFF + 256 /*barriers*/;
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(2 * BN <= 512, "two accumulators must fit in TMEM");
};

// Bounded wait that also gives up once another role of the CTA has flagged an abort.
__device__ __forceinline__ bool pwait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (tc::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = tc::globaltimer_ns();
  for (uint32_t i = 1;; i++) {
    if (tc::mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (*abort) return false;
      if (tc::globaltimer_ns() - t0 > 2000000000ull) {
        *abort = 1;
        return false;
      }
    }
  }
}

__device__ __forceinline__ void store2(void* c, int dtype, long off, float x0, float x1, bool pair) {
  if (dtype == DUO_BF16) {
    __nv_bfloat16* C = static_cast<__nv_bfloat16*>(c) + off;
    if (pair) *reinterpret_cast<__nv_bfloat162*>(C) = __floats2bfloat162_rn(x0, x1);
    else C[0] = __float2bfloat16_rn(x0);
  } else {
    __half* C = static_cast<__half*>(c) + off;
    if (pair) *reinterpret_cast<__half2*>(C) = __floats2half2_rn(x0, x1);
    else C[0] = __float2half_rn(x0);
  }
}

template <int BN, int EPI, bool F16>
__global__ void __launch_bounds__(PTHREADS, 1)
    gemm_persist_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b, int M,
                        int N, int K, int m_fast, GemmEpiArgs ep, unsigned* fault) {
  using C = PCfg<BN>;
  if (tc::fault_pending(fault)) {  // an earlier kernel gave up a wait
    pdl_wait();
    return;
  }
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + C::STAGES * C::A_BYTES;
  float* epi = reinterpret_cast<float*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (N + BN - 1) / BN, m_tiles = (M + PBM - 1) / PBM;
  const int tiles = n_tiles * m_tiles;
  const int num_k = K / PBK;
  // tile t -> (m tile, n tile).  Consecutive tiles share the larger operand's panel so that, with the whole grid
  // working on neighbouring tiles, it streams from HBM once: n fastest when A is the larger (prefill projections keep
  // all of B in L2), m fastest when B is (the LM head reads its 250k-row weight once for every m tile).
  auto tile_mn = [&](int t, int& tm, int& tn) {
    if (m_fast) { tm = (t % m_tiles) * PBM; tn = (t / m_tiles) * BN; }
    else { tm = (t / n_tiles) * PBM; tn = (t % n_tiles) * BN; }
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; s++) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      tc::mbar_init(&acc_full[b], 1);
      tc::mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    *abort = 0;
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tma_a);
    tc::prefetch_tmap(&tma_b);
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 2 * BN);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  // Programmatic launch: constant weight tiles of the first tile's first stages stream in while the preceding kernel
  // finishes; everything else waits for it.
  const int pre = ep.b_const ? min(num_k, C::STAGES) : 0;
  if (warp == 0 && lane == 0 && pre > 0) {
    int tile_m, tile_n;
    tile_mn(blockIdx.x, tile_m, tile_n);
    for (int kb = 0; kb < pre; kb++) {
      tc::mbar_arrive_expect_tx(&full[kb], C::STAGE_BYTES);
      tc::tma_load_2d(sb + kb * C::B_BYTES, &tma_b, kb * PBK, tile_n, &full[kb]);
    }
  }
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      long fill = 0;
      for (int t = blockIdx.x; t < tiles && !*abort; t += gridDim.x) {
        int tile_m, tile_n;
        tile_mn(t, tile_m, tile_n);
        for (int kb = 0; kb < num_k; kb++, fill++) {
          const int s = (int)(fill % C::STAGES);
          const uint32_t ph = (uint32_t)((fill / C::STAGES) & 1);
          if (fill < pre) {  // its B tile is already on the way
            tc::tma_load_2d(sa + s * C::A_BYTES, &tma_a, kb * PBK, tile_m, &full[s]);
            continue;
          }
          if (fill >= C::STAGES && !pwait(&empty[s], ph ^ 1, abort)) {
            atomicOr(fault, 1u);
            break;
          }
          tc::mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
          tc::tma_load_2d(sa + s * C::A_BYTES, &tma_a, kb * PBK, tile_m, &full[s]);
          tc::tma_load_2d(sb + s * C::B_BYTES, &tma_b, kb * PBK, tile_n, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_16_f32(PBM, BN, F16);
      const uint64_t da0 = tc::desc_kmajor_sw128(tc::smem_u32(sa)), db0 = tc::desc_kmajor_sw128(tc::smem_u32(sb));
      long use = 0;
      int it = 0;
      for (int t = blockIdx.x; t < tiles && !*abort; t += gridDim.x, it++) {
        const int b = it & 1;
        const uint32_t round = (uint32_t)(it >> 1);  // earlier uses of accumulator b
        if (round > 0 && !pwait(&acc_empty[b], (round - 1) & 1, abort)) {
          atomicOr(fault, 8u);
          break;
        }
        tc::fence_after_sync();
        const uint32_t acc = tmem + b * BN;
        bool ok = true;
        for (int kb = 0; kb < num_k; kb++, use++) {
          const int s = (int)(use % C::STAGES);
          const uint32_t ph = (uint32_t)((use / C::STAGES) & 1);
          if (!pwait(&full[s], ph, abort)) {
            atomicOr(fault, 2u);
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint64_t da = tc::desc_add(da0, s * C::A_BYTES), db = tc::desc_add(db0, s * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < PBK / 16; k++)  // 16 k = 32 bytes along the swizzled rows
            tc::mma_bf16(acc, tc::desc_add(da, 32 * k), tc::desc_add(db, 32 * k), idesc, (kb | k) != 0);
          tc::mma_commit(&empty[s]);
        }
        if (!ok) break;
        tc::mma_commit(&acc_full[b]);
      }
    }
  } else {
    constexpr int NC = (EPI == EPI_SWIGLU) ? BN / 2 : BN;  // output columns per tile
    const int quad = warp & 3;
    float* wb = epi + (warp - 2) * 32 * PEPI_PITCH;
    const int ncols = (EPI == EPI_SWIGLU) ? N / 2 : N;
    const bool f32_out = EPI == EPI_ADD_F32 || ep.c_dtype == DUO_F32;
    // 16-byte global accesses need a 16-byte aligned base and rows a multiple of 16 bytes apart
    const bool v16 = (reinterpret_cast<uintptr_t>(ep.c) & 15) == 0 && ep.ldc % (f32_out ? 4 : 8) == 0 &&
                     (ep.vec == nullptr || (reinterpret_cast<uintptr_t>(ep.vec) & 15) == 0);
    int it = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, it++) {
      const int b = it & 1;
      int tile_m, tile_n;
      tile_mn(t, tile_m, tile_n);
      const int row0 = tile_m + quad * 32;
      // fused RMSNorm (consumer): the factor rsqrt(mean x^2 + eps) of this thread's accumulator row, from the
      // producer's per-block partials, requested before the accumulator wait
      float rrow = 1.f;
      if (EPI != EPI_ADD_F32 && EPI != EPI_ARGMAX && ep.row_part && row0 + lane < M) {
        float sum = 0.f;
        for (int q = 0; q < ep.row_blocks; q++) sum += ep.row_part[(long)(row0 + lane) * ep.row_blocks + q];
        rrow = rsqrtf(sum / (float)ep.row_d + ep.row_eps);
      }
      if (!pwait(&acc_full[b], (uint32_t)((it >> 1) & 1), abort)) {
        if (lane == 0) atomicOr(fault, 4u);
        break;
      }
      tc::fence_after_sync();
      const uint32_t trow = tmem + b * BN + ((uint32_t)(quad * 32) << 16);
      const int n0 = (EPI == EPI_SWIGLU) ? tile_n / 2 : tile_n;
      if (EPI == EPI_ARGMAX) {
        // thread = row: scan its BN columns in ascending order, keeping the first maximum
        float best = -INFINITY;
        int bidx = 0x7fffffff;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t r0[32];
          tc::tmem_ld32_issue(trow + c0, r0);
          // column scales of the chunk: one coalesced load (lane j holds column c0 + j), broadcast by shuffles
          const float csl = ep.colscale ? (tile_n + c0 + lane < N ? ep.colscale[tile_n + c0 + lane] : 0.f) : 1.f;
          tc::tmem_ld_wait(r0);
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const int n = tile_n + c0 + j;
            float x = __uint_as_float(r0[j]);
            if (ep.colscale) x *= __shfl_sync(0xffffffffu, csl, j);
            if (n < N && x > best) {
              best = x;
              bidx = n;
            }
          }
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&acc_empty[b]);
        const int m = row0 + lane;
        if (m < M) {
          static_cast<float*>(ep.c)[(long)m * ep.ldc + tile_n / BN] = best;
          ep.idx[(long)m * ep.ldc + tile_n / BN] = bidx;
        }
        continue;
      }
      float rowss[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // fused RMSNorm (producer): rows s8 * 4 + lane / 8
#pragma unroll 1
      for (int c0 = 0; c0 < NC; c0 += 32) {
        // (1) 32 accumulator columns of this thread's row -> scaled (SwiGLU: combined) values -> the transpose buffer
        float v[32];
        {
          uint32_t r0[32];
          if (EPI == EPI_SWIGLU) {
            // 128-wide column groups [64 gate rows | the matching 64 up rows]
            const int gc = (c0 / 64) * 128 + (c0 % 64);
            uint32_t r1[32];
            tc::tmem_ld32_issue(trow + gc, r0);
            tc::tmem_ld32_issue(trow + gc + 64, r1);
            // the 32 gate and 32 up column scales, as 16-byte loads issued while the TMEM loads are in flight (a
            // ragged last tile, N % 256 == 128, ends at column N: its scales past N read as 1)
            float cg[32], cu[32];
#pragma unroll
            for (int j = 0; j < 32; j++) cg[j] = cu[j] = 1.f;
            if (ep.colscale) {
              const int c0g = tile_n + gc;
              if (c0g + 96 <= N) {
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                  const float4 a4 = *reinterpret_cast<const float4*>(ep.colscale + c0g + j);
                  const float4 b4 = *reinterpret_cast<const float4*>(ep.colscale + c0g + 64 + j);
                  cg[j] = a4.x; cg[j + 1] = a4.y; cg[j + 2] = a4.z; cg[j + 3] = a4.w;
                  cu[j] = b4.x; cu[j + 1] = b4.y; cu[j + 2] = b4.z; cu[j + 3] = b4.w;
                }
              } else {
#pragma unroll
                for (int j = 0; j < 32; j++) {
                  if (c0g + j < N) cg[j] = ep.colscale[c0g + j];
                  if (c0g + 64 + j < N) cu[j] = ep.colscale[c0g + 64 + j];
                }
              }
            }
            tc::tmem_ld_wait(r0);
            tc::tmem_ld_wait(r1);
#pragma unroll
            for (int j = 0; j < 32; j++)
              v[j] = silu16_(__uint_as_float(r0[j]) * cg[j] * rrow) * (__uint_as_float(r1[j]) * cu[j] * rrow);
          } else {
            tc::tmem_ld32_issue(trow + c0, r0);
            tc::tmem_ld_wait(r0);
#pragma unroll
            for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r0[j]) * rrow;  // column scales after the transpose
          }
        }
        if (c0 + 32 >= NC) {  // every TMEM read of this tile is done: hand the accumulator back to the MMA warp
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&acc_empty[b]);
        }
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<float4*>(wb + lane * PEPI_PITCH + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        __syncwarp();
        // (2) write the 32 x 32 block out row-contiguously
        const int nb = n0 + c0;  // first output column of the chunk
        if (f32_out) {
          // 8 lanes x 4 columns per row, 4 rows per step; every load of the residual is issued before any store
          const int cq = (lane & 7) * 4, n = nb + cq;
          // this lane's 4 column scales (store / residual add; SwiGLU values are scaled already)
          float cs4[4] = {1.f, 1.f, 1.f, 1.f};
          if (EPI != EPI_SWIGLU && ep.colscale) {
#pragma unroll
            for (int i = 0; i < 4; i++) cs4[i] = n + i < ncols ? ep.colscale[n + i] : 0.f;
          }
          float4 old[8], add[8], nw4 = make_float4(0.f, 0.f, 0.f, 0.f);
          const unsigned pm = (EPI == EPI_SWIGLU && ep.push.count) ? push_mask(ep.push, n, 4) : 0u;
          if (EPI == EPI_ADD_F32 && ep.nrm_out) nw4 = *reinterpret_cast<const float4*>(ep.nrm_w + n);
#pragma unroll
          for (int s8 = 0; s8 < 8; s8++) {
            const int m = row0 + s8 * 4 + (lane >> 3);
            old[s8] = add[s8] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (m < M && n < ncols) {
              const long off = (long)m * ep.ldc + n;
              const float* vr = (EPI == EPI_ADD_F32 && ep.vec)
                                    ? ep.vec + (long)(ep.row_base + m / ep.t) * ep.ldc + n : nullptr;
              if (v16 && n + 4 <= ncols) {
                if (EPI == EPI_ADD_F32) old[s8] = *reinterpret_cast<const float4*>(static_cast<float*>(ep.c) + off);
                if (vr) add[s8] = *reinterpret_cast<const float4*>(vr);
              } else {
                float o[4] = {0, 0, 0, 0}, a4[4] = {0, 0, 0, 0};
                for (int i = 0; i < 4 && n + i < ncols; i++) {
                  if (EPI == EPI_ADD_F32) o[i] = static_cast<float*>(ep.c)[off + i];
                  if (vr) a4[i] = vr[i];
                }
                old[s8] = make_float4(o[0], o[1], o[2], o[3]);
                add[s8] = make_float4(a4[0], a4[1], a4[2], a4[3]);
              }
            }
          }
#pragma unroll
          for (int s8 = 0; s8 < 8; s8++) {
            const int row = s8 * 4 + (lane >> 3);
            const int m = row0 + row;
            if (m >= M || n >= ncols) continue;
            float4 x = *reinterpret_cast<const float4*>(wb + row * PEPI_PITCH + cq);
            x.x *= cs4[0]; x.y *= cs4[1]; x.z *= cs4[2]; x.w *= cs4[3];
            float o[4] = {old[s8].x + x.x + add[s8].x, old[s8].y + x.y + add[s8].y, old[s8].z + x.z + add[s8].z,
                          old[s8].w + x.w + add[s8].w};
            if (EPI == EPI_SWIGLU && pm) {
              const int r = ep.row_base + m / ep.t;
              for (int i = 0; i < 4; i++) o[i] = push_apply_masked(ep.push, pm, r, n + i, o[i]);
            }
            float* X = static_cast<float*>(ep.c) + (long)m * ep.ldc + n;
            if (v16 && n + 4 <= ncols) *reinterpret_cast<float4*>(X) = make_float4(o[0], o[1], o[2], o[3]);
            else for (int i = 0; i < 4 && n + i < ncols; i++) X[i] = o[i];
            if (EPI == EPI_ADD_F32 && ep.nrm_out) {  // the next norm's weighted input (host: N % 256 == 0, aligned)
              const float y[4] = {o[0] * (1.f + nw4.x), o[1] * (1.f + nw4.y), o[2] * (1.f + nw4.z), o[3] * (1.f + nw4.w)};
              uint32_t w2[2];
#pragma unroll
              for (int i = 0; i < 2; i++) {
                if (F16) {
                  const __half2 h = __floats2half2_rn(y[2 * i], y[2 * i + 1]);
                  w2[i] = *reinterpret_cast<const uint32_t*>(&h);
                } else {
                  const __nv_bfloat162 h = __floats2bfloat162_rn(y[2 * i], y[2 * i + 1]);
                  w2[i] = *reinterpret_cast<const uint32_t*>(&h);
                }
              }
              *reinterpret_cast<uint2*>(static_cast<uint8_t*>(ep.nrm_out) + ((long)m * ep.ldc + n) * 2) =
                  make_uint2(w2[0], w2[1]);
              rowss[s8] += o[0] * o[0] + o[1] * o[1] + o[2] * o[2] + o[3] * o[3];
            }
          }
        } else {
          // 16-bit output: 4 lanes x 8 columns (16 bytes) per row, 8 rows per step
          const int c8 = (lane & 3) * 8, n = nb + c8;
          // this lane's 8 column scales (store; SwiGLU values are scaled already)
          float cs8[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
          const unsigned pm = (EPI == EPI_SWIGLU && ep.push.count) ? push_mask(ep.push, n, 8) : 0u;
          if (EPI != EPI_SWIGLU && ep.colscale) {
#pragma unroll
            for (int i = 0; i < 8; i++) cs8[i] = n + i < ncols ? ep.colscale[n + i] : 0.f;
          }
#pragma unroll
          for (int s4 = 0; s4 < 4; s4++) {
            const int row = s4 * 8 + (lane >> 2);
            const int m = row0 + row;
            if (m >= M || n >= ncols) continue;
            const float4 lo = *reinterpret_cast<const float4*>(wb + row * PEPI_PITCH + c8);
            const float4 hi = *reinterpret_cast<const float4*>(wb + row * PEPI_PITCH + c8 + 4);
            float x[8] = {lo.x * cs8[0], lo.y * cs8[1], lo.z * cs8[2], lo.w * cs8[3],
                          hi.x * cs8[4], hi.y * cs8[5], hi.z * cs8[6], hi.w * cs8[7]};
            if (EPI == EPI_SWIGLU && pm) {
              const int r = ep.row_base + m / ep.t;
              for (int i = 0; i < 8 && n + i < ncols; i++) x[i] = push_apply_masked(ep.push, pm, r, n + i, x[i]);
            }
            const long off = (long)m * ep.ldc + n;
            if (v16 && n + 8 <= ncols) {
              uint32_t w[4];
#pragma unroll
              for (int i = 0; i < 4; i++) {
                if (ep.c_dtype == DUO_BF16) {
                  const __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
                  w[i] = *reinterpret_cast<const uint32_t*>(&h);
                } else {
                  const __half2 h = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
                  w[i] = *reinterpret_cast<const uint32_t*>(&h);
                }
              }
              *reinterpret_cast<uint4*>(static_cast<uint8_t*>(ep.c) + off * 2) = make_uint4(w[0], w[1], w[2], w[3]);
            } else {
              for (int i = 0; i < 8 && n + i < ncols; i++) store2(ep.c, ep.c_dtype, off + i, x[i], 0.f, false);
            }
          }
        }
        __syncwarp();  // wb is rewritten by the next chunk
      }
      if (EPI == EPI_ADD_F32 && ep.nrm_out) {
        // the 8 lanes of a row hold its 4-column pieces: sum them, then one lane per row writes the tile's partial
#pragma unroll
        for (int s8 = 0; s8 < 8; s8++) {
          float v = rowss[s8];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          v += __shfl_xor_sync(0xffffffffu, v, 4);
          const int m = row0 + s8 * 4 + (lane >> 3);
          if ((lane & 7) == 0 && m < M) ep.nrm_part[(long)m * (N / BN) + tile_n / BN] = v;
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, 2 * BN);
  }
}

template <int BN, int EPI, bool F16>
int run_persist(const CUtensorMap& ta, const CUtensorMap& tb, int m, int n, int k, const GemmEpiArgs& ep,
                cudaStream_t st) {
  using C = PCfg<BN>;
  DUO_TRY(ensure_smem_attr(gemm_persist_kernel<BN, EPI, F16>, C::SMEM));
  unsigned* fault = tc_fault_ptr();
  if (!fault) return fail(DUO_ECUDA, "tensor-core fault word is not addressable");
  const long tiles = (long)cdiv(n, BN) * cdiv(m, PBM);
  const int grid = (int)std::min<long>(tiles, sm_count());
  const int m_fast = (long)m > (long)n ? 0 : 1;  // same element size: A is the larger operand iff m > n
  DUO_CUDA_TRY(::duo::launch_kernel(gemm_persist_kernel<BN, EPI, F16>, grid, PTHREADS, C::SMEM, st, ta, tb, m, n, k,
                                    m_fast, ep, fault));
  DUO_LAUNCH_CHECK("gemm_persist_kernel");
  return DUO_OK;
}

template <bool F16>
int dispatch_persist(const CUtensorMap& ta, const CUtensorMap& tb, int m, int n, int k, const GemmEpiArgs& ep,
                     cudaStream_t st) {
  if (ep.epi == EPI_ARGMAX) return run_persist<256, EPI_ARGMAX, F16>(ta, tb, m, n, k, ep, st);
  if (ep.epi == EPI_SWIGLU) return run_persist<256, EPI_SWIGLU, F16>(ta, tb, m, n, k, ep, st);
  if (ep.epi == EPI_ADD_F32) return run_persist<256, EPI_ADD_F32, F16>(ta, tb, m, n, k, ep, st);
  return run_persist<256, EPI_STORE, F16>(ta, tb, m, n, k, ep, st);
}

// out[row] = column of the largest partial (lowest column among equal maxima); 0 if no column beat -inf
__global__ void __launch_bounds__(256) argmax_partials_kernel(const float* __restrict__ pv,
                                                              const int32_t* __restrict__ pi, int m, int parts,
                                                              int32_t* __restrict__ out) {
  pdl_enter();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= m) return;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int p = lane; p < parts; p += 32) {
    const float v = pv[(long)row * parts + p];
    const int i = pi[(long)row * parts + p];
    if (v > best || (v == best && i < idx)) { best = v; idx = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
  }
  if (lane == 0) out[row] = idx == 0x7fffffff ? 0 : idx;
}

}  // namespace

int launch_lm_argmax(const void* a, int m, int k, const void* b, int n, int ab_dtype, const float* colscale,
                     bool b_const, float* scratch, int32_t* out, cudaStream_t st) {
  if (m == 0) return DUO_OK;
  DUO_CHECK_ARG(k % PBK == 0 && n > 0, "lm_argmax: k must be a multiple of 64");
  DUO_CHECK_ARG(ab_dtype == DUO_BF16 || ab_dtype == DUO_F16, "lm_argmax: operands must be bf16 or f16");
  const int parts = cdiv(n, 256);
  CUtensorMap ta, tb;
  DUO_TRY(make_tmap_16(&ta, a, ab_dtype, m, k, k, PBM, PBK));
  DUO_TRY(make_tmap_16(&tb, b, ab_dtype, n, k, k, 256, PBK));
  GemmEpiArgs ep;
  ep.epi = EPI_ARGMAX;
  ep.c = scratch;
  ep.c_dtype = DUO_F32;
  ep.ldc = parts;
  ep.colscale = colscale;
  ep.idx = reinterpret_cast<int32_t*>(scratch + (long)m * parts);
  ep.b_const = b_const;
  DUO_TRY(launch_gemm_persist(ta, tb, 256, m, n, k, ab_dtype, ep, st));
  DUO_CUDA_TRY(::duo::launch_kernel(argmax_partials_kernel, cdiv(m, 8), 256, 0, st, scratch, ep.idx, m, parts, out));
  DUO_LAUNCH_CHECK("argmax_partials_kernel");
  return DUO_OK;
}

// A [m, k] and B [n, k] are described by `ta` (box 128 x 64) and `tb` (box 256 x 64).
int launch_gemm_persist(const CUtensorMap& ta, const CUtensorMap& tb, int bn, int m, int n, int k, int ab_dtype,
                        const GemmEpiArgs& ep, cudaStream_t st) {
  DUO_CHECK_ARG(bn == 256, "gemm_persist: tile width must be 256");
  return ab_dtype == DUO_F16 ? dispatch_persist<true>(ta, tb, m, n, k, ep, st)
                             : dispatch_persist<false>(ta, tb, m, n, k, ep, st);
}

}  // namespace duo
