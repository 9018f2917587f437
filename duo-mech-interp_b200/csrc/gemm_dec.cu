// Decode-sized tcgen05 GEMM (M <= 256 rows): C[m, n] = sum_k X[m, k] W[n, k] with the weights on the MMA's M side.
//
// With few rows the cost of a GEMM is streaming the weights once and getting every SM to work on them.  A CTA owns
// 128 weight rows (MMA M = 128) and a group of NB = 64 or 128 X rows (MMA N = NB; rows past M read as zeros), so
// grid = (weight blocks, row groups, K slices).  Wide outputs (the in-projections, gate|up) fill the SMs with the
// first two dimensions and need no K split; narrow ones (N = 1024, long K) split K over a thread-block cluster of
// KS <= 8 CTAs (grid z = cluster rank).
//
// Epilogues.  Without a K split the accumulator goes TMEM -> registers -> (colscale, SwiGLU + pushes, 16-bit or f32
// convert) -> a dense shared-memory tile -> one TMA store, so the tile leaves the SM as whole rows.  With a K split,
// or for the residual add, each CTA drains its raw f32 partial into shared memory (m-major); after a cluster barrier
// CTA z takes rows [z R, z R + R) of the group (R = NB / KS), sums the KS partials over distributed shared memory in
// rank order (deterministic) and runs the epilogue with consecutive lanes on consecutive weight rows n, i.e.
// coalesced along the output row: store, SwiGLU (+ pushes; gate / up packs interleaved per 64 rows) or
// X += acc * colscale (+ vec).
//
// int8 weights (Q8).  The weight tile can also arrive as the int8 matrix itself (half the bytes of the 16-bit pack):
// TMA brings 128 rows x 64 int8 per stage, four converter warps turn it into the 16-bit tile of the MMA's A operand
// (the 128-byte swizzled K-major layout TMA would have written) in one of two converted slots, and the MMA reads it
// from there.  With group scales (G < K) the converted value is 16-bit(f32(q) * s), the exact value of the 16-bit
// pack; with one scale per row it is q itself (exact) and the scale is the epilogue's colscale, as for the pack.  So
// both forms feed the tensor core identical operands and give identical results.
//
// The arithmetic is the reference's matmul (engine/kernels.js:97-151): f32 accumulation of products of the 16-bit
// operands; the per-row int8 scale (colscale) multiplies the reduced sum.
#include <cooperative_groups.h>

#include <algorithm>
#include <cstring>

#include "kernels.cuh"
#include "tc.cuh"

namespace cg = cooperative_groups;

namespace duo {

namespace {

constexpr int DBM = 128, DBK = 64, DTHREADS = 256, DP = DBM + 4;  // DP: partial-tile row pitch (floats)
constexpr int kQ8Groups = 8;  // group scales of one CTA's K slice held in shared memory (per weight row)

// Shared memory: [16-bit weight tiles: one per stage, or (Q8) CV converted slots | X tiles | (Q8) int8 weight tiles |
// (Q8) group scales | barriers].  A stage is what one TMA transaction brings: the weight tile (16-bit or int8) and the
// X tile.
template <int NB, bool Q8> struct DCfg {
  static constexpr int W_BYTES = DBM * DBK * 2;         // 16-bit weight tile (the MMA's A operand)
  static constexpr int RAW_BYTES = Q8 ? DBM * DBK : 0;  // int8 weight tile as loaded
  static constexpr int X_BYTES = NB * DBK * 2;
  static constexpr int CV = Q8 ? 3 : 0;                 // converted slots
  static constexpr int CVN = Q8 ? CV : 1;               // CV as a divisor
  static constexpr int SCALE_BYTES = Q8 ? DBM * kQ8Groups * 4 : 0;
  static constexpr int STAGE_BYTES = (Q8 ? RAW_BYTES : W_BYTES) + X_BYTES;
  static constexpr int BUDGET = Q8 ? 221 * 1024 : 200 * 1024;
  static constexpr int STAGES = (BUDGET - CV * W_BYTES - SCALE_BYTES) / STAGE_BYTES;
  static constexpr int RING = CV * W_BYTES + STAGES * STAGE_BYTES;
  static constexpr int BARS = (2 * STAGES + 2 * CV + 1) * 8 + 8;
  static constexpr int SMEM = 1024 + RING + SCALE_BYTES + BARS;
  static constexpr int OUT_OFF = (NB * DP * 4 + 1023) / 1024 * 1024;  // SwiGLU output tile, after the partial
  static_assert(OUT_OFF + NB * 64 * 2 <= RING, "the partial and SwiGLU tiles must fit in the ring");
  static_assert(NB * DBM * 4 <= RING, "the f32 output tile must fit in the ring");
  static_assert(SMEM + NB * 4 <= 227 * 1024, "shared memory (with the static row factors)");
};

// int8 weight operand (Q8 kernels)
struct Q8Args {
  const float* s = nullptr;  // scales [n][k / group], rows in the int8 matrix's order
  int group = 0;             // group size, a multiple of 64 (= k: one scale per row, applied as the colscale)
  int ngroups = 0;           // k / group
  int inter = 0;             // > 0: SwiGLU weights [gate (inter rows) | up (inter rows)], block b = gate rows
                             // 64 b .. 64 b + 63 then up rows inter + 64 b .., the 16-bit pack's interleave
  int apply = 0;             // group scales multiplied into the converted operand (group < k)
};

template <bool F16> __device__ __forceinline__ uint32_t pack2_16(float a, float b) {
  if (F16) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <typename T> __device__ __forceinline__ T cvt16(float v);
template <> __device__ __forceinline__ __nv_bfloat16 cvt16<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half cvt16<__half>(float v) { return __float2half_rn(v); }

template <int NB, int EPI, bool F16, bool Q8>
__global__ void __launch_bounds__(DTHREADS, 1)
    gemm_dec_kernel(const __grid_constant__ CUtensorMap tma_w, const __grid_constant__ CUtensorMap tma_x,
                    const __grid_constant__ CUtensorMap tma_c, int M, int N, int K, int kper, int direct,
                    GemmEpiArgs ep, Q8Args qa, unsigned* fault) {
  using C = DCfg<NB, Q8>;
  constexpr int CW = NB / 2;  // accumulator columns (X rows) drained per warp
  if (gridDim.z == 1 && tc::fault_pending(fault)) {  // an earlier kernel gave up a wait (no cluster when z == 1)
    pdl_wait();
    return;
  }
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sw = smem;
  uint8_t* sx = smem + (Q8 ? C::CV : C::STAGES) * C::W_BYTES;
  uint8_t* sraw = sx + C::STAGES * C::X_BYTES;                    // Q8: int8 weight tiles
  float* scl = reinterpret_cast<float*>(smem + C::RING);          // Q8: group scales [DBM rows][kQ8Groups]
  float* part = reinterpret_cast<float*>(smem);  // epilogue tiles reuse the ring once every MMA has completed
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::RING + C::SCALE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* cfull = empty + C::STAGES;  // Q8: converted slot written (6 converter warps)
  uint64_t* cempty = cfull + C::CV;     // Q8: converted slot read by the MMAs
  uint64_t* tmem_full = cempty + C::CV;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * DBM, m0 = blockIdx.y * NB;
  const int ks = gridDim.z, z = blockIdx.z;
  const int kb0 = z * kper;
  const int num_k = max(0, min(kper, K / DBK - kb0));

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; s++) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int c = 0; c < C::CV; c++) {
      tc::mbar_init(&cfull[c], 6);
      tc::mbar_init(&cempty[c], 1);
    }
    tc::mbar_init(tmem_full, 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tma_w);
    tc::prefetch_tmap(&tma_x);
    if (direct) tc::prefetch_tmap(&tma_c);
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, NB);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  // The weight slice is requested in full at once: the first ring stages by TMA loads, the rest as L2 prefetches,
  // so HBM latency is paid about once rather than once per ring turn.  Programmatic launch: constant weights are
  // requested while the preceding kernel finishes.
  const int pre = ep.b_const ? min(num_k, C::STAGES) : 0;
  // the weight tile of K block kb into stage s (Q8 SwiGLU: the gate and up halves of the block, 64 rows each)
  auto load_w = [&](int kb, int s, uint64_t* bar) {
    const int kx = (kb0 + kb) * DBK;
    if (!Q8) {
      tc::tma_load_2d(sw + s * C::W_BYTES, &tma_w, kx, n0, bar);
    } else if (qa.inter > 0) {
      tc::tma_load_2d(sraw + s * C::RAW_BYTES, &tma_w, kx, blockIdx.x * 64, bar);
      tc::tma_load_2d(sraw + s * C::RAW_BYTES + C::RAW_BYTES / 2, &tma_w, kx, qa.inter + blockIdx.x * 64, bar);
    } else {
      tc::tma_load_2d(sraw + s * C::RAW_BYTES, &tma_w, kx, n0, bar);
    }
  };
  auto request_w = [&](int from) {
    for (int kb = from; kb < num_k; kb++) {
      if (kb < pre) {
        tc::mbar_arrive_expect_tx(&full[kb], C::STAGE_BYTES);
        load_w(kb, kb, &full[kb]);
      } else if (kb >= C::STAGES) {
        const int kx = (kb0 + kb) * DBK;
        if (Q8 && qa.inter > 0) {
          tc::tma_prefetch_2d(&tma_w, kx, blockIdx.x * 64);
          tc::tma_prefetch_2d(&tma_w, kx, qa.inter + blockIdx.x * 64);
        } else {
          tc::tma_prefetch_2d(&tma_w, kx, n0);
        }
      }
    }
  };
  if (warp == 0 && lane == 0 && ep.b_const) request_w(0);
  pdl_wait();
  pdl_trigger();
  if (warp == 0 && lane == 0 && !ep.b_const) request_w(C::STAGES);

  // Rows [r_lo, r_hi) of the group are this CTA's in the reducing epilogue.  For the residual add with at most four
  // rows per warp, each thread's residual (and vector) entries are loaded now and arrive while the mainloop runs (X
  // is written only by kernels that have completed once pdl_wait returns).
  constexpr int RB = 4;
  const int R = (NB + ks - 1) / ks;
  const int r_lo = z * R, r_hi = min(min(NB, r_lo + R), M - m0);
  const int n4 = n0 + lane * 4;
  const bool al = (reinterpret_cast<uintptr_t>(ep.c) & 15) == 0 && ep.ldc % 4 == 0 &&
                  (ep.vec == nullptr || (reinterpret_cast<uintptr_t>(ep.vec) & 15) == 0);
  const bool pre_x = EPI == EPI_ADD_F32 && R <= 8 * RB && al && n4 + 4 <= N;
  float4 xold[RB], vold[RB];
  if (pre_x) {
#pragma unroll
    for (int i = 0; i < RB; i++) {
      const int cr = r_lo + warp + 8 * i;
      if (cr < r_hi) {
        const int m = m0 + cr;
        xold[i] = *reinterpret_cast<const float4*>(static_cast<const float*>(ep.c) + (long)m * ep.ldc + n4);
        vold[i] = ep.vec ? *reinterpret_cast<const float4*>(ep.vec + (long)(ep.row_base + m / ep.t) * ep.ldc + n4)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  }
  // colscale entry of SwiGLU weight row p (interleaved order), or of the int8 matrix's row behind it (cs_inter > 0)
  auto cs_row = [&](int p) {
    if (ep.cs_inter <= 0) return p;
    const int j = p & 127;
    return j < 64 ? (p >> 7) * 64 + j : ep.cs_inter + (p >> 7) * 64 + j - 64;
  };
  // The column scales of this thread's epilogue columns, loaded now so that their latency hides under the mainloop:
  // direct path weight row n0 + (warp % 4) 32 + lane; reduce path rows n4 .. n4 + 3, or for SwiGLU the gate and up
  // rows of output columns 4 (lane % 16) .. + 3.
  float cs_d = 1.f;
  float csv[4] = {1.f, 1.f, 1.f, 1.f}, cu_[4] = {1.f, 1.f, 1.f, 1.f};
  if (ep.colscale) {
    if (direct) {
      const int nd = n0 + (warp & 3) * 32 + lane;
      cs_d = EPI == EPI_SWIGLU ? ep.colscale[cs_row(nd)] : (nd < N ? ep.colscale[nd] : 0.f);
    } else if (EPI == EPI_SWIGLU) {
      const int j4 = (lane & 15) * 4;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        csv[i] = ep.colscale[cs_row(n0 + j4 + i)];
        cu_[i] = ep.colscale[cs_row(n0 + 64 + j4 + i)];
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; i++) csv[i] = (n4 + i < N) ? ep.colscale[n4 + i] : 0.f;
    }
  }
  // fused RMSNorm of the activation rows (consumer side): rrs[c] = rsqrt(mean x^2 + eps) of row m0 + c, from the
  // producer's per-block partials, by warps 2-7 while the mainloop runs (published by the barrier after the drain)
  __shared__ float rrs[NB];
  if (ep.row_part && threadIdx.x >= 64) {
    for (int c = threadIdx.x - 64; c < NB; c += DTHREADS - 64) {
      const int m = m0 + c;
      float sum = 0.f;
      if (m < M)
        for (int b = 0; b < ep.row_blocks; b++) sum += ep.row_part[(long)m * ep.row_blocks + b];
      rrs[c] = rsqrtf(sum / (float)ep.row_d + ep.row_eps);
    }
  }

  bool ok = true;
  if (warp == 0 && lane == 0) {
    for (int kb = 0; kb < num_k; kb++) {
      const int s = kb % C::STAGES;
      const uint32_t ph = (kb / C::STAGES) & 1;
      if (kb < pre) {
        tc::tma_load_2d(sx + s * C::X_BYTES, &tma_x, (kb0 + kb) * DBK, m0, &full[s]);
        continue;
      }
      if (kb >= C::STAGES && !tc::mbar_wait(&empty[s], ph ^ 1)) {
        atomicOr(fault, 1u);
        break;
      }
      tc::mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
      load_w(kb, s, &full[s]);
      tc::tma_load_2d(sx + s * C::X_BYTES, &tma_x, (kb0 + kb) * DBK, m0, &full[s]);
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = tc::idesc_16_f32(DBM, NB, F16);
    const uint64_t dw0 = tc::desc_kmajor_sw128(tc::smem_u32(sw)), dx0 = tc::desc_kmajor_sw128(tc::smem_u32(sx));
    for (int kb = 0; kb < num_k; kb++) {
      const int s = kb % C::STAGES;
      const uint32_t ph = (kb / C::STAGES) & 1;
      const int c = Q8 ? kb % C::CVN : 0;
      if (!tc::mbar_wait(&full[s], ph) || (Q8 && !tc::mbar_wait(&cfull[c], (kb / C::CVN) & 1))) {
        atomicOr(fault, 2u);
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const uint64_t dw = tc::desc_add(dw0, (Q8 ? c : s) * C::W_BYTES), dx = tc::desc_add(dx0, s * C::X_BYTES);
#pragma unroll
      for (int k = 0; k < DBK / 16; k++)  // 16 k = 32 bytes along the swizzled rows
        tc::mma_bf16(tmem, tc::desc_add(dw, 32 * k), tc::desc_add(dx, 32 * k), idesc, (kb | k) != 0);
      tc::mma_commit(&empty[s]);
      if (Q8) tc::mma_commit(&cempty[c]);
    }
    if (ok) tc::mma_commit(tmem_full);
  } else if (Q8 && warp >= 2) {
    // converters (warps 2..7): int8 stage s -> 16-bit converted slot c.  Thread ct takes 16-byte pieces ct + 192 i
    // (row p / 4, quarter p % 4): a warp's loads cover 512 consecutive bytes and its stores the 8 chunk positions of
    // 8 rows, so neither has bank conflicts.
    constexpr int NCV = DTHREADS - 64;
    const int ct = threadIdx.x - 64;
    const int g0 = qa.apply ? kb0 * DBK / qa.group : 0;
    if (qa.apply) {
      for (int i = ct; i < DBM * kQ8Groups; i += NCV) {
        const int r = i / kQ8Groups, g = g0 + i % kQ8Groups;
        const int orow = qa.inter > 0 ? (r < 64 ? blockIdx.x * 64 + r : qa.inter + blockIdx.x * 64 + r - 64) : n0 + r;
        scl[i] = (orow < N && g < qa.ngroups) ? qa.s[(long)orow * qa.ngroups + g] : 0.f;
      }
      tc::bar_sync(1, NCV);
    }
    for (int kb = 0; kb < num_k; kb++) {
      const int s = kb % C::STAGES, c = kb % C::CVN;
      if (!tc::mbar_wait(&full[s], (kb / C::STAGES) & 1) ||
          (kb >= C::CV && !tc::mbar_wait(&cempty[c], ((kb / C::CVN) & 1) ^ 1))) {
        if (lane == 0) atomicOr(fault, 2u);
        break;
      }
      const uint8_t* raw = sraw + s * C::RAW_BYTES;
      uint8_t* dst = sw + c * C::W_BYTES;
      const int gi = qa.apply ? (kb0 + kb) * DBK / qa.group - g0 : 0;
#pragma unroll
      for (int i = 0; i < (DBM * 4 + NCV - 1) / NCV; i++) {
        const int p = ct + NCV * i, r = p >> 2, qd = p & 3;
        if (p >= DBM * 4) break;
        const uint4 u = *reinterpret_cast<const uint4*>(raw + r * DBK + qd * 16);
        float f[16];
        i8x4_to_f32(u.x, f);
        i8x4_to_f32(u.y, f + 4);
        i8x4_to_f32(u.z, f + 8);
        i8x4_to_f32(u.w, f + 12);
        uint32_t w[8];
        if (qa.apply) {
          const float sc = scl[r * kQ8Groups + gi];
#pragma unroll
          for (int j = 0; j < 16; j++) f[j] *= sc;
#pragma unroll
          for (int j = 0; j < 8; j++) w[j] = pack2_16<F16>(f[2 * j], f[2 * j + 1]);
        } else if (F16) {
#pragma unroll
          for (int j = 0; j < 8; j++) w[j] = pack2_16<true>(f[2 * j], f[2 * j + 1]);
        } else {
          // an int8 value has at most 8 significant bits: the upper half of its f32 pattern is its bf16 value
#pragma unroll
          for (int j = 0; j < 8; j++) w[j] = __byte_perm(__float_as_uint(f[2 * j]), __float_as_uint(f[2 * j + 1]), 0x7632);
        }
        uint8_t* row = dst + r * 128;
        *reinterpret_cast<uint4*>(row + (((2 * qd) ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(row + (((2 * qd + 1) ^ (r & 7)) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
      }
      tc::fence_proxy_async();  // the generic-proxy stores become visible to the tensor core's reads
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&cfull[c]);
    }
  }

  // Drain: warp w holds TMEM lane quarter q = w % 4 (weight rows nl = 32 q + lane) and accumulator columns
  // [h CW, h CW + CW), h = w / 4 (X rows m0 + c); every load of the warp is issued before the one wait.
  __syncwarp();  // warps 0 and 1 reconverge after their single-lane roles (tcgen05.ld is warp-wide)
  const int q = warp & 3, h = warp >> 2;
  const int nl = q * 32 + lane, c_lo = h * CW;
  uint32_t r[CW / 32][32];
  if (num_k > 0) {
    if (!tc::mbar_wait(tmem_full, 0)) {
      if (lane == 0) atomicOr(fault, 4u);
    }
    tc::fence_after_sync();
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c_lo;
#pragma unroll
    for (int j = 0; j < CW / 32; j++) tc::tmem_ld32_issue(trow + 32 * j, r[j]);
#pragma unroll
    for (int j = 0; j < CW / 32; j++) tc::tmem_ld_wait(r[j]);
  } else {  // an empty K slice contributes zeros
#pragma unroll
    for (int j = 0; j < CW / 32; j++)
#pragma unroll
      for (int i = 0; i < 32; i++) r[j][i] = 0u;
  }
  auto acc = [&](int c) { return __uint_as_float(r[c >> 5][c & 31]); };  // accumulator column c_lo + c
  if (ep.row_part) __syncthreads();  // rrs complete
  auto rr = [&](int c) { return ep.row_part ? rrs[c] : 1.f; };  // factor of accumulator column (row) c

  if (direct) {
    // no K split, store or SwiGLU: the output tile is assembled in shared memory and leaves by one TMA store
    if (EPI == EPI_SWIGLU) {
      // weight rows 0..63 of the block are gate rows, 64..127 the matching up rows (interleave_gate_up order): the
      // scaled accumulators go to part[c][nl], then a rolled sweep (small code: each CTA runs it once, from a cold
      // instruction cache) forms 4 outputs per step into the [NB][64] 16-bit tile that follows the partial
      const float cs = cs_d;
#pragma unroll
      for (int c = 0; c < CW; c++) part[(c_lo + c) * DP + nl] = acc(c) * cs * rr(c_lo + c);
      __syncthreads();
      uint8_t* tile = smem + C::OUT_OFF;
      // this thread's 4 output columns are the same in every iteration (DTHREADS is a multiple of 16)
      const unsigned pm = ep.push.count ? push_mask(ep.push, n0 / 2 + (threadIdx.x & 15) * 4, 4) : 0u;
#pragma unroll 1
      for (int idx = threadIdx.x; idx < NB * 16; idx += DTHREADS) {
        const int c = idx >> 4, j4 = (idx & 15) * 4, m = m0 + c;
        const float4 g = *reinterpret_cast<const float4*>(part + c * DP + j4);
        const float4 u = *reinterpret_cast<const float4*>(part + c * DP + 64 + j4);
        float o[4] = {silu16_(g.x) * u.x, silu16_(g.y) * u.y, silu16_(g.z) * u.z, silu16_(g.w) * u.w};
        if (pm && m < M) {
          const int rw = ep.row_base + m / ep.t;
#pragma unroll
          for (int i = 0; i < 4; i++) o[i] = push_apply_masked(ep.push, pm, rw, n0 / 2 + j4 + i, o[i]);
        }
        uint2 pk;
        if (F16) {
          const __half2 lo = __floats2half2_rn(o[0], o[1]), hi = __floats2half2_rn(o[2], o[3]);
          pk = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
        } else {
          const __nv_bfloat162 lo = __floats2bfloat162_rn(o[0], o[1]), hi = __floats2bfloat162_rn(o[2], o[3]);
          pk = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
        }
        *reinterpret_cast<uint2*>(tile + (c * 64 + j4) * 2) = pk;
      }
    } else {
      const float cs = cs_d;
      if (ep.c_dtype == DUO_F32) {
        float* o = reinterpret_cast<float*>(smem);
#pragma unroll
        for (int c = 0; c < CW; c++) o[(c_lo + c) * DBM + nl] = acc(c) * cs * rr(c_lo + c);
      } else if (ep.c_dtype == DUO_F16) {
        __half* o = reinterpret_cast<__half*>(smem);
#pragma unroll
        for (int c = 0; c < CW; c++) o[(c_lo + c) * DBM + nl] = cvt16<__half>(acc(c) * cs * rr(c_lo + c));
      } else {
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(smem);
#pragma unroll
        for (int c = 0; c < CW; c++) o[(c_lo + c) * DBM + nl] = cvt16<__nv_bfloat16>(acc(c) * cs * rr(c_lo + c));
      }
    }
    tc::fence_proxy_async();
    __syncthreads();
    if (threadIdx.x == 0) {
      if (EPI == EPI_SWIGLU) tc::tma_store_2d(&tma_c, smem + C::OUT_OFF, n0 / 2, m0);
      else tc::tma_store_2d(&tma_c, smem, n0, m0);
      tc::bulk_commit();
      tc::bulk_wait_read();  // the tile may be released; the grid's completion publishes the writes
    }
  } else {
    // raw partial tile -> shared memory, m-major: part[c][nl]
#pragma unroll
    for (int c = 0; c < CW; c++) part[(c_lo + c) * DP + nl] = acc(c);
    if (ks > 1) cg::this_cluster().sync();
    else __syncthreads();

    // reduce rows [r_lo, r_hi) of the group over the cluster and run the epilogue
    cg::cluster_group cluster = cg::this_cluster();
    // Every partial of a batch of RB rows is loaded (distributed shared memory, all ranks unrolled) before any result
    // is stored, so the remote-load latency is paid about once per batch rather than once per row and rank.
    auto gather = [&](const int (&cr)[RB], int col, float4 (&out)[RB]) {  // out[i] = sum over ranks of part[cr[i]][col..]
#pragma unroll
      for (int i = 0; i < RB; i++) out[i] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int qq = 0; qq < 8; qq++) {
        if (qq < ks) {
          const float* pq = ks > 1 ? cluster.map_shared_rank(part, qq) : part;
          float4 v[RB];
#pragma unroll
          for (int i = 0; i < RB; i++)
            if (cr[i] >= 0) v[i] = *reinterpret_cast<const float4*>(pq + cr[i] * DP + col);
#pragma unroll
          for (int i = 0; i < RB; i++) {
            if (cr[i] < 0) continue;
            out[i].x += v[i].x; out[i].y += v[i].y; out[i].z += v[i].z; out[i].w += v[i].w;
          }
        }
      }
    };
    auto store4_16 = [&](long off, const float* o) {  // 4 consecutive 16-bit outputs, one 8-byte store when aligned
      uint32_t w[2];
      for (int i = 0; i < 2; i++) {
        if (ep.c_dtype == DUO_BF16) {
          const __nv_bfloat162 hh = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
          w[i] = *reinterpret_cast<const uint32_t*>(&hh);
        } else {
          const __half2 hh = __floats2half2_rn(o[2 * i], o[2 * i + 1]);
          w[i] = *reinterpret_cast<const uint32_t*>(&hh);
        }
      }
      uint8_t* base = static_cast<uint8_t*>(ep.c) + off * 2;
      if ((reinterpret_cast<uintptr_t>(base) & 7) == 0) {
        *reinterpret_cast<uint2*>(base) = make_uint2(w[0], w[1]);
      } else {
        reinterpret_cast<uint32_t*>(base)[0] = w[0];
        reinterpret_cast<uint32_t*>(base)[1] = w[1];
      }
    };
    if (EPI == EPI_SWIGLU) {
      // half-warp per row: lane & 15 -> output columns 4 (lane & 15) .. + 3 of the block's 64 neurons
      const int j4 = (lane & 15) * 4;
      const int nout = n0 / 2 + j4;  // first output column
      const float* cg_ = csv;  // gate column scales (preloaded)
      const unsigned pm = ep.push.count ? push_mask(ep.push, nout, 4) : 0u;
      for (int cb = r_lo + warp * 2 + (lane >> 4); cb < r_hi; cb += 16 * RB) {
        int cr[RB];
#pragma unroll
        for (int i = 0; i < RB; i++) cr[i] = cb + 16 * i < r_hi ? cb + 16 * i : -1;
        float4 g[RB], u[RB];
        gather(cr, j4, g);
        gather(cr, 64 + j4, u);
#pragma unroll
        for (int i = 0; i < RB; i++) {
          if (cr[i] < 0) break;
          const int m = m0 + cr[i];
          const float f = rr(cr[i]);
          const float gv[4] = {g[i].x * f, g[i].y * f, g[i].z * f, g[i].w * f};
          const float uv[4] = {u[i].x * f, u[i].y * f, u[i].z * f, u[i].w * f};
          const int rw = ep.row_base + m / ep.t;
          float o[4];
#pragma unroll
          for (int c = 0; c < 4; c++) {
            o[c] = silu16_(gv[c] * cg_[c]) * (uv[c] * cu_[c]);
            if (pm) o[c] = push_apply_masked(ep.push, pm, rw, nout + c, o[c]);
          }
          store4_16((long)m * ep.ldc + nout, o);
        }
      }
    } else {
      // one row per warp step: lane -> weight rows n0 + 4 lane .. + 3
      const int n = n4;
      for (int cb = r_lo + warp; cb < r_hi && n < N; cb += 8 * RB) {
        int cr[RB];
#pragma unroll
        for (int i = 0; i < RB; i++) cr[i] = cb + 8 * i < r_hi ? cb + 8 * i : -1;
        float4 a[RB];
        gather(cr, lane * 4, a);
#pragma unroll
        for (int i = 0; i < RB; i++) {
          if (cr[i] < 0) break;
          const int m = m0 + cr[i];
          const float f = EPI == EPI_ADD_F32 ? 1.f : rr(cr[i]);
          float x[4] = {a[i].x * csv[0] * f, a[i].y * csv[1] * f, a[i].z * csv[2] * f, a[i].w * csv[3] * f};
          const long off = (long)m * ep.ldc + n;
          const bool full4 = al && n + 4 <= N;
          if (EPI == EPI_ADD_F32) {
            float* X = static_cast<float*>(ep.c) + off;
            const float* vr = ep.vec ? ep.vec + (long)(ep.row_base + m / ep.t) * ep.ldc + n : nullptr;
            float4 o = make_float4(0.f, 0.f, 0.f, 0.f);  // the new residual values (for the fused norm)
            if (pre_x) {  // one batch: i is the preload slot of this row
              o = xold[i];
              o.x += x[0]; o.y += x[1]; o.z += x[2]; o.w += x[3];
              if (ep.vec) { o.x += vold[i].x; o.y += vold[i].y; o.z += vold[i].z; o.w += vold[i].w; }
              *reinterpret_cast<float4*>(X) = o;
            } else if (full4) {
              o = *reinterpret_cast<float4*>(X);
              o.x += x[0]; o.y += x[1]; o.z += x[2]; o.w += x[3];
              if (vr) {
                const float4 v4 = *reinterpret_cast<const float4*>(vr);
                o.x += v4.x; o.y += v4.y; o.z += v4.z; o.w += v4.w;
              }
              *reinterpret_cast<float4*>(X) = o;
            } else {
              for (int c = 0; c < 4 && n + c < N; c++) X[c] += x[c] + (vr ? vr[c] : 0.f);
            }
            if (ep.nrm_out) {  // the next RMSNorm's input (host: n % 128 == 0, aligned, so every lane is in range)
              const float4 w4 = *reinterpret_cast<const float4*>(ep.nrm_w + n);
              const float y[4] = {o.x * (1.f + w4.x), o.y * (1.f + w4.y), o.z * (1.f + w4.z), o.w * (1.f + w4.w)};
              uint2 u;
              if (F16) {
                const __half2 lo = __floats2half2_rn(y[0], y[1]), hi = __floats2half2_rn(y[2], y[3]);
                u = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
              } else {
                const __nv_bfloat162 lo = __floats2bfloat162_rn(y[0], y[1]), hi = __floats2bfloat162_rn(y[2], y[3]);
                u = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
              }
              *reinterpret_cast<uint2*>(static_cast<uint8_t*>(ep.nrm_out) + off * 2) = u;
              const float ss = warp_sum(o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w);
              if (lane == 0) ep.nrm_part[(long)m * gridDim.x + blockIdx.x] = ss;
            }
          } else if (ep.c_dtype == DUO_F32) {
            float* Cp = static_cast<float*>(ep.c) + off;
            if (full4) *reinterpret_cast<float4*>(Cp) = make_float4(x[0], x[1], x[2], x[3]);
            else for (int c = 0; c < 4 && n + c < N; c++) Cp[c] = x[c];
          } else if (n + 4 <= N) {
            store4_16(off, x);
          } else {
            for (int c = 0; c < 4 && n + c < N; c++) {
              if (ep.c_dtype == DUO_BF16) static_cast<__nv_bfloat16*>(ep.c)[off + c] = __float2bfloat16_rn(x[c]);
              else static_cast<__half*>(ep.c)[off + c] = __float2half_rn(x[c]);
            }
          }
        }
      }
    }
    // no CTA leaves while a peer may still read its partial: every remote load of this CTA has returned (its value
    // was stored above), so a relaxed arrive suffices and the stores need not drain first
    if (ks > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, NB);
  }
}

template <int NB, int EPI, bool F16, bool Q8>
int run_dec(const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& tcm, int m, int n, int k, int groups,
            int ks, int kper, int direct, const GemmEpiArgs& ep, const Q8Args& qa, cudaStream_t st) {
  using C = DCfg<NB, Q8>;
  auto kern = gemm_dec_kernel<NB, EPI, F16, Q8>;
  DUO_TRY(ensure_smem_attr(kern, C::SMEM));
  unsigned* fault = tc_fault_ptr();
  if (!fault) return fail(DUO_ECUDA, "tensor-core fault word is not addressable");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cdiv(n, DBM), groups, ks);
  cfg.blockDim = dim3(DTHREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (ks > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = ks;
    na++;
  }
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    na++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  DUO_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, tw, tx, tcm, m, n, k, kper, direct, ep, qa, fault));
  DUO_LAUNCH_CHECK("gemm_dec_kernel");
  return DUO_OK;
}

template <int NB, bool F16, bool Q8>
int dispatch_dec(const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& tcm, int m, int n, int k,
                 int groups, int ks, int kper, int direct, const GemmEpiArgs& ep, const Q8Args& qa, cudaStream_t st) {
  if (ep.epi == EPI_SWIGLU)
    return run_dec<NB, EPI_SWIGLU, F16, Q8>(tw, tx, tcm, m, n, k, groups, ks, kper, direct, ep, qa, st);
  if (ep.epi == EPI_ADD_F32)
    return run_dec<NB, EPI_ADD_F32, F16, Q8>(tw, tx, tcm, m, n, k, groups, ks, kper, direct, ep, qa, st);
  return run_dec<NB, EPI_STORE, F16, Q8>(tw, tx, tcm, m, n, k, groups, ks, kper, direct, ep, qa, st);
}

// Clusters of ks CTAs of the kernel that can be resident at once (one CTA per SM; a cluster must fit in one GPC).
// The resources are those of every epilogue and operand type, so one instantiation answers for all.
template <int NB> int max_clusters(int ks) {
  static int cache[9] = {};
  if (ks <= 1) return sm_count();
  if (cache[ks]) return cache[ks];
  auto kern = gemm_dec_kernel<NB, EPI_STORE, false, false>;
  int n = 0;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, DCfg<NB, false>::SMEM) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, ks);
    cfg.blockDim = dim3(DTHREADS);
    cfg.dynamicSmemBytes = DCfg<NB, false>::SMEM;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 1;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = ks;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
  }
  (void)cudaGetLastError();
  if (n <= 0) n = sm_count() / ks;
  cache[ks] = n;
  return n;
}

// Launch plan: row-group size nb and K split ks, chosen to minimise waves x (a fixed cost per wave + the bytes each
// CTA pulls in: its weight and X slices, plus the partials it reads back over the cluster).  The fixed cost (launch,
// first-load latency, epilogue: ~4 us) is counted as the bytes a CTA streams in that time (~90 GB/s per SM when
// every SM streams).
constexpr double kWaveBytes = 360e3;
struct DecPlan {
  int nb = 0, groups = 0, ks = 1, kper = 0;
  double cost = 0.0;
};
template <int NB> void plan_dec(int m, int n, int num_k, bool q8, int max_kper, DecPlan& best) {
  const long sms = sm_count();
  const int groups = cdiv(m, NB);
  const long base = (long)cdiv(n, DBM) * groups;
  for (int want = 1; want <= std::min(8, num_k); want++) {
    const int kper = cdiv(num_k, want);
    const int ks = cdiv(num_k, kper);
    if (ks != want || kper > max_kper) continue;  // the same split as a smaller want, or too long a slice
    const long slots = ks > 1 ? (long)max_clusters<NB>(ks) : sms;
    const long waves = (base + slots - 1) / slots;
    const double ingest = (double)(DBM * (q8 ? 1 : 2) + NB * 2) * kper * DBK;
    const double reduce = ks > 1 ? (double)NB * DBM * 4 * (ks - 1) / ks : 0.0;
    const double cost = (double)waves * (kWaveBytes + ingest + reduce);
    if (best.nb == 0 || cost < best.cost) {
      best.nb = NB; best.groups = groups; best.ks = ks; best.kper = kper; best.cost = cost;
    }
  }
}

int make_tmap_u8(CUtensorMap* map, const int8_t* base, long rows, long cols, int box_rows, int box_cols) {
  typedef CUresult (*Enc)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                          const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                          CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static Enc enc = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (Enc) nullptr;
    return reinterpret_cast<Enc>(p);
  }();
  if (!enc) return fail(DUO_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || cols % 16)
    return fail(DUO_EINVAL, "tensor map: int8 base 16-byte aligned and rows a multiple of 16 bytes");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DUO_ECUDA, "cuTensorMapEncodeTiled (int8) failed with code " + std::to_string((int)r));
  return DUO_OK;
}

// shared host path: w is the 16-bit weight matrix, or (q8 != nullptr) the int8 matrix with its scales
int launch_dec(const void* x, int m, int k, const void* w, const Q8Args* q8, int n, int ab_dtype,
               const GemmEpiArgs& ep, cudaStream_t st) {
  if (m == 0 || n == 0) return DUO_OK;
  DUO_CHECK_ARG(m <= 256, "gemm_dec: at most 256 rows");
  DUO_CHECK_ARG(k % DBK == 0, "gemm_dec: k must be a multiple of 64");
  DUO_CHECK_ARG(ab_dtype == DUO_BF16 || ab_dtype == DUO_F16, "gemm_dec: operands must be bf16 or f16");
  DUO_CHECK_ARG(ep.epi == EPI_STORE || ep.epi == EPI_SWIGLU || ep.epi == EPI_ADD_F32,
                "gemm_dec: store, SwiGLU or residual-add epilogue");
  if (ep.epi == EPI_SWIGLU) {
    DUO_CHECK_ARG(n % 128 == 0, "gemm_dec: SwiGLU needs n a multiple of 128");
    DUO_CHECK_ARG(ep.c_dtype == ab_dtype, "gemm_dec: SwiGLU output is 16-bit");
  }
  if (ep.epi == EPI_ADD_F32) DUO_CHECK_ARG(ep.c_dtype == DUO_F32, "gemm_dec: the residual add is into f32");
  if (ep.nrm_out) {
    const bool al = ((reinterpret_cast<uintptr_t>(ep.nrm_out) | reinterpret_cast<uintptr_t>(ep.c) |
                      reinterpret_cast<uintptr_t>(ep.nrm_w)) & 15) == 0 && ep.ldc % 8 == 0 &&
                    (ep.vec == nullptr || (reinterpret_cast<uintptr_t>(ep.vec) & 15) == 0);
    DUO_CHECK_ARG(ep.epi == EPI_ADD_F32 && n % DBM == 0 && al && ep.nrm_w && ep.nrm_part,
                  "gemm_dec: the fused norm needs the residual add, n a multiple of 128 and 16-byte aligned rows");
  }
  if (ep.row_part)
    DUO_CHECK_ARG((ep.epi == EPI_STORE || ep.epi == EPI_SWIGLU) && ep.row_blocks > 0 && ep.row_d > 0,
                  "gemm_dec: row factors apply to the store and SwiGLU epilogues");
  Q8Args qa;
  int max_kper = 1 << 30;
  if (q8) {
    qa = *q8;
    DUO_CHECK_ARG(qa.s && qa.group > 0 && k % qa.group == 0 && qa.group % DBK == 0,
                  "q8 gemm: the group size must divide k and be a multiple of 64");
    qa.ngroups = k / qa.group;
    qa.apply = qa.group < k;
    if (qa.apply) max_kper = (kQ8Groups - 1) * qa.group / DBK;  // a slice spans at most kQ8Groups groups
    if (qa.inter > 0)
      DUO_CHECK_ARG(ep.epi == EPI_SWIGLU && n == 2 * qa.inter && qa.inter % 64 == 0,
                    "q8 gemm: the gate / up interleave is the SwiGLU epilogue's, n = 2 inter");
    else
      DUO_CHECK_ARG(ep.epi != EPI_SWIGLU, "q8 gemm: SwiGLU reads gate and up rows through the interleave");
  }
  const int num_k = k / DBK;
  DecPlan p;
  if (m > 64) plan_dec<128>(m, n, num_k, q8 != nullptr, max_kper, p);
  plan_dec<64>(m, n, num_k, q8 != nullptr, max_kper, p);
  if (p.nb == 0) return fail(DUO_EINVAL, "q8 gemm: k too long for the group scales of one K split");
  // direct epilogue (TMA store of the finished tile): no K split, a store or SwiGLU, an output whose base and rows
  // are 16-byte aligned, and at least one row group of rows (the store box is never taller than the whole output)
  const int es = ep.c_dtype == DUO_F32 ? 4 : 2;
  const bool c_aligned = (reinterpret_cast<uintptr_t>(ep.c) & 15) == 0 && ((long)ep.ldc * es) % 16 == 0;
  const int direct = p.ks == 1 && ep.epi != EPI_ADD_F32 && c_aligned && m >= p.nb;
  CUtensorMap tw, tx, tcm;
  std::memset(&tcm, 0, sizeof(tcm));
  if (q8) DUO_TRY(make_tmap_u8(&tw, static_cast<const int8_t*>(w), n, k, qa.inter > 0 ? 64 : DBM, DBK));
  else DUO_TRY(make_tmap_16(&tw, w, ab_dtype, n, k, k, DBM, DBK));
  DUO_TRY(make_tmap_16(&tx, x, ab_dtype, m, k, k, p.nb, DBK));
  if (direct) {
    const bool sw = ep.epi == EPI_SWIGLU;
    DUO_TRY(make_tmap_plain(&tcm, ep.c, ep.c_dtype, m, sw ? n / 2 : n, ep.ldc, p.nb, sw ? 64 : DBM));
  }
  const bool f16 = ab_dtype == DUO_F16;
#define DUO_DEC_DISPATCH(NB_, F16_, Q8_) \
  return dispatch_dec<NB_, F16_, Q8_>(tw, tx, tcm, m, n, k, p.groups, p.ks, p.kper, direct, ep, qa, st)
  if (q8) {
    if (p.nb == 64) { if (f16) DUO_DEC_DISPATCH(64, true, true); DUO_DEC_DISPATCH(64, false, true); }
    if (f16) DUO_DEC_DISPATCH(128, true, true);
    DUO_DEC_DISPATCH(128, false, true);
  }
  if (p.nb == 64) { if (f16) DUO_DEC_DISPATCH(64, true, false); DUO_DEC_DISPATCH(64, false, false); }
  if (f16) DUO_DEC_DISPATCH(128, true, false);
  DUO_DEC_DISPATCH(128, false, false);
#undef DUO_DEC_DISPATCH
}

}  // namespace

int launch_gemm_dec(const void* x, int m, int k, const void* w, int n, int ab_dtype, const GemmEpiArgs& ep,
                    cudaStream_t st) {
  return launch_dec(x, m, k, w, nullptr, n, ab_dtype, ep, st);
}

int launch_gemm_dec_q8(const void* x, int m, int k, const int8_t* wq, const float* ws, int group, int inter, int n,
                       int ab_dtype, const GemmEpiArgs& ep, cudaStream_t st) {
  Q8Args qa;
  qa.s = ws;
  qa.group = group;
  qa.inter = inter;
  return launch_dec(x, m, k, wq, &qa, n, ab_dtype, ep, st);
}

}  // namespace duo
