// Gated DeltaNet token mixer, part 1: the fused short-conv prologue and the recurrent (token-by-token) scan.
//
// Reference: engine/kernels_qwen35.js:129-247 (`conv`, `convState`, `delta`) and, for the arithmetic of its PyTorch
// path, transformers' Qwen3_5GatedDeltaNet (causal conv1d + SiLU, l2norm of q/k, beta = sigmoid(b),
// g = -exp(A_log) softplus(a + dt_bias), the delta rule, gated RMSNorm).
#include <cooperative_groups.h>

#include "kernels.cuh"
#include "tc.cuh"

namespace cg = cooperative_groups;

namespace duo {

// ---------------------------------------------------------------------------------------------------------------
// conv prologue.  Block = (128-channel group = one q, k or v head, row, 64-token tile), 256 threads.  The tile's inputs
// (tokens t0 - 3 .. t0 + 63; before the call's first token they come from the row's carried f32 state) are staged in
// shared memory as f32 with 16-byte loads.  Half-warp h of the block handles tokens h, h + 16, h + 32, h + 48; its
// thread c owns channels 4c .. 4c + 3 and 64 + 4c .. 64 + 4c + 3 (conflict-free float4 reads): causal depthwise conv
// (KS = 4) + SiLU, the head's l2norm (eps 1e-6) for q / k by half-warp shuffles, two 8-byte stores.  v-head blocks
// also compute beta and g for their tokens.  The block of tile 0 is the only reader of the old conv state and writes
// the new one after reading it.

constexpr int CONV_TT = 64, CONV_KS = 4, CONV_ROWS = CONV_TT + CONV_KS - 1, CONV_P = 128 + 4;

template <typename T>
__device__ __forceinline__ void load8(const T* p, float* o);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float* o) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}
template <typename T>
__device__ __forceinline__ void load8(const T* p, float* o) {  // 8 x 16-bit
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; i++) o[i] = to_f(h[i]);
}
__device__ __forceinline__ uint32_t pack2(__nv_bfloat16*, float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack2(__half*, float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <typename T>
__device__ __forceinline__ void store4(T* p, const float* v) {  // p 8-byte (16-bit T) / 16-byte (f32) aligned
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack2(p, v[0], v[1]), pack2(p, v[2], v[3]));
  }
}

template <typename T>
__global__ void __launch_bounds__(256) gdn_conv_kernel(GdnConvArgs a) {
  pdl_enter();
  __shared__ __align__(16) float xs[CONV_ROWS][CONV_P];
  const int cgp = blockIdx.x, rr = blockIdx.y, t0 = blockIdx.z * CONV_TT;
  const int conv_dim = 2 * a.hk * a.dk + a.hv * a.dv;
  const int tid = threadIdx.x;
  const int R = a.row_base + rr;
  const long m0 = (long)rr * a.t;
  const T* y = static_cast<const T*>(a.y);
  const int tn = min(CONV_TT, a.t - t0);
  const float* st = a.conv_state + ((long)R * (CONV_KS - 1)) * conv_dim + cgp * 128;  // st[j * conv_dim + c]

  // 1. stage rows r = 0 .. tn + 2 (token t0 - 3 + r), 16 threads x 8 channels per row (16-byte loads when the
  // projection rows allow it)
  const bool vec = a.w % 8 == 0 && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0;
  constexpr int NIT = (CONV_ROWS * 16 + 255) / 256;  // staging iterations per thread (5)
  const int nq = (tn + CONV_KS - 1) * 16;
  float v[NIT][8];
#pragma unroll
  for (int it = 0; it < NIT; it++) {  // every load is issued before any shared-memory store
    const int q = tid + 256 * it;
    if (q >= nq) continue;
    const int r = q >> 4, c8 = (q & 15) * 8;
    const int tt = t0 - (CONV_KS - 1) + r;
    if (tt < 0) {
      load8<float>(st + (long)((CONV_KS - 1) + tt) * conv_dim + c8, v[it]);
    } else {
      const T* src = y + (m0 + tt) * a.w + cgp * 128 + c8;
      if (vec) load8<T>(src, v[it]);
      else for (int i = 0; i < 8; i++) v[it][i] = to_f(src[i]);
    }
  }
#pragma unroll
  for (int it = 0; it < NIT; it++) {
    const int q = tid + 256 * it;
    if (q >= nq) continue;
    const int r = q >> 4, c8 = (q & 15) * 8;
    *reinterpret_cast<float4*>(&xs[r][c8]) = make_float4(v[it][0], v[it][1], v[it][2], v[it][3]);
    *reinterpret_cast<float4*>(&xs[r][c8 + 4]) = make_float4(v[it][4], v[it][5], v[it][6], v[it][7]);
  }
  // the new conv state = the last KS-1 inputs of (old state ++ this call's inputs); only tile 0 reads the old state
  float ns[CONV_KS - 1];
  const int sc = tid & 127;
  if (blockIdx.z == 0 && tid < 128) {
#pragma unroll
    for (int j = 0; j < CONV_KS - 1; j++) {
      const int idx = a.t + j;  // index into old ++ new
      ns[j] = idx < CONV_KS - 1 ? st[(long)idx * conv_dim + sc]
                                : to_f(y[(m0 + idx - (CONV_KS - 1)) * a.w + cgp * 128 + sc]);
    }
  }
  __syncthreads();
  if (blockIdx.z == 0 && tid < 128) {
    float* stw = a.conv_state + ((long)R * (CONV_KS - 1)) * conv_dim + cgp * 128 + sc;
#pragma unroll
    for (int j = 0; j < CONV_KS - 1; j++) stw[(long)j * conv_dim] = ns[j];
  }

  // 2. conv + SiLU (+ l2norm) per token, half-warp per token
  const int c = tid & 15, hw = tid >> 4;
  const unsigned hmask = 0xFFFFu << (tid & 16);  // the lanes of this thread's half-warp
  const bool norm = cgp < 2 * a.hk;  // q and k heads are l2-normalised; v heads pass through
  float w[8][CONV_KS];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int ch = cgp * 128 + (j < 4 ? 4 * c + j : 64 + 4 * c + j - 4);
    const float4 ww = *reinterpret_cast<const float4*>(a.conv_w + (long)ch * CONV_KS);
    w[j][0] = ww.x; w[j][1] = ww.y; w[j][2] = ww.z; w[j][3] = ww.w;
  }
  T* out = static_cast<T*>(a.qkv_out);
  for (int i = hw; i < tn; i += 16) {
    float v[8];
#pragma unroll
    for (int half = 0; half < 2; half++) {
      const int col = half * 64 + 4 * c;
      float4 x[CONV_KS];
#pragma unroll
      for (int d = 0; d < CONV_KS; d++) x[d] = *reinterpret_cast<const float4*>(&xs[i + d][col]);
      const float xv[CONV_KS][4] = {{x[0].x, x[0].y, x[0].z, x[0].w}, {x[1].x, x[1].y, x[1].z, x[1].w},
                                    {x[2].x, x[2].y, x[2].z, x[2].w}, {x[3].x, x[3].y, x[3].z, x[3].w}};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float* wj = w[half * 4 + j];
        v[half * 4 + j] = silu_bf<T>(wj[0] * xv[0][j] + wj[1] * xv[1][j] + wj[2] * xv[2][j] + wj[3] * xv[3][j]);
      }
    }
    if (norm) {
      // the two half-warps of a warp may be on different tokens, or one of them past the last token (tn mod 16
      // odd): the reduction names only this half-warp's lanes
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 8; j++) ss += v[j] * v[j];
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(hmask, ss, o);
      const float inv = rsqrtf(ss + 1e-6f);
#pragma unroll
      for (int j = 0; j < 8; j++) v[j] *= inv;
    }
    T* o = out + (m0 + t0 + i) * conv_dim + cgp * 128;
    store4<T>(o + 4 * c, v);
    store4<T>(o + 64 + 4 * c, v + 4);
  }
  if (!norm && tid < tn) {
    const int h = cgp - 2 * a.hk;
    const long m = m0 + t0 + tid;
    const long base = m * a.w + conv_dim + a.hv * a.dv;
    const float b = to_f(y[base + h]);
    const float av = to_f(y[base + a.hv + h]);
    a.beta_out[m * a.hv + h] = sigmoidf_(b);
    a.g_out[m * a.hv + h] = -expf(a.a_log[h]) * softplusf_(av + a.dt_bias[h]);
  }
}

// TMA-fed form of the conv prologue (16-bit projections whose rows are 16-byte aligned).  Block = (128-channel group,
// row, CONV_TPC consecutive 64-token tiles).  Thread 0 streams the tiles' raw [64 tokens][128 channels] inputs into a
// CONV_NS-deep shared-memory ring by 2D TMA loads, so two tiles are in flight while one is processed; a tile's 3-token
// halo is the previous tile's last 3 rows, kept in f32 (the block's first tile takes it from the carried conv state
// or from the projection).  Per tile the arithmetic is that of gdn_conv_kernel: half-warp h takes tokens h, h + 16, ..,
// thread c channels 4c .. 4c + 3 and 64 + 4c .. 64 + 4c + 3.
constexpr int CONV_NS = 3, CONV_TPC = 8;
constexpr int CONV_TMA_SMEM = 1024 + CONV_NS * CONV_TT * 128 * 2 + 3 * 128 * 4 + 64;

template <typename T>
__global__ void __launch_bounds__(256) gdn_conv_tma_kernel(const __grid_constant__ CUtensorMap tmy, GdnConvArgs a,
                                                           unsigned* fault) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  T* ring = reinterpret_cast<T*>(smem);                                                // [NS][64][128]
  float* halo = reinterpret_cast<float*>(smem + CONV_NS * CONV_TT * 128 * sizeof(T));  // [3][128]
  uint64_t* full = reinterpret_cast<uint64_t*>(halo + 3 * 128);                        // [NS]
  constexpr uint32_t TILE_BYTES = CONV_TT * 128 * sizeof(T);
  const int cgp = blockIdx.x, rr = blockIdx.y;
  const int tiles = (a.t + CONV_TT - 1) / CONV_TT;
  const int j0 = blockIdx.z * CONV_TPC, j1 = min(tiles, j0 + CONV_TPC);
  const int conv_dim = 2 * a.hk * a.dk + a.hv * a.dv;
  const int tid = threadIdx.x, c = tid & 15, hw = tid >> 4;
  const unsigned hmask = 0xFFFFu << (tid & 16);  // the lanes of this thread's half-warp
  const int R = a.row_base + rr;
  const long m0 = (long)rr * a.t;
  const T* y = static_cast<const T*>(a.y);
  float* st = a.conv_state + ((long)R * (CONV_KS - 1)) * conv_dim + cgp * 128;  // st[j * conv_dim + ch]

  if (tc::fault_pending(fault)) {  // an earlier kernel gave up a wait
    pdl_wait();
    return;
  }
  if (tid == 0) {
    for (int s2 = 0; s2 < CONV_NS; s2++) tc::mbar_init(&full[s2], 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmy);
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  if (tid == 0) {
    for (int s2 = 0; s2 < CONV_NS && j0 + s2 < j1; s2++) {
      tc::mbar_arrive_expect_tx(&full[s2], TILE_BYTES);
      tc::tma_load_2d(ring + s2 * CONV_TT * 128, &tmy, cgp * 128, (int)(m0 + (long)(j0 + s2) * CONV_TT), &full[s2]);
    }
  }
  // halo of the first tile; the new conv state = the last KS-1 inputs of (old state ++ this call's inputs), written by
  // the block of tile 0 (the only reader of the old state) once every read of it is done
  float ns[CONV_KS - 1];
  if (tid < 128) {
#pragma unroll
    for (int d = 0; d < CONV_KS - 1; d++) {
      const int tt = j0 * CONV_TT - (CONV_KS - 1) + d;
      halo[d * 128 + tid] = tt < 0 ? st[(long)((CONV_KS - 1) + tt) * conv_dim + tid]
                                   : to_f(y[(m0 + tt) * a.w + cgp * 128 + tid]);
    }
    if (blockIdx.z == 0) {
#pragma unroll
      for (int d = 0; d < CONV_KS - 1; d++) {
        const int idx = a.t + d;  // index into old ++ new
        ns[d] = idx < CONV_KS - 1 ? st[(long)idx * conv_dim + tid]
                                  : to_f(y[(m0 + idx - (CONV_KS - 1)) * a.w + cgp * 128 + tid]);
      }
    }
  }
  __syncthreads();
  if (blockIdx.z == 0 && tid < 128) {
#pragma unroll
    for (int d = 0; d < CONV_KS - 1; d++) st[(long)d * conv_dim + tid] = ns[d];
  }

  const bool norm = cgp < 2 * a.hk;  // q and k heads are l2-normalised; v heads pass through
  float w[8][CONV_KS];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int ch = cgp * 128 + (j < 4 ? 4 * c + j : 64 + 4 * c + j - 4);
    const float4 ww = *reinterpret_cast<const float4*>(a.conv_w + (long)ch * CONV_KS);
    w[j][0] = ww.x; w[j][1] = ww.y; w[j][2] = ww.z; w[j][3] = ww.w;
  }
  T* out = static_cast<T*>(a.qkv_out);
  const int hv_idx = cgp - 2 * a.hk;  // v-head blocks: the head whose gates they compute
  const float neg_ea = norm ? 0.f : -expf(a.a_log[hv_idx]), dtb = norm ? 0.f : a.dt_bias[hv_idx];
  for (int j = j0; j < j1; j++) {
    const int s2 = (j - j0) % CONV_NS;
    const uint32_t ph = (uint32_t)(((j - j0) / CONV_NS) & 1);
    const int t0 = j * CONV_TT, tn = min(CONV_TT, a.t - t0);
    // v-head blocks: this tile's b and a inputs (one per token, 16 KB apart) requested before the wait, so that
    // their latency overlaps it rather than the tile's tail
    float yb = 0.f, ya = 0.f;
    if (!norm && tid < tn) {
      const long base = (m0 + t0 + tid) * a.w + conv_dim + a.hv * a.dv + hv_idx;
      yb = to_f(y[base]);
      ya = to_f(y[base + a.hv]);
    }
    const bool ok = tc::mbar_wait(&full[s2], ph);
    if (__syncthreads_or(!ok)) {  // a load that never landed: give up (the fault word says so)
      if (tid == 0) {
        atomicOr(fault, 16u);
        // tiles j .. j + NS - 1 may still be in flight into this CTA's ring: wait for them (bounded) before the CTA
        // and its shared memory go away
        for (int jj = j; jj < j1 && jj < j + CONV_NS; jj++)
          tc::mbar_wait(&full[(jj - j0) % CONV_NS], (uint32_t)(((jj - j0) / CONV_NS) & 1));
      }
      __syncthreads();
      return;
    }
    const T* tile = ring + s2 * CONV_TT * 128;
    for (int i = hw; i < tn; i += 16) {
      float v[8];
#pragma unroll
      for (int half = 0; half < 2; half++) {
        const int col = half * 64 + 4 * c;
        float x[CONV_KS][4];
#pragma unroll
        for (int d = 0; d < CONV_KS; d++) {
          const int row = i - (CONV_KS - 1) + d;
          if (row >= 0) {
            const uint2 u = *reinterpret_cast<const uint2*>(tile + row * 128 + col);
            const T* hh = reinterpret_cast<const T*>(&u);
#pragma unroll
            for (int e = 0; e < 4; e++) x[d][e] = to_f(hh[e]);
          } else {
            const float4 f = *reinterpret_cast<const float4*>(halo + (row + CONV_KS - 1) * 128 + col);
            x[d][0] = f.x; x[d][1] = f.y; x[d][2] = f.z; x[d][3] = f.w;
          }
        }
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const float* wj = w[half * 4 + e];
          v[half * 4 + e] = silu_bf<T>(wj[0] * x[0][e] + wj[1] * x[1][e] + wj[2] * x[2][e] + wj[3] * x[3][e]);
        }
      }
      if (norm) {
        // half-warp reduction: when tn mod 16 is odd the other half-warp of this warp has left the loop and waits
        // at the block barrier below, so a full-warp mask would never complete
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 8; e++) ss += v[e] * v[e];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(hmask, ss, o);
        const float inv = rsqrtf(ss + 1e-6f);
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] *= inv;
      }
      T* o = out + (m0 + t0 + i) * conv_dim + cgp * 128;
      store4<T>(o + 4 * c, v);
      store4<T>(o + 64 + 4 * c, v + 4);
    }
    if (!norm && tid < tn) {
      const long m = m0 + t0 + tid;
      a.beta_out[m * a.hv + hv_idx] = sigmoidf_(yb);
      a.g_out[m * a.hv + hv_idx] = neg_ea * softplusf_(ya + dtb);
    }
    __syncthreads();  // every read of this slot and of the halo is done
    if (j + 1 < j1 && tid < 128) {
#pragma unroll
      for (int d = 0; d < CONV_KS - 1; d++) halo[d * 128 + tid] = to_f(tile[(CONV_TT - (CONV_KS - 1) + d) * 128 + tid]);
    }
    __syncthreads();  // the next tile's halo is in place; this slot may be refilled
    if (tid == 0 && j + CONV_NS < j1) {
      tc::fence_proxy_async();
      tc::mbar_arrive_expect_tx(&full[s2], TILE_BYTES);
      tc::tma_load_2d(ring + s2 * CONV_TT * 128, &tmy, cgp * 128, (int)(m0 + (long)(j + CONV_NS) * CONV_TT), &full[s2]);
    }
  }
}

int launch_gdn_conv(const GdnConvArgs& a, int dtype, cudaStream_t st) {
  if (a.rows == 0 || a.t == 0) return DUO_OK;
  if (a.dk != 128 || a.dv != 128 || a.ks != CONV_KS) return fail(DUO_EINVAL, "gdn_conv: needs dk = dv = 128, ks = 4");
  const int conv_dim = 2 * a.hk * a.dk + a.hv * a.dv;
  // the TMA-fed form for 16-bit projections whose rows are 16-byte aligned, with at least one box (64 tokens) per row:
  // shorter rows would stream a mostly unused box per tile (the register-staged kernel loads only their tokens)
  if (dtype != DUO_F32 && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0 && a.w % 8 == 0 && a.t >= CONV_TT) {
    CUtensorMap tmy;
    DUO_TRY(make_tmap_plain(&tmy, a.y, dtype, (long)a.rows * a.t, a.w, a.w, CONV_TT, 128));
    unsigned* fault = tc_fault_ptr();
    if (!fault) return fail(DUO_ECUDA, "tensor-core fault word is not addressable");
    dim3 grid(conv_dim / 128, a.rows, cdiv(cdiv(a.t, CONV_TT), CONV_TPC));
    return with_act(dtype, [&](auto tag) -> int {
      using T = decltype(tag);
      if constexpr (sizeof(T) == 2) {
        DUO_TRY(ensure_smem_attr(gdn_conv_tma_kernel<T>, CONV_TMA_SMEM));
        DUO_CUDA_TRY(::duo::launch_kernel(gdn_conv_tma_kernel<T>, grid, 256, CONV_TMA_SMEM, st, tmy, a, fault));
        DUO_LAUNCH_CHECK("gdn_conv_tma_kernel");
      }
      return DUO_OK;
    });
  }
  dim3 grid(conv_dim / 128, a.rows, cdiv(a.t, CONV_TT));
  return with_act(dtype, [&](auto tag) -> int {
    DUO_CUDA_TRY(::duo::launch_kernel(gdn_conv_kernel<decltype(tag)>, grid, 256, 0, st, a));
    DUO_LAUNCH_CHECK("gdn_conv_kernel");
    return DUO_OK;
  });
}

// ---------------------------------------------------------------------------------------------------------------
// recurrent scan.  One thread-block cluster of CS CTAs per (row, value head); CTA s owns state columns
// [s * 128 / CS, (s + 1) * 128 / CS) -- the delta rule is independent per state column -- and all 128 state rows.
// Thread (rg, jj) keeps rows rg * RPT .. rg * RPT + RPT - 1 of column jj in registers for the whole call.
// Per token: S *= exp(g); u = S^T k; S += k (beta (v - u))^T; o = S^T (q / sqrt(dk)), then (engine path) the gated
// RMSNorm over the head's 128 outputs, whose sum of squares is reduced across the cluster through distributed
// shared memory.

template <typename T, int CS, bool NORM>
__global__ void __cluster_dims__(CS, 1, 1) __launch_bounds__(128) gdn_recurrent_kernel(GdnScanArgs a) {
  pdl_enter();
  constexpr int CW = 128 / CS;   // columns per CTA
  constexpr int RPT = 128 / CS;  // state rows per thread (CS threads share a column)
  __shared__ float qs[128], ks[128];
  __shared__ float red_u[CS][CW], red_o[CS][CW];
  __shared__ float red32[32];
  __shared__ float part[2];
  const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x;
  const int jj = tid % CW, rg = tid / CW;
  const int j = s * CW + jj;
  const int kh = h / (a.h / a.hq);
  float* S = a.state + (((long)(a.state_row0 + b) * a.h + h) * 128) * 128;
  float st[RPT];
#pragma unroll
  for (int r = 0; r < RPT; r++) st[r] = S[(long)(rg * RPT + r) * 128 + j];
  const T* qp = static_cast<const T*>(a.q);
  const T* kp = static_cast<const T*>(a.k);
  const T* vp = static_cast<const T*>(a.v);
  T* op = static_cast<T*>(a.o);
  const float qscale = rsqrtf(128.f);
  cg::cluster_group cluster = cg::this_cluster();

  for (int t = 0; t < a.t; t++) {
    const long m = (long)b * a.t + t;
    float qv = to_f(qp[m * a.q_stride + kh * 128 + tid]);
    float kv = to_f(kp[m * a.k_stride + kh * 128 + tid]);
    if (a.l2norm_qk) {
      const float sq = block_sum(qv * qv, red32);
      const float sk = block_sum(kv * kv, red32);
      qv *= rsqrtf(sq + 1e-6f);
      kv *= rsqrtf(sk + 1e-6f);
    }
    __syncthreads();  // previous token's readers of qs / ks / red_* are done
    qs[tid] = qv * qscale;
    ks[tid] = kv;
    const float gt = a.g[m * a.h + h];
    const float bt = a.beta[m * a.h + h];
    __syncthreads();
    const float dec = expf(gt);
    float pu = 0.f;
#pragma unroll
    for (int r = 0; r < RPT; r++) {
      st[r] *= dec;
      pu = fmaf(st[r], ks[rg * RPT + r], pu);
    }
    red_u[rg][jj] = pu;
    __syncthreads();
    float u = 0.f;
#pragma unroll
    for (int i = 0; i < CS; i++) u += red_u[i][jj];
    const float vj = to_f(vp[m * a.v_stride + h * 128 + j]);
    const float d = bt * (vj - u);
    float po = 0.f;
#pragma unroll
    for (int r = 0; r < RPT; r++) {
      st[r] = fmaf(ks[rg * RPT + r], d, st[r]);
      po = fmaf(st[r], qs[rg * RPT + r], po);
    }
    red_o[rg][jj] = po;
    __syncthreads();
    float o = 0.f;
#pragma unroll
    for (int i = 0; i < CS; i++) o += red_o[i][jj];
    if (NORM) {
      // sum of o^2 over this CTA's columns (rows rg == 0 hold each column once), then over the cluster
      const float ss = block_sum(rg == 0 ? o * o : 0.f, red32);
      if (tid == 0) part[t & 1] = ss;
      cluster.sync();
      float tot = 0.f;
#pragma unroll
      for (int i = 0; i < CS; i++) tot += *cluster.map_shared_rank(&part[t & 1], i);
      const float rms = rsqrtf(tot / 128.f + a.eps);
      if (rg == 0) {
        const float z = to_f(static_cast<const T*>(a.z)[m * a.z_stride + h * 128 + j]);
        const float hs = a.head_scale ? a.head_scale[h] : 1.f;
        op[m * a.o_stride + h * 128 + j] = from_f<T>(o * rms * a.norm_w[j] * silu_t<T>(z) * hs);
      }
    } else if (rg == 0) {
      op[m * a.o_stride + h * 128 + j] = from_f<T>(o);
    }
  }
#pragma unroll
  for (int r = 0; r < RPT; r++) S[(long)(rg * RPT + r) * 128 + j] = st[r];
  if (NORM) cluster.sync();  // peers may still read this CTA's `part`
}

template <typename T, bool NORM>
static int run_recurrent(const GdnScanArgs& a, cudaStream_t st) {
  const long pairs = (long)a.b * a.h;
  // 8 column slices while the (row, head) pairs alone cannot fill the GPU, else 4 (32 state rows per thread)
  if (pairs <= 64) DUO_CUDA_TRY(::duo::launch_kernel(gdn_recurrent_kernel<T, 8, NORM>, dim3(8, a.h, a.b), 128, 0, st, a));
  else DUO_CUDA_TRY(::duo::launch_kernel(gdn_recurrent_kernel<T, 4, NORM>, dim3(4, a.h, a.b), 128, 0, st, a));
  DUO_LAUNCH_CHECK("gdn_recurrent_kernel");
  return DUO_OK;
}

// ---------------------------------------------------------------------------------------------------------------
// short prefill (2 <= t <= SHORT_T tokens per row, 16-bit engines): the delta rule token by token with the (row,
// head) state held in registers across the call's tokens.  The chunked kernel computes a whole 64-token chunk
// whatever t, and its one CTA per (row, head) owns an SM (its shared memory) for its fixed costs; here a persistent
// grid of 2 CTAs per SM walks the (row, head) items, stages the item's q (times 1 / sqrt(dk)), k, v, e^g and beta in
// shared memory, reads and writes the 64 KB state once, and per token runs S *= e^g; u = S^T k;
// S += k (beta (v - u))^T; o = S^T q.  Lane l of warp w owns state column 16 w + l % 16, rows 64 (l / 16) ..
// + 63, so both column sums close with one shuffle and a token needs no block barrier.  q and k arrive l2-normalised
// from the conv prologue (l2norm_qk == 0).  Then the gated RMSNorm per token.
constexpr int SHORT_T = 16, SHORT_THREADS = 256;

template <typename T>
__global__ void __launch_bounds__(SHORT_THREADS, 2) gdn_short_kernel(GdnScanArgs a) {
  pdl_enter();
  __shared__ __align__(16) float qs[SHORT_T][128], ks[SHORT_T][128], vs[SHORT_T][128], os[SHORT_T][128];
  __shared__ float gs[SHORT_T], bs[SHORT_T];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = warp * 16 + (lane & 15), r0 = (lane >> 4) * 64;  // this lane's state column and first row
  const int H = a.h, TT = a.t;
  const int items = a.b * H;
  const T* q = static_cast<const T*>(a.q);
  const T* k = static_cast<const T*>(a.k);
  const T* v = static_cast<const T*>(a.v);
  const float qscale = rsqrtf(128.f);
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const int b = item / H, h = item % H, kh = h / (H / a.hq);
    float* S = a.state + (((long)(a.state_row0 + b) * H + h) * 128) * 128;  // [dk][dv]
    for (int idx = tid; idx < TT * 128; idx += SHORT_THREADS) {
      const int t = idx >> 7, cc = idx & 127;
      const long m = (long)b * TT + t;
      qs[t][cc] = to_f(q[m * a.q_stride + kh * 128 + cc]) * qscale;
      ks[t][cc] = to_f(k[m * a.k_stride + kh * 128 + cc]);
      vs[t][cc] = to_f(v[m * a.v_stride + h * 128 + cc]);
    }
    if (tid < TT) {
      const long m = (long)b * TT + tid;
      gs[tid] = expf(a.g[m * H + h]);
      bs[tid] = a.beta[m * H + h];
    }
    float st[64];
#pragma unroll
    for (int r = 0; r < 64; r++) st[r] = S[(long)(r0 + r) * 128 + c];
    __syncthreads();
#pragma unroll 1
    for (int t = 0; t < TT; t++) {
      const float gd = gs[t];
      const float4* k4 = reinterpret_cast<const float4*>(&ks[t][r0]);
      const float4* q4 = reinterpret_cast<const float4*>(&qs[t][r0]);
      float ua = 0.f, ub = 0.f, uc = 0.f, ud = 0.f;  // four independent chains
#pragma unroll
      for (int r = 0; r < 16; r++) {
        const float4 kk = k4[r];
        st[4 * r] *= gd; st[4 * r + 1] *= gd; st[4 * r + 2] *= gd; st[4 * r + 3] *= gd;
        ua = fmaf(st[4 * r], kk.x, ua); ub = fmaf(st[4 * r + 1], kk.y, ub);
        uc = fmaf(st[4 * r + 2], kk.z, uc); ud = fmaf(st[4 * r + 3], kk.w, ud);
      }
      float u = (ua + ub) + (uc + ud);
      u += __shfl_xor_sync(0xffffffffu, u, 16);
      const float d = bs[t] * (vs[t][c] - u);
      float oa = 0.f, ob = 0.f, oc = 0.f, od = 0.f;
#pragma unroll
      for (int r = 0; r < 16; r++) {
        const float4 kk = k4[r], qq = q4[r];
        st[4 * r] = fmaf(kk.x, d, st[4 * r]); st[4 * r + 1] = fmaf(kk.y, d, st[4 * r + 1]);
        st[4 * r + 2] = fmaf(kk.z, d, st[4 * r + 2]); st[4 * r + 3] = fmaf(kk.w, d, st[4 * r + 3]);
        oa = fmaf(st[4 * r], qq.x, oa); ob = fmaf(st[4 * r + 1], qq.y, ob);
        oc = fmaf(st[4 * r + 2], qq.z, oc); od = fmaf(st[4 * r + 3], qq.w, od);
      }
      float o = (oa + ob) + (oc + od);
      o += __shfl_xor_sync(0xffffffffu, o, 16);
      if (lane < 16) os[t][c] = o;
    }
#pragma unroll
    for (int r = 0; r < 64; r++) S[(long)(r0 + r) * 128 + c] = st[r];
    __syncthreads();  // os complete
    // per token: gated RMSNorm over the head's 128 outputs (warp w takes tokens w, w + 8; lane: columns 4 lane ..)
    const float hs = a.head_scale ? a.head_scale[h] : 1.f;
    for (int t = warp; t < TT; t += SHORT_THREADS / 32) {
      const long m = (long)b * TT + t;
      float ov[4], ss = 0.f;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        ov[i] = os[t][lane * 4 + i];
        ss += ov[i] * ov[i];
      }
      ss = warp_sum(ss);
      const float rms = a.norm_w ? rsqrtf(ss / 128.f + a.eps) : 1.f;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int cc = lane * 4 + i;
        float y = ov[i];
        if (a.norm_w)
          y = y * rms * a.norm_w[cc] * silu_bf<T>(to_f(static_cast<const T*>(a.z)[m * a.z_stride + h * 128 + cc])) * hs;
        static_cast<T*>(a.o)[m * a.o_stride + h * 128 + cc] = from_f<T>(y);
      }
    }
    __syncthreads();  // the staged inputs and os are rewritten by the next item
  }
}

int launch_gdn_short(const GdnScanArgs& a, int dtype, cudaStream_t st) {
  if (a.b == 0 || a.t == 0) return DUO_OK;
  if (a.t > SHORT_T || a.dk != 128 || a.dv != 128 || a.l2norm_qk || a.hq < 1 || a.h % a.hq ||
      (dtype != DUO_BF16 && dtype != DUO_F16))
    return fail(DUO_EINVAL, "gdn_short: 16-bit inputs, t <= 16, dk = dv = 128, q and k already normalised");
  const int items = a.b * a.h;
  const int grid = std::min(items, 2 * sm_count());
  return with_act(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    if constexpr (sizeof(T) == 2) {
      DUO_CUDA_TRY(::duo::launch_kernel(gdn_short_kernel<T>, grid, SHORT_THREADS, 0, st, a));
      DUO_LAUNCH_CHECK("gdn_short_kernel");
    }
    return DUO_OK;
  });
}

int launch_gdn_recurrent(const GdnScanArgs& a, int dtype, cudaStream_t st) {
  if (a.b == 0 || a.t == 0) return DUO_OK;
  if (a.dk != 128 || a.dv != 128) return fail(DUO_EINVAL, "gdn: needs dk = dv = 128");
  if (a.hq <= 0 || a.h % a.hq) return fail(DUO_EINVAL, "gdn: value heads must be a multiple of q/k heads");
  const bool norm = a.norm_w != nullptr;
  return with_act(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    return norm ? run_recurrent<T, true>(a, st) : run_recurrent<T, false>(a, st);
  });
}

// ---------------------------------------------------------------------------------------------------------------
// decode step (t = 1) of the engine, everything of a Gated DeltaNet layer between the projection and out_proj in one
// kernel: conv1d + SiLU on this token (with the carried state, which it also shifts), l2norm of q and k, the gates,
// the delta-rule update of the f32 state and the gated RMSNorm.
//
// The step is bound by the state: 64 KB read and written per (row, head).  A persistent grid (DEC_CPS CTAs per SM)
// walks the (row, head) items; each item is two slices of 64 state columns x 128 rows (32 KB) that stream through a
// DEC_NS-deep shared-memory ring filled by cp.async, so while one slice is updated the next two are in flight, across
// item boundaries too.  Thread (rg = tid / 16, cg = tid % 16) owns rows 8 rg .. 8 rg + 7 of the slice's columns
// 4 cg .. 4 cg + 3: it copies exactly those 8 float4 into the ring and is their only reader, so the ring needs no
// barrier (a thread's cp.async.wait_group makes its own copies visible to it).  Needs hk == hv (one CTA owns each
// q/k channel's conv-state shift).

constexpr int DEC_THREADS = 256, DEC_NS = 3, DEC_CPS = 2;
constexpr int DEC_SLICE = 128 * 64;  // floats
constexpr int DEC_SMEM = DEC_NS * DEC_SLICE * 4;

template <typename T>
__global__ void __launch_bounds__(DEC_THREADS, DEC_CPS) gdn_decode_kernel(GdnConvArgs ca, GdnScanArgs a) {
  extern __shared__ __align__(16) float ring[];  // [DEC_NS][128 rows][64 columns]
  __shared__ float qs[128], ks[128], vs[128], os[128];
  // per-warp partial column sums of u (redu) and o (redo): two buffers, so that each is rewritten only after a
  // barrier that every reader of its previous contents has passed (two barriers per slice instead of four)
  __shared__ __align__(16) float redu[8][64], redo[8][64];
  __shared__ float red8[8];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cg = tid & 15, rg = tid >> 4;
  const int H = a.h;
  const int items = a.b * H;
  const int conv_dim = 2 * ca.hk * 128 + ca.hv * 128;
  const T* y = static_cast<const T*>(ca.y);
  // this CTA's items are blockIdx.x + j gridDim.x; its slices are numbered 2 j + half
  const int my_items = items > (int)blockIdx.x ? (items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int nslices = 2 * my_items;
  auto state_of = [&](int j) {
    const int item = blockIdx.x + j * gridDim.x;
    const int b = item / H, h = item % H;
    return reinterpret_cast<float4*>(a.state + (((long)(a.state_row0 + b) * H + h) * 128) * 128);
  };
  auto issue = [&](int g) {  // cp.async this thread's 8 float4 of slice g into its ring slot
    if (g < nslices) {
      const float4* src = state_of(g >> 1) + (g & 1) * 16 + cg;
      float* dst = ring + (g % DEC_NS) * DEC_SLICE + cg * 4;
#pragma unroll
      for (int r = 0; r < 8; r++) cp_async16(dst + (rg * 8 + r) * 64, src + (rg * 8 + r) * 32);
    }
    cp_commit();  // possibly empty: keeps one group per slice so the wait count stays fixed
  };
#pragma unroll
  for (int g = 0; g < DEC_NS - 1; g++) issue(g);
  // Programmatic launch: the first state slices stream in while the preceding kernel (the layer's in-projection,
  // which never touches the recurrent state) finishes; the conv inputs, conv state and outputs wait for it.
  pdl_enter();

  // The conv inputs of an item (its channels' carried conv state and new input, z, the gate inputs) are loaded one
  // item ahead, so their latency hides behind the previous item's state slices.  Items own disjoint channels, and
  // the projection output is read only after the programmatic-launch wait.
  const int c = tid & 127;
  struct ConvIn {
    float xq[4], xv[4], z, yb, ya;
  };
  auto fetch = [&](int j, ConvIn& in) {
    if (j >= my_items) return;
    const int item = blockIdx.x + j * gridDim.x;
    const int b = item / H, h = item % H;
    const long yrow = (long)b * ca.w;
    const float* cs = ca.conv_state + ((long)(a.state_row0 + b) * 3) * conv_dim;
    const int chq = (tid < 128 ? 0 : ca.hk * 128) + h * 128 + c;
    in.xq[0] = cs[chq]; in.xq[1] = cs[conv_dim + chq]; in.xq[2] = cs[2L * conv_dim + chq];
    in.xq[3] = to_f(y[yrow + chq]);
    if (tid < 128) {
      const int chv = 2 * ca.hk * 128 + h * 128 + c;
      in.xv[0] = cs[chv]; in.xv[1] = cs[conv_dim + chv]; in.xv[2] = cs[2L * conv_dim + chv];
      in.xv[3] = to_f(y[yrow + chv]);
      in.z = to_f(static_cast<const T*>(a.z)[(long)b * a.z_stride + h * 128 + c]);
    }
    const long gb = yrow + conv_dim + ca.hv * 128;
    in.yb = to_f(y[gb + h]);
    in.ya = to_f(y[gb + ca.hv + h]);
  };
  ConvIn nxt{};
  fetch(0, nxt);

  for (int j = 0; j < my_items; j++) {
    const int item = blockIdx.x + j * gridDim.x;
    const int b = item / H, h = item % H;
    const int R = a.state_row0 + b;
    const ConvIn cur = nxt;
    fetch(j + 1, nxt);
    // 1. conv + SiLU of the head's q (threads 0..127, also v) and k (128..255) channels, shifting their conv state
    const float z = cur.z;
    auto conv_ch = [&](int ch, const float (&x)[4]) {
      float* cs = ca.conv_state + ((long)R * 3) * conv_dim + ch;
      const float4 w = *reinterpret_cast<const float4*>(ca.conv_w + (long)ch * 4);
      cs[0] = x[1]; cs[(long)conv_dim] = x[2]; cs[2L * conv_dim] = x[3];
      return silu_t<T>(w.x * x[0] + w.y * x[1] + w.z * x[2] + w.w * x[3]);
    };
    const float qk = conv_ch((tid < 128 ? 0 : ca.hk * 128) + h * 128 + c, cur.xq);
    if (tid < 128) vs[c] = conv_ch(2 * ca.hk * 128 + h * 128 + c, cur.xv);
    const float ssq = warp_sum(qk * qk);
    if (lane == 0) red8[warp] = ssq;
    const float beta = sigmoidf_(cur.yb);
    const float gdec = expf(-expf(ca.a_log[h]) * softplusf_(cur.ya + ca.dt_bias[h]));
    __syncthreads();
    {
      const int w0 = tid < 128 ? 0 : 4;
      const float tot = red8[w0] + red8[w0 + 1] + red8[w0 + 2] + red8[w0 + 3];
      if (tid < 128) qs[c] = qk * rsqrtf(tot + 1e-6f) * rsqrtf(128.f);
      else ks[c] = qk * rsqrtf(tot + 1e-6f);
    }
    __syncthreads();

    // 2. per 64-column slice: decay, u = S^T k, delta = beta (v - u), S += k delta^T, o = S^T q
#pragma unroll 1
    for (int half = 0; half < 2; half++) {
      const int g = 2 * j + half;
      issue(g + DEC_NS - 1);
      cp_wait<DEC_NS - 1>();
      const float* sl = ring + (g % DEC_NS) * DEC_SLICE + cg * 4;
      float4 st[8];
#pragma unroll
      for (int r = 0; r < 8; r++) st[r] = *reinterpret_cast<const float4*>(sl + (rg * 8 + r) * 64);
      float u4[4] = {0, 0, 0, 0};
#pragma unroll
      for (int r = 0; r < 8; r++) {
        const float kr = ks[rg * 8 + r];
        st[r].x *= gdec; st[r].y *= gdec; st[r].z *= gdec; st[r].w *= gdec;
        u4[0] = fmaf(st[r].x, kr, u4[0]); u4[1] = fmaf(st[r].y, kr, u4[1]);
        u4[2] = fmaf(st[r].z, kr, u4[2]); u4[3] = fmaf(st[r].w, kr, u4[3]);
      }
#pragma unroll
      for (int i = 0; i < 4; i++) u4[i] += __shfl_xor_sync(0xffffffffu, u4[i], 16);
      if (lane < 16) *reinterpret_cast<float4*>(&redu[warp][cg * 4]) = make_float4(u4[0], u4[1], u4[2], u4[3]);
      __syncthreads();
      float d4[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int col = cg * 4 + i;
        float u = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++) u += redu[w][col];
        d4[i] = beta * (vs[half * 64 + col] - u);
      }
      float o4[4] = {0, 0, 0, 0};
      float4* S4 = state_of(j) + half * 16 + cg;
#pragma unroll
      for (int r = 0; r < 8; r++) {
        const float kr = ks[rg * 8 + r], qr = qs[rg * 8 + r];
        st[r].x = fmaf(kr, d4[0], st[r].x); st[r].y = fmaf(kr, d4[1], st[r].y);
        st[r].z = fmaf(kr, d4[2], st[r].z); st[r].w = fmaf(kr, d4[3], st[r].w);
        o4[0] = fmaf(st[r].x, qr, o4[0]); o4[1] = fmaf(st[r].y, qr, o4[1]);
        o4[2] = fmaf(st[r].z, qr, o4[2]); o4[3] = fmaf(st[r].w, qr, o4[3]);
        S4[(rg * 8 + r) * 32] = st[r];
      }
#pragma unroll
      for (int i = 0; i < 4; i++) o4[i] += __shfl_xor_sync(0xffffffffu, o4[i], 16);
      if (lane < 16) *reinterpret_cast<float4*>(&redo[warp][cg * 4]) = make_float4(o4[0], o4[1], o4[2], o4[3]);
      __syncthreads();
      if (tid < 64) {
        float o = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++) o += redo[w][tid];
        os[half * 64 + tid] = o;
      }
    }
    __syncthreads();  // os complete

    // 3. gated RMSNorm over the head's 128 outputs (warps 0..3)
    if (tid < 128) {
      const float o = os[c];
      const float ss = warp_sum(o * o);
      if (lane == 0) red8[warp] = ss;
    }
    __syncthreads();
    if (tid < 128) {
      const float tot = red8[0] + red8[1] + red8[2] + red8[3];
      const float rms = rsqrtf(tot / 128.f + a.eps);
      const float hs = a.head_scale ? a.head_scale[h] : 1.f;
      static_cast<T*>(a.o)[(long)b * a.o_stride + h * 128 + c] = from_f<T>(os[c] * rms * a.norm_w[c] * silu_t<T>(z) * hs);
    }
    __syncthreads();  // qs / ks / vs / os / red8 are rewritten by the next item
  }
  cp_wait<0>();
}

int launch_gdn_decode(const GdnConvArgs& ca, const GdnScanArgs& a, int dtype, cudaStream_t st) {
  if (a.b == 0) return DUO_OK;
  if (a.t != 1 || ca.t != 1) return fail(DUO_EINVAL, "gdn_decode: one token per row");
  if (a.dk != 128 || a.dv != 128 || ca.ks != 4 || ca.hk != ca.hv || !a.norm_w)
    return fail(DUO_EINVAL, "gdn_decode: needs dk = dv = 128, ks = 4, hk == hv and the gated norm");
  const int items = a.b * a.h;
  const int slots = DEC_CPS * sm_count();
  // as many CTAs as fit, trimmed so that the busiest CTA's item count is unchanged
  const int per = cdiv(items, slots);
  const int grid = cdiv(items, per);
  return with_act(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    DUO_TRY(ensure_smem_attr(gdn_decode_kernel<T>, DEC_SMEM));
    DUO_CUDA_TRY(::duo::launch_kernel(gdn_decode_kernel<T>, grid, DEC_THREADS, DEC_SMEM, st, ca, a));
    DUO_LAUNCH_CHECK("gdn_decode_kernel");
    return DUO_OK;
  });
}

static int check_gdn_op(const void* q, const void* k, const void* v, int in_dtype, const float* g, const float* beta,
                        float* state, void* o, int o_dtype, int b, int t, int h, int dk, int dv) {
  DUO_CHECK_ARG(b >= 0 && t >= 0 && h > 0, "gdn: bad shape");
  DUO_CHECK_ARG(dk == 128 && dv == 128, "gdn: dk and dv must be 128");
  DUO_CHECK_ARG(valid_act(in_dtype) && o_dtype == in_dtype, "gdn: q/k/v/o dtype must be f32, bf16 or f16 (the same)");
  DUO_CHECK_ARG(b == 0 || t == 0 || (q && k && v && g && beta && state && o), "gdn: null pointer");
  return DUO_OK;
}

GdnScanArgs op_scan_args(const void* q, const void* k, const void* v, const float* g, const float* beta,
                         float* state, void* o, int b, int t, int h, int l2norm_qk) {
  GdnScanArgs a{};
  a.q = q; a.k = k; a.v = v;
  a.q_stride = a.k_stride = a.v_stride = a.o_stride = (long)h * 128;
  a.g = g; a.beta = beta; a.state = state; a.state_row0 = 0; a.o = o;
  a.b = b; a.t = t; a.hq = h; a.h = h; a.dk = 128; a.dv = 128;
  a.l2norm_qk = l2norm_qk;
  return a;
}

}  // namespace duo

using namespace duo;

extern "C" int duo_gdn_recurrent_fwd(const void* q, const void* k, const void* v, int in_dtype, const float* g,
                                     const float* beta, float* state, void* o, int o_dtype, int b, int t, int h,
                                     int dk, int dv, int l2norm_qk, duo_stream stream) {
  DUO_TRY(check_gdn_op(q, k, v, in_dtype, g, beta, state, o, o_dtype, b, t, h, dk, dv));
  return launch_gdn_recurrent(op_scan_args(q, k, v, g, beta, state, o, b, t, h, l2norm_qk), in_dtype,
                              as_stream(stream));
}

extern "C" int duo_gdn_conv_fwd(const void* y, int dtype, int w, const float* conv_w, float* conv_state,
                                const float* a_log, const float* dt_bias, void* qkv, float* g, float* beta, int b,
                                int t, int hk, int hv, int dk, int dv, duo_stream stream) {
  DUO_CHECK_ARG(valid_act(dtype), "gdn_conv: dtype must be f32, bf16 or f16");
  DUO_CHECK_ARG(dk == 128 && dv == 128, "gdn_conv: dk and dv must be 128");
  DUO_CHECK_ARG(b >= 0 && t >= 0 && hk > 0 && hv > 0 && hv % hk == 0, "gdn_conv: bad shape");
  const long conv_dim = 2L * hk * dk + (long)hv * dv;
  DUO_CHECK_ARG(w >= conv_dim + (long)hv * dv + 2L * hv, "gdn_conv: w must hold [q k v | z | b | a]");
  if (b == 0 || t == 0) return DUO_OK;
  DUO_CHECK_ARG(y && conv_w && conv_state && a_log && dt_bias && qkv && g && beta, "gdn_conv: null pointer");
  GdnConvArgs a{};
  a.y = y; a.w = w; a.conv_w = conv_w; a.conv_state = conv_state; a.a_log = a_log; a.dt_bias = dt_bias;
  a.qkv_out = qkv; a.g_out = g; a.beta_out = beta;
  a.hk = hk; a.hv = hv; a.dk = dk; a.dv = dv; a.ks = CONV_KS;
  a.rows = b; a.t = t; a.row_base = 0;
  return launch_gdn_conv(a, dtype, as_stream(stream));
}
