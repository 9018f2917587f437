// Gated DeltaNet token mixer, part 2: the chunked (WY / UT-transform) scan for prefill.
//
// Chunk form of the gated delta rule, as published with the PyTorch path the reference runs (transformers
// torch_chunk_gated_delta_rule, chunk 64).  Per chunk of C = 64 tokens with cumulative log-decay G (inclusive cumsum
// of g inside the chunk):
//   L[i, j] = beta_i (k_i . k_j) exp(G_i - G_j) for j < i,   T = (I + L)^-1            (unit lower triangular)
//   U = T diag(beta) V,   W = T diag(beta e^G) K
//   V' = U - W S,   O = diag(e^G) Q S + tril(Q K^T * exp(G_i - G_j)) V'
//   S <- e^{G_63} S + (diag(e^{G_63 - G}) K)^T V'
// Everything up to W and the masked Q K^T depends only on the chunk itself, so it runs in a first kernel with one CTA
// per (chunk, head, row) -- thousands of independent CTAs, two per SM -- that writes T diag(beta), W and
// A = tril(Q K^T * decay) for every chunk to a workspace (32 KiB per chunk, f16).  The second kernel keeps the
// recurrence: one CTA (8 warps) per (row, value head) walks the chunks in order computing U = T diag(beta) V,
// V' = U - W S, the output and the state update, with 4 block barriers per chunk.  All products run on the tensor
// cores (f16 operands, f32 accumulation; f16 keeps 8x more mantissa than bf16 for these normalised, decay-bounded
// intermediates); the state lives in registers as f32 accumulators for the whole sequence and is rounded to f16
// only as an operand copy.  T is formed by blocked forward substitution: the 16 x 16 diagonal blocks in f32 (registers
// and shuffles), then the off-diagonal blocks by distance as 16 x 16 tensor-core products.  The gated RMSNorm of the
// engine path is fused into the output.
#include <mutex>
#include <type_traits>

#include "kernels.cuh"
#include "mma.cuh"

namespace duo {

namespace {

constexpr int CK = 64;         // chunk length
constexpr int PD = 128 + 8;    // pitch (elements) of the 128-wide f16 tiles
constexpr int PC = 64 + 8;     // pitch of the 64-wide f16 tiles
constexpr int PF = 64 + 1;     // pitch of the f32 64 x 64 tiles

constexpr long CHUNK_WS = 64 * 64 * 2 * 2 + 64 * 128 * 2;  // per chunk: T1 [64][64], A [64][64], W [64][128] f16

struct PrepSmem {
  __half q[CK * PD], k[CK * PD];  // chunk inputs (q scaled by 1/sqrt(dk))
  __half t2[CK * PC];              // T diag(beta e^G)
  __half lh[CK * PC], th[CK * PC];  // f16 copies of L and T for the off-diagonal block products
  __half xh[3 * 16 * 24];          // per-warp 16 x 16 scratch of the off-diagonal solve
  float a[CK * PF];                // L (strictly lower), f32
  float t[CK * PF];                // T = (I + L)^-1, f32
  float gcum[CK], eg[CK], beta[CK];
};

struct ScanSmem {
  __half q[CK * PD], k[CK * PD], v[CK * PD];  // chunk inputs (q scaled by 1/sqrt(dk))
  __half w[CK * PD];                          // W (from the prep kernel)
  __half vn[CK * PD];                         // V'
  __half vd[CK * PD];                         // diag(e^{G_63 - G}) V'
  __half s[128 * PD];                         // f16 copy of the state [dk][dv]
  __half aq[CK * PC];                         // tril(Q K^T) * decay (from the prep kernel)
  __half t1[CK * PC];                         // T diag(beta) (from the prep kernel)
  float gcum[CK], eg[CK], egl[CK];
  float rowss[2][CK];                         // gated-norm partial sums (two column halves)
};

template <typename T> __device__ __forceinline__ void ld4f(const T* p, float* o);
template <> __device__ __forceinline__ void ld4f<float>(const float* p, float* o) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
}
template <> __device__ __forceinline__ void ld4f<__nv_bfloat16>(const __nv_bfloat16* p, float* o) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
}
template <> __device__ __forceinline__ void ld4f<__half>(const __half* p, float* o) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
}

__device__ __forceinline__ void st4h(__half* p, const float* v) {
  uint2 u;
  u.x = wm::pack_f16(v[0], v[1]);
  u.y = wm::pack_f16(v[2], v[3]);
  *reinterpret_cast<uint2*>(p) = u;
}


// chunk inputs -> shared memory: warp w takes token rows w, w + 8, ..., 4 values per lane, every load issued before
// any is used; q and k optionally l2-normalised, q scaled by 1/sqrt(dk); padded tokens are zero
template <typename TI>
__device__ __forceinline__ void load_chunk_qk(const GdnScanArgs& a, int b, int kh, int t0, __half* sq, __half* sk,
                                              int warp, int lane) {
  using Raw = typename std::conditional<sizeof(TI) == 4, uint4, uint2>::type;  // 4 values of TI
  const TI* qp = static_cast<const TI*>(a.q);
  const TI* kp = static_cast<const TI*>(a.k);
  const float qscale = rsqrtf(128.f);
  Raw rq[8], rk[8];
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int t = t0 + warp + 8 * i;
    if (t < a.t) {
      const long m = (long)b * a.t + t;
      rq[i] = *reinterpret_cast<const Raw*>(qp + m * a.q_stride + kh * 128 + lane * 4);
      rk[i] = *reinterpret_cast<const Raw*>(kp + m * a.k_stride + kh * 128 + lane * 4);
    }
  }
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int r = warp + 8 * i, t = t0 + r;
    float qv[4] = {0, 0, 0, 0}, kv[4] = {0, 0, 0, 0};
    if (t < a.t) {
      ld4f(reinterpret_cast<const TI*>(&rq[i]), qv);
      ld4f(reinterpret_cast<const TI*>(&rk[i]), kv);
      if (a.l2norm_qk) {
        const float sq2 = warp_sum(qv[0] * qv[0] + qv[1] * qv[1] + qv[2] * qv[2] + qv[3] * qv[3]);
        const float sk2 = warp_sum(kv[0] * kv[0] + kv[1] * kv[1] + kv[2] * kv[2] + kv[3] * kv[3]);
        const float iq = rsqrtf(sq2 + 1e-6f), ik = rsqrtf(sk2 + 1e-6f);
#pragma unroll
        for (int e = 0; e < 4; e++) { qv[e] *= iq; kv[e] *= ik; }
      }
#pragma unroll
      for (int e = 0; e < 4; e++) qv[e] *= qscale;
    }
    st4h(sq + r * PD + lane * 4, qv);
    st4h(sk + r * PD + lane * 4, kv);
  }
}

// inclusive cumulative log-decay of the chunk (warp 0): gcum <- cumsum, eg <- e^G, egl <- e^{G_63 - G}
__device__ __forceinline__ void chunk_decay(float* gcum, float* eg, float* egl, int lane) {
  const float g0 = gcum[2 * lane], g1 = gcum[2 * lane + 1];
  float s = g0 + g1;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float n = __shfl_up_sync(0xffffffffu, s, o);
    if (lane >= o) s += n;
  }
  const float excl = s - g0 - g1;
  const float G0 = excl + g0, G1 = excl + g0 + g1;
  const float Gl = __shfl_sync(0xffffffffu, G1, 31);
  gcum[2 * lane] = G0;
  gcum[2 * lane + 1] = G1;
  eg[2 * lane] = expf(G0);
  eg[2 * lane + 1] = expf(G1);
  if (egl) {
    egl[2 * lane] = expf(Gl - G0);
    egl[2 * lane + 1] = expf(Gl - G1);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// kernel 1: per (chunk, head, row): T diag(beta), W = T diag(beta e^G) K and A = tril(Q K^T * decay) -> workspace

template <typename TI>
__global__ void __launch_bounds__(256, 2) gdn_chunk_prep_kernel(GdnScanArgs a) {
  pdl_enter();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  PrepSmem& sm = *reinterpret_cast<PrepSmem*>(smem_raw);
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q4 = lane & 3;
  const int kh = h / (a.h / a.hq);
  const int nch = gridDim.x, t0 = c * CK;
  uint8_t* ws = static_cast<uint8_t*>(a.chunk_ws) + (((long)b * a.h + h) * nch + c) * CHUNK_WS;
  __half* gT1 = reinterpret_cast<__half*>(ws);
  __half* gA = gT1 + CK * CK;
  __half* gW = gA + CK * CK;

  load_chunk_qk<TI>(a, b, kh, t0, sm.q, sm.k, warp, lane);
  if (tid < CK) {
    const int t = t0 + tid;
    const long m = (long)b * a.t + t;
    sm.gcum[tid] = t < a.t ? a.g[m * a.h + h] : 0.f;
    sm.beta[tid] = t < a.t ? a.beta[m * a.h + h] : 0.f;
  }
  __syncthreads();
  if (warp == 0) chunk_decay(sm.gcum, sm.eg, nullptr, lane);
  // Q K^T and K K^T, 64 x 64 each: warp tile 16 rows x 32 columns
  float qk[4][4], kk[4][4];
  const int wr = (warp & 3) * 16, wc = (warp >> 2) * 32;
  {
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
      for (int e = 0; e < 4; e++) qk[j][e] = kk[j][e] = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < 128; k0 += 16) {
      uint32_t aq[4], ak[4], bf[2][4];
      wm::lda(aq, sm.q, PD, wr, k0);
      wm::lda(ak, sm.k, PD, wr, k0);
      wm::ldb_nk(bf[0], sm.k, PD, wc, k0);
      wm::ldb_nk(bf[1], sm.k, PD, wc + 16, k0);
#pragma unroll
      for (int jj = 0; jj < 2; jj++) {
        wm::mma_f16(qk[2 * jj], aq, bf[jj]);
        wm::mma_f16(qk[2 * jj + 1], aq, bf[jj] + 2);
        wm::mma_f16(kk[2 * jj], ak, bf[jj]);
        wm::mma_f16(kk[2 * jj + 1], ak, bf[jj] + 2);
      }
    }
  }
  __syncthreads();  // G ready
#pragma unroll
  for (int j = 0; j < 4; j++) {
#pragma unroll
    for (int hf = 0; hf < 2; hf++) {
      const int i = wr + g + hf * 8, jc = wc + 8 * j + 2 * q4;
      float av[2], lv[2];
#pragma unroll
      for (int e2 = 0; e2 < 2; e2++) {
        const int jj = jc + e2;
        const float dec = jj <= i ? expf(sm.gcum[i] - sm.gcum[jj]) : 0.f;
        lv[e2] = jj < i ? sm.beta[i] * kk[j][hf * 2 + e2] * dec : 0.f;
        sm.a[i * PF + jj] = lv[e2];
        sm.t[i * PF + jj] = 0.f;
        av[e2] = qk[j][hf * 2 + e2] * dec;
      }
      *reinterpret_cast<uint32_t*>(gA + i * CK + jc) = wm::pack_f16(av[0], av[1]);
      *reinterpret_cast<uint32_t*>(sm.lh + i * PC + jc) = wm::pack_f16(lv[0], lv[1]);
      *reinterpret_cast<uint32_t*>(sm.th + i * PC + jc) = 0u;
    }
  }
  __syncthreads();
  // ---- T = (I + L)^-1.  The four 16 x 16 diagonal blocks by forward substitution in f32: 4 threads per column
  // (column = tid / 4 of the 64), thread `sub` keeping rows sub, sub + 4, ... of its column in registers and the
  // partial dot products combined by two shuffles.
  {
    const int col = tid >> 2, sub = tid & 3, o = (col >> 4) * 16, cl = col & 15;
    float tr[4] = {0.f, 0.f, 0.f, 0.f};  // T[o + 4u + sub][o + cl]
#pragma unroll
    for (int i = 0; i < 16; i++) {
      float part = 0.f;
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int j = 4 * u + sub;
        if (j < i) part += sm.a[(o + i) * PF + o + j] * tr[u];
      }
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      const float v = (i == cl ? 1.f : 0.f) - part;
      if ((i & 3) == sub) tr[i >> 2] = v;
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int r = o + 4 * u + sub;
      sm.t[r * PF + o + cl] = tr[u];
      sm.th[r * PC + o + cl] = __float2half_rn(tr[u]);
    }
  }
  __syncthreads();
  // ... then the off-diagonal blocks by distance d on the tensor cores (f16 operands, f32 accumulation; T is rounded
  // to f16 for its uses anyway): T[bi][bj] = -T[bi][bi] (sum_{bj <= bk < bi} L[bi][bk] T[bk][bj]), warp bj of 4 - d
  for (int d = 1; d < 4; d++) {
    if (warp < 4 - d) {
      const int bj = warp, bi = warp + d;
      float X[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      for (int bk = bj; bk < bi; bk++) {
        uint32_t af[4], bf[4];
        wm::lda(af, sm.lh, PC, bi * 16, bk * 16);
        wm::ldb_kn(bf, sm.th, PC, bj * 16, bk * 16);
        wm::mma_f16(X[0], af, bf);
        wm::mma_f16(X[1], af, bf + 2);
      }
      __half* xh = sm.xh + warp * 16 * 24;
#pragma unroll
      for (int h2 = 0; h2 < 2; h2++) {
        *reinterpret_cast<uint32_t*>(xh + g * 24 + h2 * 8 + 2 * q4) = wm::pack_f16(X[h2][0], X[h2][1]);
        *reinterpret_cast<uint32_t*>(xh + (g + 8) * 24 + h2 * 8 + 2 * q4) = wm::pack_f16(X[h2][2], X[h2][3]);
      }
      __syncwarp();
      float Y[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      {
        uint32_t af[4], bf[4];
        wm::lda(af, sm.th, PC, bi * 16, bi * 16);
        wm::ldb_kn(bf, xh, 24, 0, 0);
        wm::mma_f16(Y[0], af, bf);
        wm::mma_f16(Y[1], af, bf + 2);
      }
#pragma unroll
      for (int h2 = 0; h2 < 2; h2++) {
        const int cc = bj * 16 + h2 * 8 + 2 * q4;
        const int r0 = bi * 16 + g, r1 = r0 + 8;
        sm.t[r0 * PF + cc] = -Y[h2][0];
        sm.t[r0 * PF + cc + 1] = -Y[h2][1];
        sm.t[r1 * PF + cc] = -Y[h2][2];
        sm.t[r1 * PF + cc + 1] = -Y[h2][3];
        *reinterpret_cast<uint32_t*>(sm.th + r0 * PC + cc) = wm::pack_f16(-Y[h2][0], -Y[h2][1]);
        *reinterpret_cast<uint32_t*>(sm.th + r1 * PC + cc) = wm::pack_f16(-Y[h2][2], -Y[h2][3]);
      }
    }
    __syncthreads();
  }
  // T1 = T diag(beta) -> workspace, T2 = T diag(beta e^G) in f16
  for (int e = tid; e < CK * CK / 2; e += 256) {
    const int i = (2 * e) >> 6, j = (2 * e) & 63;
    const float t0v = sm.t[i * PF + j], t1v = sm.t[i * PF + j + 1];
    reinterpret_cast<uint32_t*>(gT1)[e] = wm::pack_f16(t0v * sm.beta[j], t1v * sm.beta[j + 1]);
    *reinterpret_cast<uint32_t*>(sm.t2 + i * PC + j) =
        wm::pack_f16(t0v * sm.beta[j] * sm.eg[j], t1v * sm.beta[j + 1] * sm.eg[j + 1]);
  }
  __syncthreads();
  // ---- W = T2 K (64 x 128, K = 64): warp tile 16 rows x 64 columns -> workspace
  {
    const int wr2 = (warp & 3) * 16, wc2 = (warp >> 2) * 64;
    float Wt[8][4];
#pragma unroll
    for (int j = 0; j < 8; j++)
#pragma unroll
      for (int e = 0; e < 4; e++) Wt[j][e] = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < CK; k0 += 16) {
      uint32_t a2[4];
      wm::lda(a2, sm.t2, PC, wr2, k0);
#pragma unroll
      for (int jj = 0; jj < 4; jj++) {
        uint32_t bk[4];
        wm::ldb_kn(bk, sm.k, PD, wc2 + 16 * jj, k0);
        wm::mma_f16(Wt[2 * jj], a2, bk);
        wm::mma_f16(Wt[2 * jj + 1], a2, bk + 2);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int cc = wc2 + 8 * j + 2 * q4;
      *reinterpret_cast<uint32_t*>(gW + (wr2 + g) * 128 + cc) = wm::pack_f16(Wt[j][0], Wt[j][1]);
      *reinterpret_cast<uint32_t*>(gW + (wr2 + g + 8) * 128 + cc) = wm::pack_f16(Wt[j][2], Wt[j][3]);
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// kernel 2: per (row, value head) the recurrence over the chunks

template <typename TI, bool NORM>
__global__ void __launch_bounds__(256, 1) gdn_chunk_scan_kernel(GdnScanArgs a) {
  pdl_enter();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  ScanSmem& sm = *reinterpret_cast<ScanSmem*>(smem_raw);
  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q4 = lane & 3;
  const int kh = h / (a.h / a.hq);
  const TI* vp = static_cast<const TI*>(a.v);
  float* Sg = a.state + (((long)(a.state_row0 + b) * a.h + h) * 128) * 128;
  const int nchunks = (a.t + CK - 1) / CK;
  const uint8_t* wsb = static_cast<const uint8_t*>(a.chunk_ws) + ((long)b * a.h + h) * nchunks * CHUNK_WS;

  // state: warp w owns dk rows 16w .. 16w + 15, all 128 dv columns (16 n-tiles of 8)
  float S[16][4];
  {
    const int r0 = warp * 16 + g;
#pragma unroll
    for (int j = 0; j < 16; j++) {
      const int c = 8 * j + 2 * q4;
      const float2 lo = *reinterpret_cast<const float2*>(Sg + (long)r0 * 128 + c);
      const float2 hi = *reinterpret_cast<const float2*>(Sg + (long)(r0 + 8) * 128 + c);
      S[j][0] = lo.x; S[j][1] = lo.y; S[j][2] = hi.x; S[j][3] = hi.y;
      *reinterpret_cast<uint32_t*>(sm.s + r0 * PD + c) = wm::pack_f16(lo.x, lo.y);
      *reinterpret_cast<uint32_t*>(sm.s + (r0 + 8) * PD + c) = wm::pack_f16(hi.x, hi.y);
    }
  }

  const int wr = (warp & 3) * 16, wc = (warp >> 2) * 64;
  for (int c = 0; c < nchunks; c++) {
    const int t0 = c * CK;
    __syncthreads();  // previous chunk's readers are done with every tile
    // ---- the chunk: q, k, v, the prep kernel's T1, A, W, g and this thread's gate values z.  Every global load is
    // issued before any is used, so the chunk pays one memory latency rather than one per row.
    using Raw = typename std::conditional<sizeof(TI) == 4, uint4, uint2>::type;  // 4 values of TI
    Raw rq[8], rk[8], rv[8];
    uint4 rw[8];
    uint32_t rz[16];
    float gv = 0.f;
    {
      const TI* qp = static_cast<const TI*>(a.q);
      const TI* kp = static_cast<const TI*>(a.k);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const int t = t0 + warp + 8 * i;
        if (t < a.t) {
          const long m = (long)b * a.t + t;
          rq[i] = *reinterpret_cast<const Raw*>(qp + m * a.q_stride + kh * 128 + lane * 4);
          rk[i] = *reinterpret_cast<const Raw*>(kp + m * a.k_stride + kh * 128 + lane * 4);
          rv[i] = *reinterpret_cast<const Raw*>(vp + m * a.v_stride + h * 128 + lane * 4);
        }
      }
      const uint4* src = reinterpret_cast<const uint4*>(wsb + (long)c * CHUNK_WS);
#pragma unroll
      for (int i = 0; i < 8; i++) rw[i] = src[tid + 256 * i];  // T1 and A (i < 4), then W
      if (tid < CK && t0 + tid < a.t) gv = a.g[((long)b * a.t + t0 + tid) * a.h + h];
      if (NORM) {
        const TI* zp = static_cast<const TI*>(a.z);
#pragma unroll
        for (int half = 0; half < 2; half++) {
          const int t = t0 + wr + g + half * 8;
          const long m = (long)b * a.t + min(t, a.t - 1);
#pragma unroll
          for (int j = 0; j < 8; j++) {
            const int cc = wc + 8 * j + 2 * q4;
            float z0 = to_f(zp[m * a.z_stride + h * 128 + cc]), z1 = to_f(zp[m * a.z_stride + h * 128 + cc + 1]);
            rz[half * 8 + j] = wm::pack_f16(silu16_(z0), silu16_(z1));
          }
        }
      }
    }
    {
      const float qscale = rsqrtf(128.f);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const int r = warp + 8 * i, t = t0 + r;
        float qv[4] = {0, 0, 0, 0}, kv[4] = {0, 0, 0, 0}, vv[4] = {0, 0, 0, 0};
        if (t < a.t) {
          ld4f(reinterpret_cast<const TI*>(&rq[i]), qv);
          ld4f(reinterpret_cast<const TI*>(&rk[i]), kv);
          ld4f(reinterpret_cast<const TI*>(&rv[i]), vv);
          if (a.l2norm_qk) {
            const float sq = warp_sum(qv[0] * qv[0] + qv[1] * qv[1] + qv[2] * qv[2] + qv[3] * qv[3]);
            const float sk = warp_sum(kv[0] * kv[0] + kv[1] * kv[1] + kv[2] * kv[2] + kv[3] * kv[3]);
            const float iq = rsqrtf(sq + 1e-6f), ik = rsqrtf(sk + 1e-6f);
#pragma unroll
            for (int e = 0; e < 4; e++) { qv[e] *= iq; kv[e] *= ik; }
          }
#pragma unroll
          for (int e = 0; e < 4; e++) qv[e] *= qscale;
        }
        st4h(sm.q + r * PD + lane * 4, qv);
        st4h(sm.k + r * PD + lane * 4, kv);
        st4h(sm.v + r * PD + lane * 4, vv);
      }
#pragma unroll
      for (int i = 0; i < 4; i++) {  // T1 and A: 64 rows x 128 bytes each
        const int e = tid + 256 * i, which = e >> 9, r = (e >> 3) & 63, cc = (e & 7) * 8;
        *reinterpret_cast<uint4*>((which ? sm.aq : sm.t1) + r * PC + cc) = rw[i];
      }
#pragma unroll
      for (int i = 0; i < 4; i++) {  // W: 64 rows x 256 bytes
        const int e = tid + 256 * i, r = e >> 4, cc = (e & 15) * 8;
        *reinterpret_cast<uint4*>(sm.w + r * PD + cc) = rw[4 + i];
      }
      if (tid < CK) sm.gcum[tid] = gv;
    }
    __syncthreads();
    if (warp == 0) chunk_decay(sm.gcum, sm.eg, sm.egl, lane);
    // ---- U = T1 V; W S and Q S (one pass over the state copy)
    float U[8][4], Wt[8][4], O[8][4];
#pragma unroll
    for (int j = 0; j < 8; j++)
#pragma unroll
      for (int e = 0; e < 4; e++) U[j][e] = Wt[j][e] = O[j][e] = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < CK; k0 += 16) {
      uint32_t a1[4];
      wm::lda(a1, sm.t1, PC, wr, k0);
#pragma unroll
      for (int jj = 0; jj < 4; jj++) {
        uint32_t bv[4];
        wm::ldb_kn(bv, sm.v, PD, wc + 16 * jj, k0);
        wm::mma_f16(U[2 * jj], a1, bv);
        wm::mma_f16(U[2 * jj + 1], a1, bv + 2);
      }
    }
#pragma unroll
    for (int k0 = 0; k0 < 128; k0 += 16) {
      uint32_t aw[4], aq2[4];
      wm::lda(aw, sm.w, PD, wr, k0);
      wm::lda(aq2, sm.q, PD, wr, k0);
#pragma unroll
      for (int jj = 0; jj < 4; jj++) {
        uint32_t bs[4];
        wm::ldb_kn(bs, sm.s, PD, wc + 16 * jj, k0);
        wm::mma_f16(Wt[2 * jj], aw, bs);
        wm::mma_f16(Wt[2 * jj + 1], aw, bs + 2);
        wm::mma_f16(O[2 * jj], aq2, bs);
        wm::mma_f16(O[2 * jj + 1], aq2, bs + 2);
      }
    }
    __syncthreads();  // e^G ready
    // ---- V' = U - W S; O = diag(e^G) Q S
    {
      const float e0 = sm.eg[wr + g], e1 = sm.eg[wr + g + 8];
      const float l0 = sm.egl[wr + g], l1 = sm.egl[wr + g + 8];
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int cc = wc + 8 * j + 2 * q4;
        const float v0 = U[j][0] - Wt[j][0], v1 = U[j][1] - Wt[j][1];
        const float v2 = U[j][2] - Wt[j][2], v3 = U[j][3] - Wt[j][3];
        *reinterpret_cast<uint32_t*>(sm.vn + (wr + g) * PD + cc) = wm::pack_f16(v0, v1);
        *reinterpret_cast<uint32_t*>(sm.vn + (wr + g + 8) * PD + cc) = wm::pack_f16(v2, v3);
        *reinterpret_cast<uint32_t*>(sm.vd + (wr + g) * PD + cc) = wm::pack_f16(v0 * l0, v1 * l0);
        *reinterpret_cast<uint32_t*>(sm.vd + (wr + g + 8) * PD + cc) = wm::pack_f16(v2 * l1, v3 * l1);
        O[j][0] *= e0; O[j][1] *= e0; O[j][2] *= e1; O[j][3] *= e1;
      }
    }
    __syncthreads();
    // ---- O += tril(QK^T decay) V' (K = 64)
#pragma unroll
    for (int k0 = 0; k0 < CK; k0 += 16) {
      uint32_t aa[4];
      wm::lda(aa, sm.aq, PC, wr, k0);
#pragma unroll
      for (int jj = 0; jj < 4; jj++) {
        uint32_t bv[4];
        wm::ldb_kn(bv, sm.vn, PD, wc + 16 * jj, k0);
        wm::mma_f16(O[2 * jj], aa, bv);
        wm::mma_f16(O[2 * jj + 1], aa, bv + 2);
      }
    }
    // ---- state update S = e^{G_63} S + K^T diag(e^{G_63 - G}) V' (128 x 128, K = 64); rows 16w ..
    {
      const float el = sm.eg[CK - 1];
#pragma unroll
      for (int j = 0; j < 16; j++)
#pragma unroll
        for (int e = 0; e < 4; e++) S[j][e] *= el;
#pragma unroll
      for (int k0 = 0; k0 < CK; k0 += 16) {
        uint32_t ak[4];
        wm::lda_t(ak, sm.k, PD, warp * 16, k0);
#pragma unroll
        for (int jj = 0; jj < 8; jj++) {
          uint32_t bv[4];
          wm::ldb_kn(bv, sm.vd, PD, 16 * jj, k0);
          wm::mma_f16(S[2 * jj], ak, bv);
          wm::mma_f16(S[2 * jj + 1], ak, bv + 2);
        }
      }
    }
    // ---- output rows (optionally the gated RMSNorm over the 128 columns of the head)
    if (NORM) {
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        s0 += O[j][0] * O[j][0] + O[j][1] * O[j][1];
        s1 += O[j][2] * O[j][2] + O[j][3] * O[j][3];
      }
      s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
      s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
      s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
      s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
      if (q4 == 0) {
        sm.rowss[warp >> 2][wr + g] = s0;
        sm.rowss[warp >> 2][wr + g + 8] = s1;
      }
    }
    __syncthreads();  // every warp is past its reads of sm.s; row sums are in
    // write the new f16 state copy for the next chunk
    {
      const int r0 = warp * 16 + g;
#pragma unroll
      for (int j = 0; j < 16; j++) {
        const int cc = 8 * j + 2 * q4;
        *reinterpret_cast<uint32_t*>(sm.s + r0 * PD + cc) = wm::pack_f16(S[j][0], S[j][1]);
        *reinterpret_cast<uint32_t*>(sm.s + (r0 + 8) * PD + cc) = wm::pack_f16(S[j][2], S[j][3]);
      }
    }
    {
      TI* op = static_cast<TI*>(a.o);
      const float hs = (NORM && a.head_scale) ? a.head_scale[h] : 1.f;
#pragma unroll
      for (int half = 0; half < 2; half++) {
        const int i = wr + g + half * 8;
        const int t = t0 + i;
        if (t >= a.t) continue;
        const long m = (long)b * a.t + t;
        float rms = 1.f;
        if (NORM) rms = rsqrtf((sm.rowss[0][i] + sm.rowss[1][i]) / 128.f + a.eps);
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const int cc = wc + 8 * j + 2 * q4;
          float o0 = O[j][half * 2], o1 = O[j][half * 2 + 1];
          if (NORM) {
            const float2 sz = __half22float2(*reinterpret_cast<const __half2*>(&rz[half * 8 + j]));
            o0 = o0 * rms * a.norm_w[cc] * sz.x * hs;
            o1 = o1 * rms * a.norm_w[cc + 1] * sz.y * hs;
          }
          op[m * a.o_stride + h * 128 + cc] = from_f<TI>(o0);
          op[m * a.o_stride + h * 128 + cc + 1] = from_f<TI>(o1);
        }
      }
    }
  }
  // final state (f32)
  {
    const int r0 = warp * 16 + g;
#pragma unroll
    for (int j = 0; j < 16; j++) {
      const int cc = 8 * j + 2 * q4;
      *reinterpret_cast<float2*>(Sg + (long)r0 * 128 + cc) = make_float2(S[j][0], S[j][1]);
      *reinterpret_cast<float2*>(Sg + (long)(r0 + 8) * 128 + cc) = make_float2(S[j][2], S[j][3]);
    }
  }
}

template <typename TI, bool NORM>
static int run_chunk(const GdnScanArgs& a, cudaStream_t st) {
  const int smem_p = (int)sizeof(PrepSmem), smem_s = (int)sizeof(ScanSmem);
  DUO_TRY(ensure_smem_attr(gdn_chunk_prep_kernel<TI>, smem_p));
  DUO_TRY(ensure_smem_attr(gdn_chunk_scan_kernel<TI, NORM>, smem_s));
  const int nch = (a.t + CK - 1) / CK;
  DUO_CUDA_TRY(::duo::launch_kernel(gdn_chunk_prep_kernel<TI>, dim3(nch, a.h, a.b), 256, smem_p, st, a));
  DUO_LAUNCH_CHECK("gdn_chunk_prep_kernel");
  DUO_CUDA_TRY(::duo::launch_kernel(gdn_chunk_scan_kernel<TI, NORM>, dim3(a.h, a.b), 256, smem_s, st, a));
  DUO_LAUNCH_CHECK("gdn_chunk_scan_kernel");
  return DUO_OK;
}

}  // namespace

long gdn_chunk_ws_bytes(int b, int t, int h) { return (long)b * h * ((t + CK - 1) / CK) * CHUNK_WS; }

static bool chunk_tc_enabled() {
  static const bool on = [] {
    const char* v = getenv("DUO_CHUNK_TC");
    return !(v && v[0] == '0');
  }();
  return on;
}

static bool short_scan_enabled() {
  static const bool on = [] {
    const char* v = getenv("DUO_SHORT_SCAN");
    return !(v && v[0] == '0');
  }();
  return on;
}

int launch_gdn_chunk(const GdnScanArgs& a, int dtype, cudaStream_t st) {
  if (a.b == 0 || a.t == 0) return DUO_OK;
  if (a.dk != 128 || a.dv != 128) return fail(DUO_EINVAL, "gdn_chunk: needs dk = dv = 128");
  if (a.hq <= 0 || a.h % a.hq) return fail(DUO_EINVAL, "gdn_chunk: value heads must be a multiple of q/k heads");
  // up to 16 tokens per row (16-bit, no l2norm option): token by token with the state in registers, which beats a
  // mostly empty 64-token chunk (DUO_SHORT_SCAN=0 keeps the chunk kernels)
  if (a.t <= 16 && !a.l2norm_qk && (dtype == DUO_BF16 || dtype == DUO_F16) && short_scan_enabled())
    return launch_gdn_short(a, dtype, st);
  // 16-bit inputs without the l2norm option: the tcgen05 kernel (no workspace); DUO_CHUNK_TC=0 keeps the warp-level
  // two-kernel form, which also serves f32 inputs and l2norm_qk
  if (chunk_tc_enabled() && gdn_chunk_tc_eligible(a, dtype)) return launch_gdn_chunk_tc(a, dtype, st);
  if ((a.q_stride | a.k_stride | a.v_stride) % 4)
    return fail(DUO_EINVAL, "gdn_chunk: q/k/v token strides must be multiples of 4 elements");
  if (!a.chunk_ws || a.chunk_ws_bytes < gdn_chunk_ws_bytes(a.b, a.t, a.h))
    return fail(DUO_EINVAL, "gdn_chunk: workspace too small");
  const bool norm = a.norm_w != nullptr;
  return with_act(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    return norm ? run_chunk<T, true>(a, st) : run_chunk<T, false>(a, st);
  });
}

// library-owned chunk workspace for the op-level entry point (grown on demand)
static void* g_chunk_ws = nullptr;
static long g_chunk_ws_bytes = 0;
static std::mutex g_chunk_ws_mu;

}  // namespace duo

using namespace duo;

extern "C" int duo_gdn_chunk_fwd(const void* q, const void* k, const void* v, int in_dtype, const float* g,
                                 const float* beta, float* state, void* o, int o_dtype, int b, int t, int h, int dk,
                                 int dv, int l2norm_qk, duo_stream stream) {
  DUO_CHECK_ARG(b >= 0 && t >= 0 && h > 0, "gdn_chunk: bad shape");
  DUO_CHECK_ARG(dk == 128 && dv == 128, "gdn_chunk: dk and dv must be 128");
  DUO_CHECK_ARG(valid_act(in_dtype) && o_dtype == in_dtype,
                "gdn_chunk: q/k/v/o dtype must be f32, bf16 or f16 (the same)");
  DUO_CHECK_ARG(b == 0 || t == 0 || (q && k && v && g && beta && state && o), "gdn_chunk: null pointer");
  GdnScanArgs a = op_scan_args(q, k, v, g, beta, state, o, b, t, h, l2norm_qk);
  std::lock_guard<std::mutex> lock(g_chunk_ws_mu);
  const long need = gdn_chunk_ws_bytes(b, t, h);
  if (need > g_chunk_ws_bytes) {
    if (g_chunk_ws) cudaFree(g_chunk_ws);
    g_chunk_ws = nullptr;
    g_chunk_ws_bytes = 0;
    if (cudaMalloc(&g_chunk_ws, need) != cudaSuccess) return fail(DUO_ENOMEM, "gdn_chunk: workspace");
    g_chunk_ws_bytes = need;
  }
  a.chunk_ws = g_chunk_ws;
  a.chunk_ws_bytes = g_chunk_ws_bytes;
  return launch_gdn_chunk(a, in_dtype, as_stream(stream));
}
