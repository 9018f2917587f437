// Gated DeltaNet chunked scan on the Blackwell tensor cores (tcgen05 + TMEM + TMA): the prefill form of the 16-bit
// engines.
//
// Chunk form of the gated delta rule (transformers torch_chunk_gated_delta_rule, chunk 64; the reference engine runs
// the same recurrence token by token, engine/kernels_qwen35.js:183-247).  Per chunk of 64 tokens with cumulative
// log-decay G:  L = strict_lower(beta_i k_i.k_j e^{G_i - G_j}),  T = (I + L)^-1,  U = T diag(beta) V,
// W = T diag(beta e^G) K,  V' = U - W S,  O = diag(e^G) Q S + tril(Q K^T e^{G_i - G_j}) V',
// S <- e^{G_63} S + K^T diag(e^{G_63 - G}) V'.
//
// One CTA per (row, value head) walks that sequence's chunks.  Everything is computed transposed, with the value
// dimension on the 128 TMEM lanes, so that every product is an M = 128 tcgen05.mma:
//   P1   [Q; K] K^T            -> TMEM 128 x 64   (rows 0-63 Q tokens, 64-127 K tokens; both operands K-major)
//   U^T = V^T (T diag beta)^T  -> TMEM 128 x 64   (V straight from its TMA tile as an MN-major operand)
//   W^T = K^T (T diag beta e^G)^T                 (the K tile MN-major; read out and stored as -W, token-major)
//   V'^T = U^T + S^T (-W)^T    (accumulated onto U^T)        O1 = S^T Q^T
//   O2 = V'^T A^T              S^T += V'^T diag(e^{G_63 - G}) K   (the K tile as an MN-major B operand)
// The f32 state S^T (lanes = dv, 128 columns = dk) stays in TMEM for the whole sequence: each chunk reads it once to
// make its 16-bit operand copy and writes it back scaled by e^{G_63}, after which the update MMA accumulates onto it.
// All MMA operands are f16 (bf16 inputs are converted in shared memory after their TMA load): the same precision as
// the warp-level kernel this replaces.  Warps 0-3 (TMEM lanes 32w ..) do the element-wise work: the conversion, the
// masked score matrices, the unit-triangular inverse T (16 x 16 diagonal blocks by forward substitution, the others
// by distance on warp-level MMAs), the operand copies and the output epilogue with the gated RMSNorm; lane 0 of
// warp 4 issues the TMA loads (two chunks in flight) and the MMAs.  TMA tiles come from 3D tensor maps over
// [rows][tokens][columns], so a chunk past a row's last token reads zeros.
//
// Shared memory (1024-aligned offsets): two 48 KB stages [Q0 | K0 | Q1 | K1 | V0 | V1] (64 tokens x 64 dims each,
// 128-byte swizzle), A (64 x 64), T diag(beta) and T diag(beta e^G) (reused for V'^T), -W (reused for
// V'^T diag(e^{G_63 - G})), S^T in f16 (128 x 128), the solve's scratch (reused for the output transpose).
#include <type_traits>

#include "kernels.cuh"
#include "mma.cuh"
#include "tc.cuh"

namespace duo {
namespace {

constexpr int GT_THREADS = 160;
constexpr uint32_t STAGE = 49152, OFF_Q0 = 0, OFF_K0 = 8192, OFF_V0 = 32768;
constexpr uint32_t OFF_A = 2 * STAGE, OFF_TB = OFF_A + 8192, OFF_TBE = OFF_TB + 8192, OFF_W = OFF_TBE + 8192;
constexpr uint32_t OFF_S16 = OFF_W + 16384, OFF_SCR = OFF_S16 + 32768;
constexpr uint32_t OFF_VT = OFF_TB, OFF_VTE = OFF_W;
constexpr int SCR_L = 0, SCR_T = 16640, SCR_LH = 33280, SCR_TH = 42496, SCR_XH = 51712, SCR_BYTES = 54016;
constexpr int LP = 65, HP = 72;  // pitches of the f32 and f16 64 x 64 solve tiles
constexpr uint32_t OFF_SMALL = OFF_SCR + SCR_BYTES;  // G, e^G, e^{G_63 - G}, beta, e^g: 64 floats each
constexpr uint32_t OFF_BAR = OFF_SMALL + 1280;
constexpr int GT_SMEM = OFF_BAR + 64 + 1024;  // + alignment slack
static_assert(GT_SMEM <= 232448, "shared memory");
// TMEM columns
constexpr uint32_t TS = 0, TQK = 128, TU = 192, TW = 256, TO1 = 320, TO2 = 384, TCOLS = 512;
constexpr uint32_t IDK64 = tc::idesc_f16_f32(128, 64, false, false);
constexpr uint32_t IDMN64 = tc::idesc_f16_f32(128, 64, true, false);   // A MN-major
constexpr uint32_t IDBMN128 = tc::idesc_f16_f32(128, 128, false, true);  // B MN-major
constexpr float QSCALE = 0.08838834764831845f;  // 1 / sqrt(128)

// byte offset of 16-byte chunk c (0..7) of row r of a K-major 128-byte-swizzled tile
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ uint4 pack8h(const float* v) {
  uint4 u;
  u.x = wm::pack_f16(v[0], v[1]);
  u.y = wm::pack_f16(v[2], v[3]);
  u.z = wm::pack_f16(v[4], v[5]);
  u.w = wm::pack_f16(v[6], v[7]);
  return u;
}

template <typename TI, bool NORM>
__global__ void __launch_bounds__(GT_THREADS, 1)
    gdn_chunk_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, GdnScanArgs a, unsigned* fault) {
  if (tc::fault_pending(fault)) {  // an earlier kernel gave up a wait
    pdl_wait();
    return;
  }
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = tc::smem_u32(sm);
  // operand descriptors at the base of shared memory, one per (LBO, SBO) layout; an operand at byte offset o is
  // desc_add(base, o) (one add per MMA for the single issuing thread)
  const uint64_t dkm = tc::desc_sw128(sb, 16, 1024);       // K-major
  const uint64_t dmn8 = tc::desc_sw128(sb, 8192, 1024);    // MN-major, 64-element blocks 8 KB apart (V tile)
  const uint64_t dmn16 = tc::desc_sw128(sb, 16384, 1024);  // MN-major, 64-element blocks 16 KB apart (K tile)
  float* Gs = reinterpret_cast<float*>(sm + OFF_SMALL);
  float* eg = Gs + 64;
  float* egl = Gs + 128;
  float* bs = Gs + 192;
  float* eg1 = Gs + 256;  // e^{g_t}: the decay of one token, e^{G_t - G_{t-1}}
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + OFF_BAR);  // [2]
  uint64_t* mbar = full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mbar + 1);
  float* Lf = reinterpret_cast<float*>(sm + OFF_SCR + SCR_L);
  float* Tf = reinterpret_cast<float*>(sm + OFF_SCR + SCR_T);
  __half* lh = reinterpret_cast<__half*>(sm + OFF_SCR + SCR_LH);
  __half* th = reinterpret_cast<__half*>(sm + OFF_SCR + SCR_TH);
  __half* xh0 = reinterpret_cast<__half*>(sm + OFF_SCR + SCR_XH);
  float* Ot = reinterpret_cast<float*>(sm + OFF_SCR);  // [64 tokens][128 dv], after the solve

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool math = tid < 128, issuer = tid == 128;
  const int h = blockIdx.x, b = blockIdx.y;
  const int kh = h / (a.h / a.hq);
  const int nch = (a.t + 63) / 64;
  float* Sg = a.state + (((long)(a.state_row0 + b) * a.h + h) * 128) * 128;

  if (tid == 0) {
    tc::mbar_init(&full[0], 1);
    tc::mbar_init(&full[1], 1);
    tc::mbar_init(mbar, 1);
    tc::fence_mbar_init();
  }
  if (issuer) {
    tc::prefetch_tmap(&tq);
    tc::prefetch_tmap(&tk);
    tc::prefetch_tmap(&tv);
  }
  if (warp == 0) tc::tmem_alloc(tmem_slot, TCOLS);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;  // this warp's TMEM lanes (math warps)
  pdl_wait();
  pdl_trigger();

  int n_tma = 0, n_commit = 0;  // issuer: chunks whose tiles were requested, MMA commits issued
  auto issue_tiles = [&](int c) {
    const int s = c & 1;
    uint8_t* st = sm + s * STAGE;
    tc::mbar_arrive_expect_tx(&full[s], STAGE);
    for (int hf = 0; hf < 2; hf++) {
      tc::tma_load_3d(st + OFF_Q0 + hf * 16384, &tq, kh * 128 + hf * 64, c * 64, b, &full[s]);
      tc::tma_load_3d(st + OFF_K0 + hf * 16384, &tk, kh * 128 + hf * 64, c * 64, b, &full[s]);
      tc::tma_load_3d(st + OFF_V0 + hf * 8192, &tv, h * 128 + hf * 64, c * 64, b, &full[s]);
    }
    n_tma = c + 1;
  };
  if (issuer && nch > 0) issue_tiles(0);

  // the entering state S [dk][dv] -> S^T in TMEM (lane dv, column dk)
  if (math) {
#pragma unroll 1
    for (int c0 = 0; c0 < 128; c0 += 32) {
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; j++) v[j] = Sg[(long)(c0 + j) * 128 + tid];
      tc::tmem_st32(tmem + TS + c0 + lane_off, v);
    }
  }
  // gates of chunk 0 (threads 0-63 hold one token's each, one chunk ahead)
  float gnext = 0.f, bnext = 0.f;
  if (tid < 64 && tid < a.t) {
    const long m = (long)b * a.t + tid;
    gnext = a.g[m * a.h + h];
    bnext = a.beta[m * a.h + h];
  }
  const float hs = (NORM && a.head_scale) ? a.head_scale[h] : 1.f;
  float4 nw = make_float4(1.f, 1.f, 1.f, 1.f);
  if (NORM && math) nw = *reinterpret_cast<const float4*>(a.norm_w + 4 * lane);
  uint32_t mph = 0;  // parity of the next MMA commit the math warps wait for
  bool ok = true;
  // bf16 tiles -> f16 in place (the MMAs mix them with f16 operands written here): part p of np of stage stg.
  // Chunk 0's stage is converted at its start; chunk c + 1's in two halves while chunk c's U / W and V' / O1 MMAs run.
  auto convert_tiles = [&](int stg, int p, int np) {
    if constexpr (sizeof(TI) == 2 && !std::is_same<TI, __half>::value) {
      uint4* ring = reinterpret_cast<uint4*>(sm + stg * STAGE);
      const int n = (int)(STAGE / 16), q0 = n * p / np, q1 = n * (p + 1) / np;
#pragma unroll 4
      for (int q = q0 + tid; q < q1; q += 128) {
        const uint4 u = ring[q];
        const __nv_bfloat162* bp = reinterpret_cast<const __nv_bfloat162*>(&u);
        float f[8];
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const float2 x = __bfloat1622float2(bp[e]);
          f[2 * e] = x.x;
          f[2 * e + 1] = x.y;
        }
        ring[q] = pack8h(f);
      }
      tc::fence_proxy_async();
    }
  };

#pragma unroll 1
  for (int c = 0; c < nch; c++) {
    const int s = c & 1, t0 = c * 64;
    const uint32_t st = sb + s * STAGE;
    if (tid < 64) {
      Gs[tid] = gnext;
      bs[tid] = bnext;
      gnext = bnext = 0.f;
      const int t = t0 + 64 + tid;
      if (t < a.t) {
        const long m = (long)b * a.t + t;
        gnext = a.g[m * a.h + h];
        bnext = a.beta[m * a.h + h];
      }
    }
    // this chunk's z (gate of the gated norm) into L2 now, into registers only for the output (32 registers held
    // across the whole chunk cost this 254-register kernel more than an L2 round trip): thread i, one 128-byte line
    if (NORM && math) {
      const int t = t0 + (tid >> 1);
      if (t < a.t) {
        const TI* zl = static_cast<const TI*>(a.z) + ((long)b * a.t + t) * a.z_stride + h * 128 + (tid & 1) * 64;
        asm volatile("prefetch.global.L2 [%0];" ::"l"(zl));
      }
    }
    if (math) ok = tc::mbar_wait(&full[s], (uint32_t)((c >> 1) & 1));
    if (__syncthreads_or(!ok)) {
      if (tid == 0) atomicOr(fault, 32u);
      goto bail;
    }
    if (issuer && c + 1 < nch) issue_tiles(c + 1);  // stage s ^ 1 was last read by chunk c - 1's MMAs (all done)
    if (math) {
      if (warp == 0) {  // G = cumsum(g), e^G, e^{G_63 - G}
        const float g0 = Gs[2 * lane], g1 = Gs[2 * lane + 1];
        float sc = g0 + g1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float n = __shfl_up_sync(0xffffffffu, sc, o);
          if (lane >= o) sc += n;
        }
        const float G0 = sc - g1, G1 = sc;
        const float Gl = __shfl_sync(0xffffffffu, G1, 31);
        Gs[2 * lane] = G0;
        Gs[2 * lane + 1] = G1;
        eg[2 * lane] = expf(G0);
        eg[2 * lane + 1] = expf(G1);
        egl[2 * lane] = expf(Gl - G0);
        egl[2 * lane + 1] = expf(Gl - G1);
        eg1[2 * lane] = expf(g0);
        eg1[2 * lane + 1] = expf(g1);
      }
      if (c == 0) convert_tiles(s, 0, 1);
      tc::fence_proxy_async();
    }
    __syncthreads();
    // ---- P1: [Q; K] K^T
    if (issuer) {
      tc::fence_after_sync();
#pragma unroll
      for (int ks = 0; ks < 8; ks++) {
        const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
        tc::mma_bf16(tmem + TQK, tc::desc_add(dkm, (st - sb) + OFF_Q0 + off),
                     tc::desc_add(dkm, (st - sb) + OFF_K0 + off), IDK64, ks > 0);
      }
      tc::mma_commit(mbar);
      n_commit++;
    }
    if (math) {
      // while P1 runs: S^T (final after chunk c - 1) -> its f16 operand copy, and back into TMEM scaled by e^{G_63}
      tc::fence_after_sync();
      {
        const float el = eg[63];
#pragma unroll 1
        for (int c0 = 0; c0 < 128; c0 += 64) {  // 64 columns per TMEM round trip
          float v[64];
          tc::tmem_ld2x32(tmem + TS + c0 + lane_off, tmem + TS + c0 + 32 + lane_off, v, v + 32);
#pragma unroll
          for (int q = 0; q < 8; q++) {
            const int dk = c0 + 8 * q;
            *reinterpret_cast<uint4*>(sm + OFF_S16 + (dk >> 6) * 16384 + swz(tid, (dk & 63) >> 3)) = pack8h(v + 8 * q);
          }
#pragma unroll
          for (int j = 0; j < 64; j++) v[j] *= el;
          tc::tmem_st32(tmem + TS + c0 + lane_off, v);
          tc::tmem_st32(tmem + TS + c0 + 32 + lane_off, v + 32);
        }
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
      ok = tc::mbar_wait(mbar, mph);
      mph ^= 1;
    }
    if (__syncthreads_or(!ok)) {
      if (tid == 0) atomicOr(fault, 64u);
      goto bail;
    }
    if (math) {
      tc::fence_after_sync();
      float x[64];
      tc::tmem_ld2x32(tmem + TQK + lane_off, tmem + TQK + 32 + lane_off, x, x + 32);
      // the decay e^{G_i - G_j} of row i, for j walking down from i: the product of the tokens' own decays e^{g_t},
      // t = j + 1 .. i (a multiply per entry instead of an exponential; it only shrinks, so it underflows to 0
      // gracefully however strong the decay)
      const int i = tid & 63;
      float d[64];
      {
        float run = 1.f;
#pragma unroll
        for (int j = 63; j >= 0; j--) {
          if (j < i) run *= eg1[j + 1];
          d[j] = j <= i ? run : 0.f;
        }
      }
      if (tid < 64) {  // Q row i: A = tril(q.k e^{G_i - G_j}) / sqrt(dk)
#pragma unroll
        for (int q = 0; q < 8; q++) {
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; e++) v[e] = x[8 * q + e] * QSCALE * d[8 * q + e];
          *reinterpret_cast<uint4*>(sm + OFF_A + swz(i, q)) = pack8h(v);
        }
      } else {  // K row i: L = strict_lower(beta_i k_i.k_j e^{G_i - G_j}): its diagonal 16 x 16 block in f32 (the
                // forward substitution) and the blocks left of it in f16 (the off-diagonal products)
        const float bi = bs[i];
        const int o = i & ~15;
#pragma unroll
        for (int j = 0; j < 64; j += 2) {
          const float l0 = j < i ? bi * x[j] * d[j] : 0.f, l1 = j + 1 < i ? bi * x[j + 1] * d[j + 1] : 0.f;
          if (j >= o && j < o + 16) {
            Lf[i * LP + j] = l0;
            Lf[i * LP + j + 1] = l1;
          } else if (j < o) {
            *reinterpret_cast<uint32_t*>(lh + i * HP + j) = wm::pack_f16(l0, l1);
          }
        }
      }
    }
    __syncthreads();
    // ---- T = (I + L)^-1: the 16 x 16 diagonal blocks, warp w on block w, by recursive doubling: once the diagonal
    // blocks of size bs of T hold the inverses of M = I + L's, each pair of them [[A, 0], [C, B]] completes to
    // [[A^-1, 0], [-B^-1 C A^-1, B^-1]] (two bs x bs products; bs = 1, 2, 4, 8).  Four dependent levels instead of a
    // 16-step substitution; every entry is an f32 dot product over the triangle only.
    if (math) {
      const int o = warp * 16;
      float* T = Tf + o * LP + o;
      const float* Lb = Lf + o * LP + o;
      float* Xs = reinterpret_cast<float*>(sm + OFF_SCR + SCR_XH) + warp * 64;  // C A^-1 of the current level
#pragma unroll
      for (int e = 0; e < 8; e++) {  // identity (the strictly upper part stays zero)
        const int idx = lane + 32 * e, r = idx >> 4, c = idx & 15;
        T[r * LP + c] = r == c ? 1.f : 0.f;
      }
      __syncwarp();
      if (lane < 8) T[(2 * lane + 1) * LP + 2 * lane] = -Lb[(2 * lane + 1) * LP + 2 * lane];  // bs = 1
      __syncwarp();
#pragma unroll
      for (int bs = 2; bs <= 8; bs *= 2) {
        const int n = 8 * bs;  // entries of the lower-left blocks of this level: (16 / 2 bs) pairs x bs x bs
#pragma unroll
        for (int idx = lane; idx < n; idx += 32) {  // X = C A^-1 (A^-1 lower triangular: k >= c)
          const int pr = idx / (bs * bs), rem = idx % (bs * bs), r = rem / bs, c = rem % bs, p0 = 2 * bs * pr;
          float x = 0.f;
#pragma unroll
          for (int k = 0; k < bs; k++)
            if (k >= c) x += Lb[(p0 + bs + r) * LP + p0 + k] * T[(p0 + k) * LP + p0 + c];
          Xs[idx] = x;
        }
        __syncwarp();
#pragma unroll
        for (int idx = lane; idx < n; idx += 32) {  // T21 = -B^-1 X (B^-1 unit lower triangular: k <= r)
          const int pr = idx / (bs * bs), rem = idx % (bs * bs), r = rem / bs, c = rem % bs, p0 = 2 * bs * pr;
          float y = Xs[pr * bs * bs + r * bs + c];
#pragma unroll
          for (int k = 0; k < bs; k++)
            if (k < r) y += T[(p0 + bs + r) * LP + p0 + bs + k] * Xs[pr * bs * bs + k * bs + c];
          T[(p0 + bs + r) * LP + p0 + c] = -y;
        }
        __syncwarp();
      }
#pragma unroll
      for (int e = 0; e < 8; e++) {  // the f16 copy for the off-diagonal products (whole blocks, zeros included)
        const int idx = lane + 32 * e, r = idx >> 4, c = idx & 15;
        th[(o + r) * HP + o + c] = __float2half_rn(T[r * LP + c]);
      }
    }
    __syncthreads();
    // ... the off-diagonal blocks by distance d on warp-level MMAs:
    // T[bi][bj] = -T[bi][bi] (sum_{bj <= bk < bi} L[bi][bk] T[bk][bj]), warp bj of the 4 - d
#pragma unroll 1
    for (int d = 1; d < 4; d++) {
      if (warp < 4 - d) {
        const int g = lane >> 2, q4 = lane & 3;
        const int bj = warp, bi = warp + d;
        float X[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        for (int bk = bj; bk < bi; bk++) {
          uint32_t af[4], bf[4];
          wm::lda(af, lh, HP, bi * 16, bk * 16);
          wm::ldb_kn(bf, th, HP, bj * 16, bk * 16);
          wm::mma_f16(X[0], af, bf);
          wm::mma_f16(X[1], af, bf + 2);
        }
        __half* xh = xh0 + warp * 16 * 24;
#pragma unroll
        for (int h2 = 0; h2 < 2; h2++) {
          *reinterpret_cast<uint32_t*>(xh + g * 24 + h2 * 8 + 2 * q4) = wm::pack_f16(X[h2][0], X[h2][1]);
          *reinterpret_cast<uint32_t*>(xh + (g + 8) * 24 + h2 * 8 + 2 * q4) = wm::pack_f16(X[h2][2], X[h2][3]);
        }
        __syncwarp();
        float Y[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        {
          uint32_t af[4], bf[4];
          wm::lda(af, th, HP, bi * 16, bi * 16);
          wm::ldb_kn(bf, xh, 24, 0, 0);
          wm::mma_f16(Y[0], af, bf);
          wm::mma_f16(Y[1], af, bf + 2);
        }
#pragma unroll
        for (int h2 = 0; h2 < 2; h2++) {
          const int cc = bj * 16 + h2 * 8 + 2 * q4;
          const int r0 = bi * 16 + g, r1 = r0 + 8;
          Tf[r0 * LP + cc] = -Y[h2][0];
          Tf[r0 * LP + cc + 1] = -Y[h2][1];
          Tf[r1 * LP + cc] = -Y[h2][2];
          Tf[r1 * LP + cc + 1] = -Y[h2][3];
          *reinterpret_cast<uint32_t*>(th + r0 * HP + cc) = wm::pack_f16(-Y[h2][0], -Y[h2][1]);
          *reinterpret_cast<uint32_t*>(th + r1 * HP + cc) = wm::pack_f16(-Y[h2][2], -Y[h2][3]);
        }
      }
      __syncthreads();
    }
    // ---- T diag(beta) and T diag(beta e^G), K-major 64 x 64 (row i, 64 tokens j)
    if (math) {
      const int i = tid >> 1, hf = tid & 1;
#pragma unroll
      for (int q = hf * 4; q < hf * 4 + 4; q++) {
        float v1[8], v2[8];
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const int j = 8 * q + e;
          v1[e] = j <= i ? Tf[i * LP + j] * bs[j] : 0.f;  // T is unit lower triangular; its upper part is not stored
          v2[e] = v1[e] * eg[j];
        }
        *reinterpret_cast<uint4*>(sm + OFF_TB + swz(i, q)) = pack8h(v1);
        *reinterpret_cast<uint4*>(sm + OFF_TBE + swz(i, q)) = pack8h(v2);
      }
      tc::fence_proxy_async();
    }
    __syncthreads();
    // ---- U^T = V^T (T diag beta)^T,  W^T = K^T (T diag beta e^G)^T  (A operands MN-major from the tiles)
    if (issuer) {
      tc::fence_after_sync();
#pragma unroll
      for (int ks = 0; ks < 4; ks++) {
        const uint64_t btb = tc::desc_add(dkm, OFF_TB + ks * 32);
        const uint64_t btbe = tc::desc_add(dkm, OFF_TBE + ks * 32);
        tc::mma_bf16(tmem + TU, tc::desc_add(dmn8, (st - sb) + OFF_V0 + ks * 2048), btb, IDMN64, ks > 0);
        tc::mma_bf16(tmem + TW, tc::desc_add(dmn16, (st - sb) + OFF_K0 + ks * 2048), btbe, IDMN64, ks > 0);
      }
      tc::mma_commit(mbar);
      n_commit++;
    }
    if (math) {
      if (c + 1 < nch) {  // while U / W run: the first half of chunk c + 1's tiles (requested at this chunk's start)
        ok = tc::mbar_wait(&full[s ^ 1], (uint32_t)(((c + 1) >> 1) & 1));
        if (ok) convert_tiles(s ^ 1, 0, 2);
      }
      ok = tc::mbar_wait(mbar, mph) && ok;
      mph ^= 1;
    }
    if (__syncthreads_or(!ok)) {
      if (tid == 0) atomicOr(fault, 64u);
      goto bail;
    }
    if (math) {
      tc::fence_after_sync();
      // -W, token-major (row i, dk contiguous; two 64-dk atoms): thread d writes column d
      {
        float w[64];
        tc::tmem_ld2x32(tmem + TW + lane_off, tmem + TW + 32 + lane_off, w, w + 32);
        const int d = tid;
        __half* wb = reinterpret_cast<__half*>(sm + OFF_W + (d >> 6) * 8192);
        const int cidx = (d & 63) >> 3, e = d & 7;
#pragma unroll
        for (int i = 0; i < 64; i++)
          wb[(i * 128 + ((cidx ^ (i & 7)) << 4)) / 2 + e] = __float2half_rn(-w[i]);
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
    }
    __syncthreads();
    // ---- V'^T = U^T + S^T (-W)^T (onto U),  O1 = S^T Q^T
    if (issuer) {
      tc::fence_after_sync();
#pragma unroll
      for (int ks = 0; ks < 8; ks++) {
        const uint32_t ak = (ks >> 2) * 16384 + (ks & 3) * 32;
        const uint64_t as16 = tc::desc_add(dkm, OFF_S16 + ak);
        tc::mma_bf16(tmem + TU, as16, tc::desc_add(dkm, OFF_W + (ks >> 2) * 8192 + (ks & 3) * 32), IDK64,
                     1);
        tc::mma_bf16(tmem + TO1, as16, tc::desc_add(dkm, (st - sb) + OFF_Q0 + ak), IDK64, ks > 0);
      }
      tc::mma_commit(mbar);
      n_commit++;
    }
    if (math) {
      if (c + 1 < nch) convert_tiles(s ^ 1, 1, 2);  // while V' / O1 run: the second half
      ok = tc::mbar_wait(mbar, mph);
      mph ^= 1;
    }
    if (__syncthreads_or(!ok)) {
      if (tid == 0) atomicOr(fault, 64u);
      goto bail;
    }
    if (math) {  // V'^T and V'^T diag(e^{G_63 - G}), K-major (row dv, 64 tokens)
      tc::fence_after_sync();
      float v[64];
      tc::tmem_ld2x32(tmem + TU + lane_off, tmem + TU + 32 + lane_off, v, v + 32);
#pragma unroll
      for (int q = 0; q < 8; q++) {
        *reinterpret_cast<uint4*>(sm + OFF_VT + swz(tid, q)) = pack8h(v + 8 * q);
        float e8[8];
#pragma unroll
        for (int e = 0; e < 8; e++) e8[e] = v[8 * q + e] * egl[8 * q + e];
        *reinterpret_cast<uint4*>(sm + OFF_VTE + swz(tid, q)) = pack8h(e8);
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
    }
    __syncthreads();
    // ---- O2 = V'^T A^T,  S^T += V'^T diag(e^{G_63 - G}) K  (B = the K tile, MN-major)
    if (issuer) {
      tc::fence_after_sync();
#pragma unroll
      for (int ks = 0; ks < 4; ks++) {
        tc::mma_bf16(tmem + TO2, tc::desc_add(dkm, OFF_VT + ks * 32),
                     tc::desc_add(dkm, OFF_A + ks * 32), IDK64, ks > 0);
        tc::mma_bf16(tmem + TS, tc::desc_add(dkm, OFF_VTE + ks * 32),
                     tc::desc_add(dmn16, (st - sb) + OFF_K0 + ks * 2048), IDBMN128, 1);
      }
      tc::mma_commit(mbar);
      n_commit++;
    }
    if (math) {
      ok = tc::mbar_wait(mbar, mph);
      mph ^= 1;
    }
    if (__syncthreads_or(!ok)) {
      if (tid == 0) atomicOr(fault, 64u);
      goto bail;
    }
    // ---- output: O = e^G O1 / sqrt(dk) + O2, through shared memory to token rows, gated RMSNorm, store
    if (math) {
      tc::fence_after_sync();
#pragma unroll 1
      for (int c0 = 0; c0 < 64; c0 += 32) {
        float o1[32], o2[32];
        tc::tmem_ld2x32(tmem + TO1 + c0 + lane_off, tmem + TO2 + c0 + lane_off, o1, o2);
#pragma unroll
        for (int t = 0; t < 32; t++) Ot[(c0 + t) * 128 + tid] = eg[c0 + t] * QSCALE * o1[t] + o2[t];
      }
    }
    __syncthreads();
    if (math) {
      TI* op = static_cast<TI*>(a.o);
      uint2 zr[16];  // z (in L2 since the chunk's start): warp w takes token rows w, w + 4, ..; lane 4 dv columns
      if (NORM) {
        const TI* zp = static_cast<const TI*>(a.z);
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const int t = t0 + warp + 4 * i;
          if (t < a.t) zr[i] = *reinterpret_cast<const uint2*>(zp + ((long)b * a.t + t) * a.z_stride + h * 128 + 4 * lane);
        }
      }
#pragma unroll
      for (int ps = 0; ps < 2; ps++) {  // token rows warp + 4 i, i = 8 ps .. 8 ps + 7 (two passes: registers)
        float o[8][4];
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const float4 ov = *reinterpret_cast<const float4*>(Ot + (warp + 4 * (8 * ps + i)) * 128 + 4 * lane);
          o[i][0] = ov.x; o[i][1] = ov.y; o[i][2] = ov.z; o[i][3] = ov.w;
        }
        if (NORM) {
          // the 8 rows' sums of squares over the warp together, by recursive halving: lane l ends with row
          // 4 b4 + 2 b3 + b2 (bits of l); 10 shuffles for the 8 rows instead of 5 dependent ones per row
          float v[8];
#pragma unroll
          for (int i = 0; i < 8; i++) v[i] = o[i][0] * o[i][0] + o[i][1] * o[i][1] + o[i][2] * o[i][2] + o[i][3] * o[i][3];
#pragma unroll
          for (int w = 16, n = 4; w >= 4; w >>= 1, n >>= 1) {
            const bool up = lane & w;
#pragma unroll
            for (int i = 0; i < n; i++) {
              const float send = up ? v[i] : v[i + n];
              const float keep = up ? v[i + n] : v[i];
              v[i] = keep + __shfl_xor_sync(0xffffffffu, send, w);
            }
          }
          v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
          v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
          const float rms_mine = rsqrtf(v[0] / 128.f + a.eps);
#pragma unroll
          for (int i = 0; i < 8; i++) {
            const float rms = __shfl_sync(0xffffffffu, rms_mine, ((i >> 2) << 4) | (((i >> 1) & 1) << 3) | ((i & 1) << 2));
            if (t0 + warp + 4 * (8 * ps + i) < a.t) {
              const TI* zt = reinterpret_cast<const TI*>(&zr[8 * ps + i]);
              o[i][0] *= rms * nw.x * silu_tanh(to_f(zt[0])) * hs;
              o[i][1] *= rms * nw.y * silu_tanh(to_f(zt[1])) * hs;
              o[i][2] *= rms * nw.z * silu_tanh(to_f(zt[2])) * hs;
              o[i][3] *= rms * nw.w * silu_tanh(to_f(zt[3])) * hs;
            }
          }
        }
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const int t = t0 + warp + 4 * (8 * ps + i);
          if (t < a.t) {
            uint2 u;
            TI* p = reinterpret_cast<TI*>(&u);
#pragma unroll
            for (int e = 0; e < 4; e++) p[e] = from_f<TI>(o[i][e]);
            *reinterpret_cast<uint2*>(op + ((long)b * a.t + t) * a.o_stride + h * 128 + 4 * lane) = u;
          }
        }
      }
    }
  }
  // final state S^T (TMEM) -> S [dk][dv]
  if (math) {
    tc::fence_after_sync();
#pragma unroll 1
    for (int c0 = 0; c0 < 128; c0 += 32) {
      float v[32];
      tc::tmem_ld32(tmem + TS + c0 + lane_off, v);
#pragma unroll
      for (int j = 0; j < 32; j++) Sg[(long)(c0 + j) * 128 + tid] = v[j];
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, TCOLS);
  }
  return;

bail:
  // A wait gave up: let the copies and MMAs already issued land (bounded) before the CTA and its TMEM go away.
  if (issuer) {
    for (int c = n_tma - 2; c < n_tma; c++)
      if (c >= 0) tc::mbar_wait(&full[c & 1], (uint32_t)((c >> 1) & 1));
    if (n_commit > 0) tc::mbar_wait(mbar, (uint32_t)((n_commit - 1) & 1));
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, TCOLS);
  }
}

template <typename TI, bool NORM>
int run_chunk_tc(const GdnScanArgs& a, int dtype, cudaStream_t st) {
  const size_t es = sizeof(TI);
  CUtensorMap tq, tk, tv;
  DUO_TRY(make_tmap_3d_16(&tq, a.q, dtype, (long)a.hq * 128, a.t, a.b, a.q_stride * es, (long)a.t * a.q_stride * es,
                          64, 64));
  DUO_TRY(make_tmap_3d_16(&tk, a.k, dtype, (long)a.hq * 128, a.t, a.b, a.k_stride * es, (long)a.t * a.k_stride * es,
                          64, 64));
  DUO_TRY(make_tmap_3d_16(&tv, a.v, dtype, (long)a.h * 128, a.t, a.b, a.v_stride * es, (long)a.t * a.v_stride * es,
                          64, 64));
  unsigned* fault = tc_fault_ptr();
  if (!fault) return fail(DUO_ECUDA, "tensor-core fault word is not addressable");
  DUO_TRY(ensure_smem_attr(gdn_chunk_tc_kernel<TI, NORM>, GT_SMEM));
  DUO_CUDA_TRY(::duo::launch_kernel(gdn_chunk_tc_kernel<TI, NORM>, dim3(a.h, a.b), GT_THREADS, GT_SMEM, st, tq, tk, tv,
                                    a, fault));
  DUO_LAUNCH_CHECK("gdn_chunk_tc_kernel");
  return DUO_OK;
}

}  // namespace

bool gdn_chunk_tc_eligible(const GdnScanArgs& a, int dtype) {
  if (dtype != DUO_BF16 && dtype != DUO_F16) return false;
  if (a.l2norm_qk || a.dk != 128 || a.dv != 128) return false;
  const auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al(a.q) || !al(a.k) || !al(a.v) || !al(a.o)) return false;
  if ((a.q_stride | a.k_stride | a.v_stride) % 8 || a.o_stride % 4) return false;
  if (a.norm_w && (!a.z || a.z_stride % 4 || (reinterpret_cast<uintptr_t>(a.z) & 7))) return false;
  return true;
}

int launch_gdn_chunk_tc(const GdnScanArgs& a, int dtype, cudaStream_t st) {
  if (a.b == 0 || a.t == 0) return DUO_OK;
  const bool norm = a.norm_w != nullptr;
  if (dtype == DUO_F16) return norm ? run_chunk_tc<__half, true>(a, dtype, st) : run_chunk_tc<__half, false>(a, dtype, st);
  return norm ? run_chunk_tc<__nv_bfloat16, true>(a, dtype, st) : run_chunk_tc<__nv_bfloat16, false>(a, dtype, st);
}

}  // namespace duo
