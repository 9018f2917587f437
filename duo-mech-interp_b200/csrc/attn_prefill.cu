// Gated GQA attention, prefill (t > 1) of the 16-bit (bf16 / f16) engine on the tensor cores.
//
// One CTA = (row, kv head, tile of 128 / rep queries); its 128 query rows are the rep q heads of that kv head over the
// same query positions, so every K / V tile is loaded once for all of them.  8 warps x 16 rows; head dim 256.
// Per 64-key tile: S = Q K^T (bf16 or f16 mma, f32 accumulate), causal mask, online softmax in f32 (base 2), O += P V with
// P taken straight from the S accumulators.  K / V tiles are double-buffered with cp.async.  The output is divided by
// the softmax sum and multiplied by sigmoid(gate) on the way out (transformers Qwen3_5Attention: attention, then
// `attn_output * sigmoid(gate)`; the reference's WGSL does the same per (token, head), kernels_qwen35.js:73-123).
#include "kernels.cuh"
#include "mma.cuh"

namespace duo {

namespace {

constexpr int HD = 256, PQ = HD + 8, BKEY = 64;

}  // namespace

template <int REP, typename T16>
__global__ void __launch_bounds__(256, 1) attn_prefill_mma_kernel(AttnArgs a) {
  pdl_enter();
  constexpr int QT = 128 / REP;  // query positions per CTA
  extern __shared__ __align__(16) uint8_t smem[];
  T16* Qs = reinterpret_cast<T16*>(smem);
  T16* Ks = Qs + 128 * PQ;
  T16* Vs = Ks + 2 * BKEY * PQ;
  const int qt = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q4 = lane & 3;
  const int R = a.cache_row0 + b;
  const int p0 = a.start ? a.start[R] : a.len[R] - a.t;
  const int tq0 = qt * QT;
  const int nq = min(QT, a.t - tq0);
  const int n_keys = p0 + tq0 + nq;
  const int ntiles = (n_keys + BKEY - 1) / BKEY;
  const T16* q = static_cast<const T16*>(a.q);
  const T16* kc = static_cast<const T16*>(a.kc);
  const T16* vc = static_cast<const T16*>(a.vc);

  // Q tile: row r = head (kvh * REP + r / QT) at query position tq0 + r % QT; 32 chunks of 16 bytes per row
  for (int e = tid; e < 128 * 32; e += 256) {
    const int r = e >> 5, c = (e & 31) * 8;
    const int qi = r % QT, hq = kvh * REP + r / QT;
    const bool ok = qi < nq;
    const T16* src = ok ? q + (((long)b * a.t + tq0 + qi) * a.nh + hq) * HD + c : q;
    cp_async16(Qs + r * PQ + c, src, ok);
  }
  auto load_kv = [&](int kt, int buf) {
    for (int e = tid; e < BKEY * 32; e += 256) {
      const int r = e >> 5, c = (e & 31) * 8;
      const int key = kt * BKEY + r;
      const bool ok = key < n_keys;
      const long at = (((long)R * a.max_len + (ok ? key : 0)) * a.nkv + kvh) * HD + c;
      cp_async16(Ks + (buf * BKEY + r) * PQ + c, kc + at, ok);
      cp_async16(Vs + (buf * BKEY + r) * PQ + c, vc + at, ok);
    }
  };
  load_kv(0, 0);
  cp_commit();

  const int wr = warp * 16;                         // first query row of this warp
  const int qi0 = (wr + g) % QT, qi1 = (wr + g + 8) % QT;
  const int pos0 = p0 + tq0 + qi0, pos1 = p0 + tq0 + qi1;
  const float sl2 = a.scale * 1.4426950408889634f;  // softmax in base 2
  float O[32][4];
#pragma unroll
  for (int j = 0; j < 32; j++)
#pragma unroll
    for (int e = 0; e < 4; e++) O[j][e] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  for (int kt = 0; kt < ntiles; kt++) {
    const int buf = kt & 1;
    if (kt + 1 < ntiles) load_kv(kt + 1, buf ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    const T16* Kb = Ks + buf * BKEY * PQ;
    const T16* Vb = Vs + buf * BKEY * PQ;
    // S = Q K^T: 16 x 64 per warp
    float S[8][4];
#pragma unroll
    for (int j = 0; j < 8; j++)
#pragma unroll
      for (int e = 0; e < 4; e++) S[j][e] = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < HD; k0 += 16) {
      uint32_t aq[4];
      wm::lda(aq, Qs, PQ, wr, k0);
#pragma unroll
      for (int jj = 0; jj < 4; jj++) {
        uint32_t bk[4];
        wm::ldb_nk(bk, Kb, PQ, 16 * jj, k0);
        wm::Ops<T16>::mma(S[2 * jj], aq, bk);
        wm::Ops<T16>::mma(S[2 * jj + 1], aq, bk + 2);
      }
    }
    // causal mask + online softmax (rows g and g + 8 of the warp; a row's 64 scores sit on 4 lanes)
    float tm0 = -INFINITY, tm1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; j++)
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const int key = kt * BKEY + 8 * j + 2 * q4 + e;
        S[j][e] = (key <= pos0 && key < n_keys) ? S[j][e] * sl2 : -INFINITY;
        S[j][2 + e] = (key <= pos1 && key < n_keys) ? S[j][2 + e] * sl2 : -INFINITY;
        tm0 = fmaxf(tm0, S[j][e]);
        tm1 = fmaxf(tm1, S[j][2 + e]);
      }
    tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, 1));
    tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, 2));
    tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, 1));
    tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, 2));
    const float mn0 = fmaxf(m0, tm0), mn1 = fmaxf(m1, tm1);
    const float al0 = mn0 == -INFINITY ? 1.f : exp2f(m0 - mn0);
    const float al1 = mn1 == -INFINITY ? 1.f : exp2f(m1 - mn1);
    float ps0 = 0.f, ps1 = 0.f;
    uint32_t pf[4][4];  // P as bf16 A fragments, one per 16-key step
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const float e0 = S[j][0] == -INFINITY ? 0.f : exp2f(S[j][0] - mn0);
      const float e1 = S[j][1] == -INFINITY ? 0.f : exp2f(S[j][1] - mn0);
      const float e2 = S[j][2] == -INFINITY ? 0.f : exp2f(S[j][2] - mn1);
      const float e3 = S[j][3] == -INFINITY ? 0.f : exp2f(S[j][3] - mn1);
      ps0 += e0 + e1;
      ps1 += e2 + e3;
      pf[j >> 1][(j & 1) * 2] = wm::Ops<T16>::pack(e0, e1);
      pf[j >> 1][(j & 1) * 2 + 1] = wm::Ops<T16>::pack(e2, e3);
    }
    ps0 += __shfl_xor_sync(0xffffffffu, ps0, 1);
    ps0 += __shfl_xor_sync(0xffffffffu, ps0, 2);
    ps1 += __shfl_xor_sync(0xffffffffu, ps1, 1);
    ps1 += __shfl_xor_sync(0xffffffffu, ps1, 2);
    l0 = l0 * al0 + ps0;
    l1 = l1 * al1 + ps1;
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int j = 0; j < 32; j++) {
      O[j][0] *= al0; O[j][1] *= al0;
      O[j][2] *= al1; O[j][3] *= al1;
    }
    // O += P V: 16 x 256 per warp, K = 64 keys
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
#pragma unroll
      for (int nn = 0; nn < 16; nn++) {
        uint32_t bv[4];
        wm::ldb_kn(bv, Vb, PQ, 16 * nn, 16 * kk);
        wm::Ops<T16>::mma(O[2 * nn], pf[kk], bv);
        wm::Ops<T16>::mma(O[2 * nn + 1], pf[kk], bv + 2);
      }
    }
    __syncthreads();  // this buffer is refilled by the next iteration's prefetch
  }
  cp_wait<0>();

  // epilogue: normalise, gate, store
  T16* op = static_cast<T16*>(a.o);
  const T16* gp = static_cast<const T16*>(a.gate);
  const int hq = kvh * REP + wr / QT;
#pragma unroll
  for (int half = 0; half < 2; half++) {
    const int qi = half ? qi1 : qi0;
    if (qi >= nq) continue;
    const float inv = 1.f / (half ? l1 : l0);
    const long tok = (long)b * a.t + tq0 + qi;
    T16* orow = op + (tok * a.nh + hq) * HD;
    const T16* grow = gp ? gp + tok * a.gate_stride + (long)hq * a.gate_hstride : nullptr;
#pragma unroll
    for (int j = 0; j < 32; j++) {
      const int d = 8 * j + 2 * q4;
      float v0 = O[j][half * 2] * inv, v1 = O[j][half * 2 + 1] * inv;
      if (grow) {
        v0 *= sigmoidf_(to_f(grow[d]));
        v1 *= sigmoidf_(to_f(grow[d + 1]));
      }
      *reinterpret_cast<uint32_t*>(orow + d) = wm::Ops<T16>::pack(v0, v1);
    }
  }
}

template <int REP, typename T16>
static int run_prefill_mma(const AttnArgs& a, cudaStream_t st) {
  constexpr int smem = (128 + 4 * BKEY) * PQ * 2;
  DUO_TRY(ensure_smem_attr(attn_prefill_mma_kernel<REP, T16>, smem));
  DUO_CUDA_TRY(::duo::launch_kernel(attn_prefill_mma_kernel<REP, T16>, dim3(cdiv(a.t, 128 / REP), a.nkv, a.b), 256, smem, st, a));
  DUO_LAUNCH_CHECK("attn_prefill_mma_kernel");
  return DUO_OK;
}

int launch_attn_prefill_mma(const AttnArgs& a, int dtype, cudaStream_t st) {
  if (a.hd != HD) return fail(DUO_EINVAL, "attention prefill: head dim must be 256");
  const int rep = a.nh / a.nkv;
  if (rep != 1 && rep != 2 && rep != 4) return fail(DUO_EINVAL, "attention prefill: nh / nkv must be 1, 2 or 4");
  if (dtype == DUO_F16) return rep == 1 ? run_prefill_mma<1, __half>(a, st) : rep == 2 ? run_prefill_mma<2, __half>(a, st)
                                                                                    : run_prefill_mma<4, __half>(a, st);
  return rep == 1 ? run_prefill_mma<1, __nv_bfloat16>(a, st) : rep == 2 ? run_prefill_mma<2, __nv_bfloat16>(a, st)
                                                                       : run_prefill_mma<4, __nv_bfloat16>(a, st);
}

}  // namespace duo
