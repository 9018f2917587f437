// Gated GQA attention, decode (one new token per row) of the 16-bit engines: an HBM-streaming kernel.
//
// One CTA = (row, kv head, key split); 4 warps.  The rep (<= 4) q heads of the kv head form rows 0..rep-1 of a 16-row
// MMA tile, so each K / V tile is read from HBM once for all of them.  64-key K and V tiles stream through a 3-stage
// cp.async ring (two tiles in flight per SM); warp w takes keys 16w .. 16w + 15 of each tile: S = Q K^T and O += P V on
// the tensor cores (mma.sync, f32 accumulate), online softmax in f32 per warp.  The four warps' (max, sum, O) merge in
// shared memory; with one split the CTA applies the sigmoid gate and writes the output, otherwise it writes its
// partial for attn_combine_kernel (attn.cu).  Same arithmetic as the reference's `attention` for t = 1
// (engine/kernels_qwen35.js:73-123): softmax(q K^T / sqrt(hd)) V over keys 0..pos, times sigmoid(gate).
#include <algorithm>

#include "kernels.cuh"
#include "mma.cuh"

namespace duo {

namespace {

constexpr int DHD = 256, DP = DHD + 8, DBK = 64, DST = 3;

}  // namespace

constexpr int kDecodeSmem = (16 + 2 * DST * DBK) * DP * 2;

template <int REP, typename T16>
__global__ void __launch_bounds__(128, 1) attn_decode_mma_kernel(AttnArgs a, int nsplit, int split_len) {
  pdl_enter();
  extern __shared__ __align__(16) uint8_t smem[];
  T16* Qs = reinterpret_cast<T16*>(smem);
  T16* Ks = Qs + 16 * DP;
  T16* Vs = Ks + DST * DBK * DP;
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q4 = lane & 3;
  const int R = a.cache_row0 + b;
  const int p0 = a.start ? a.start[R] : a.len[R] - 1;
  const int n_keys = p0 + 1;
  const int kbeg = split * split_len, kend = min(n_keys, kbeg + split_len);
  const int ntiles = kend > kbeg ? (kend - kbeg + DBK - 1) / DBK : 0;
  const T16* q = static_cast<const T16*>(a.q);
  const T16* kc = static_cast<const T16*>(a.kc);
  const T16* vc = static_cast<const T16*>(a.vc);

  // Q rows 0..REP-1 = heads kvh*REP + r of this row's token; rows REP..15 zero
  for (int e = tid; e < 16 * 32; e += 128) {
    const int r = e >> 5, c = (e & 31) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < REP) v = *reinterpret_cast<const uint4*>(q + ((long)b * a.nh + kvh * REP + r) * DHD + c);
    *reinterpret_cast<uint4*>(Qs + r * DP + c) = v;
  }
  auto load_tile = [&](int kt, int stage) {
    for (int e = tid; e < DBK * 32; e += 128) {
      const int r = e >> 5, c = (e & 31) * 8;
      const int key = kbeg + kt * DBK + r;
      const bool ok = key < kend;
      const long at = (((long)R * a.max_len + (ok ? key : 0)) * a.nkv + kvh) * DHD + c;
      cp_async16(Ks + (stage * DBK + r) * DP + c, kc + at, ok);
      cp_async16(Vs + (stage * DBK + r) * DP + c, vc + at, ok);
    }
  };
#pragma unroll
  for (int s = 0; s < DST - 1; s++) {
    if (s < ntiles) load_tile(s, s);
    cp_commit();
  }
  const float sl2 = a.scale * 1.4426950408889634f;
  float O[32][4];
#pragma unroll
  for (int j = 0; j < 32; j++)
#pragma unroll
    for (int e = 0; e < 4; e++) O[j][e] = 0.f;
  float mrow = -INFINITY, lrow = 0.f;  // row g (rows g + 8 are padding)

  for (int kt = 0; kt < ntiles; kt++) {
    cp_wait<DST - 2>();
    __syncthreads();  // tile kt is in; every warp is done with tile kt - 1
    if (kt + DST - 1 < ntiles) load_tile(kt + DST - 1, (kt + DST - 1) % DST);
    cp_commit();
    const int stage = kt % DST;
    const T16* Kb = Ks + stage * DBK * DP;
    const T16* Vb = Vs + stage * DBK * DP;
    float S[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
    for (int k0 = 0; k0 < DHD; k0 += 16) {
      uint32_t aq[4], bk[4];
      wm::lda(aq, Qs, DP, 0, k0);
      wm::ldb_nk(bk, Kb, DP, warp * 16, k0);
      wm::Ops<T16>::mma(S[0], aq, bk);
      wm::Ops<T16>::mma(S[1], aq, bk + 2);
    }
    float tm = -INFINITY;
#pragma unroll
    for (int j = 0; j < 2; j++)
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const int key = kbeg + kt * DBK + warp * 16 + 8 * j + 2 * q4 + e;
        S[j][e] = key < kend ? S[j][e] * sl2 : -INFINITY;
        tm = fmaxf(tm, S[j][e]);
      }
    tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 1));
    tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 2));
    const float mn = fmaxf(mrow, tm);
    const float al = mn == -INFINITY ? 1.f : exp2f(mrow - mn);
    float e00 = S[0][0] == -INFINITY ? 0.f : exp2f(S[0][0] - mn);
    float e01 = S[0][1] == -INFINITY ? 0.f : exp2f(S[0][1] - mn);
    float e10 = S[1][0] == -INFINITY ? 0.f : exp2f(S[1][0] - mn);
    float e11 = S[1][1] == -INFINITY ? 0.f : exp2f(S[1][1] - mn);
    float ps = e00 + e01 + e10 + e11;
    ps += __shfl_xor_sync(0xffffffffu, ps, 1);
    ps += __shfl_xor_sync(0xffffffffu, ps, 2);
    lrow = lrow * al + ps;
    mrow = mn;
    uint32_t pf[4];
    pf[0] = wm::Ops<T16>::pack(e00, e01);
    pf[1] = 0u;  // rows g + 8: padding
    pf[2] = wm::Ops<T16>::pack(e10, e11);
    pf[3] = 0u;
#pragma unroll
    for (int j = 0; j < 32; j++) {
      O[j][0] *= al;
      O[j][1] *= al;
    }
#pragma unroll
    for (int nn = 0; nn < 16; nn++) {
      uint32_t bv[4];
      wm::ldb_kn(bv, Vb + warp * 16 * DP, DP, 16 * nn, 0);
      wm::Ops<T16>::mma(O[2 * nn], pf, bv);
      wm::Ops<T16>::mma(O[2 * nn + 1], pf, bv + 2);
    }
  }
  cp_wait<0>();
  __syncthreads();  // the K / V ring is free: reuse it for the merge
  float* mw = reinterpret_cast<float*>(Ks);    // [4 warps][16]
  float* lw = mw + 4 * 16;                     // [4 warps][16]
  float* ow = lw + 4 * 16;                     // [4 warps][REP][DHD]
  if (q4 == 0) {
    mw[warp * 16 + g] = mrow;
    lw[warp * 16 + g] = lrow;
  }
  if (g < REP) {
#pragma unroll
    for (int j = 0; j < 32; j++) {
      ow[(warp * REP + g) * DHD + 8 * j + 2 * q4] = O[j][0];
      ow[(warp * REP + g) * DHD + 8 * j + 2 * q4 + 1] = O[j][1];
    }
  }
  __syncthreads();
  const float ln2 = 0.6931471805599453f;  // partial maxima leave in natural-log units for attn_combine_kernel
  for (int e = tid; e < REP * DHD; e += 128) {
    const int r = e / DHD, d = e % DHD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; w++) M = fmaxf(M, mw[w * 16 + r]);
    float L = 0.f, Ov = 0.f;
#pragma unroll
    for (int w = 0; w < 4; w++) {
      const float f = mw[w * 16 + r] == -INFINITY ? 0.f : exp2f(mw[w * 16 + r] - M);
      L += lw[w * 16 + r] * f;
      Ov += ow[(w * REP + r) * DHD + d] * f;
    }
    const int h = kvh * REP + r;
    if (nsplit == 1) {
      float v = Ov / L;
      if (a.gate) v *= sigmoidf_(to_f(static_cast<const T16*>(a.gate)[(long)b * a.gate_stride + (long)h * a.gate_hstride + d]));
      static_cast<T16*>(a.o)[((long)b * a.nh + h) * DHD + d] = from_f<T16>(v);
    } else {
      float* wp = a.work + (((long)b * a.nh + h) * nsplit + split) * (DHD + 2);
      wp[2 + d] = Ov;
      if (d == 0) {
        wp[0] = M == -INFINITY ? -INFINITY : M * ln2;
        wp[1] = L;
      }
    }
  }
}

// Splits per (row, kv head): as many as keep every split at >= 4 tiles, choosing the count whose CTAs fill the last
// wave best (one CTA per SM).
static int attn_decode_mma_splits(int b, int nkv, int max_len) {
  const long pairs = (long)std::max(1, b) * nkv;
  const int sms = sm_count();
  const int max_ns = std::max(1, std::min(64, cdiv(max_len, 4 * DBK)));
  int best = 1;
  double best_eff = 0.0;
  for (int ns = 1; ns <= max_ns; ns++) {
    const long ctas = pairs * ns;
    const long waves = (ctas + sms - 1) / sms;
    // efficiency of the last wave, weighted towards enough CTAs to cover the SMs at all
    const double eff = (double)ctas / (double)(waves * sms);
    if (eff > best_eff + 0.02) {
      best_eff = eff;
      best = ns;
    }
  }
  return best;
}

// splits after rounding each split to whole tiles (what the launch uses when the scratch does not limit it)
int attn_decode_mma_plan(int b, int nkv, int max_len, int* split_len) {
  const int ns = attn_decode_mma_splits(b, nkv, max_len);
  const int sl = cdiv(cdiv(max_len, ns), DBK) * DBK;
  if (split_len) *split_len = sl;
  return cdiv(max_len, sl);
}

int launch_attn_decode_mma(const AttnArgs& a, int dtype, cudaStream_t st) {
  const int rep = a.nh / a.nkv;
  if (a.hd != DHD || rep < 1 || rep > 4) return fail(DUO_EINVAL, "attention decode: hd 256 and nh / nkv in 1..4");
  int split_len = 0;
  int ns = attn_decode_mma_plan(a.b, a.nkv, a.max_len, &split_len);
  if (!a.work) ns = 1;
  while (ns > 1 && (long)a.b * a.nh * ns * (DHD + 2) > a.work_floats) ns--;
  if (ns == 1) split_len = cdiv(a.max_len, DBK) * DBK;
  else split_len = cdiv(cdiv(a.max_len, ns), DBK) * DBK;
  ns = cdiv(a.max_len, split_len);
  auto run = [&](auto rep_c, auto t_c) -> int {
    constexpr int RP = decltype(rep_c)::value;
    using T16 = decltype(t_c);
    DUO_TRY(ensure_smem_attr(attn_decode_mma_kernel<RP, T16>, kDecodeSmem));
    DUO_CUDA_TRY(::duo::launch_kernel(attn_decode_mma_kernel<RP, T16>, dim3(ns, a.nkv, a.b), 128, kDecodeSmem, st, a, ns, split_len));
    DUO_LAUNCH_CHECK("attn_decode_mma_kernel");
    return DUO_OK;
  };
  auto by_type = [&](auto t_c) -> int {
    switch (rep) {
      case 1: return run(std::integral_constant<int, 1>{}, t_c);
      case 2: return run(std::integral_constant<int, 2>{}, t_c);
      case 3: return run(std::integral_constant<int, 3>{}, t_c);
      default: return run(std::integral_constant<int, 4>{}, t_c);
    }
  };
  DUO_TRY(dtype == DUO_F16 ? by_type(__half{}) : by_type(__nv_bfloat16{}));
  if (ns > 1) DUO_TRY(launch_attn_combine(a, dtype, ns, st));
  return DUO_OK;
}

}  // namespace duo
