// Gated GQA attention, prefill (t > 1) of the 16-bit engines on the Blackwell tensor cores (tcgen05 + TMEM + TMA).
//
// Flash attention over the KV cache (causal, head dim 256), then the sigmoid gate (transformers Qwen3_5Attention:
// attention, then attn_output * sigmoid(gate); the reference's WGSL does the same per (token, head),
// engine/kernels_qwen35.js:73-123).  One CTA = (row, kv head, tile of 128 / rep query positions); its 128 query rows
// are the rep q heads of that kv head over the same positions, so every K / V tile is loaded once for all of them.
// Key tiles are 128 wide: an M = 128 MMA runs at the tensor core's full rate only from N = 128 up.
//   warp 0     TMA: the Q tile once, then K as 16 KB slabs (128 keys x 64 head dims) through a six-slot ring and V as
//              32 KB halves (64 keys x 256 head dims) through a two-slot ring, in the order the MMAs consume them
//   warp 1     tcgen05: S_j = Q K_j^T (M = 128, N = 128, K = 256) into TMEM buffer j % 2, then
//              O += P_{j-1} V_{j-1} (M = 128, N = 256, K = 128) with P read from TMEM and V straight from its slots
//              as an MN-major operand.  Descriptors are computed once and advanced by adds: one thread issues every
//              MMA, so its instruction count per MMA bounds the pipe at small N.
//   warps 2-9  two threads per query row (warps w and w + 4 share TMEM lanes 32 (w % 4) ..; each takes 64 of a
//              tile's 128 keys and 128 of O's 256 columns): S from TMEM, the causal mask on the tiles that cross the
//              diagonal only, online softmax in base 2 (the pair swaps tile maxima through shared memory), P as
//              16-bit pairs written over the first half of its own S buffer for the next MMA.  O (f32, 256 TMEM
//              columns) is rescaled in place only when a row's running maximum grows by more than 2^8 (until then
//              P is formed against the older maximum, so P <= 2^8); at the end O / l times sigmoid(gate) is stored.
// TMEM: S_0, S_1 (128 f32 columns each, P inside), O (256) = all 512.  S_{j+2} is issued only once P_j V_j has
// completed (it overwrites P_j).  Barriers: q_full; k_full / k_empty per K slot, v_full / v_empty per V slot; s_full,
// p_full, pv_done per S buffer.  A barrier's next completion always needs an arrival its waiter has not made yet, so
// no phase is skipped.  Cache entries past a row's length are read and masked; V there must be finite (0 x inf would
// poison O), which the engine's zero-filled caches are.
#include "kernels.cuh"
#include "tc.cuh"

namespace duo {
namespace {

constexpr int AT_THREADS = 320, AT_BK = 128, AT_HD = 256;
constexpr int KSLOTS = 6, VSLOTS = 2;
constexpr uint32_t KSLAB = 16384, VHALF = 32768;
constexpr uint32_t AO_Q = 0, AO_K = 65536, AO_V = AO_K + KSLOTS * KSLAB, AO_BAR = AO_V + VSLOTS * VHALF;
// tile maxima of the two threads of a row [parity][half][row] (a failed thread publishes the pattern kBad)
constexpr uint32_t AO_RED = AO_BAR + 256;
constexpr int AT_SMEM = AO_RED + 2 * 2 * 128 * 4;  // the base is checked to be 1024-aligned at run time
static_assert(AT_SMEM <= 232448, "shared memory");
constexpr uint32_t kBad = 0xFFFFFFFFu;  // a NaN that fmaxf never returns
constexpr uint32_t TA_S = 0, TA_O = 256, TA_COLS = 512;
constexpr float RESCALE_AT = 8.f;  // log2 units

template <typename T16> __device__ __forceinline__ uint32_t pack2_16(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2_16<__nv_bfloat16>(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <> __device__ __forceinline__ uint32_t pack2_16<__half>(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ float ex2(float x) {  // 2^x on the SFU (ex2.approx, 2 ulp; 2^-inf = 0)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T16, int REP>
__global__ void __launch_bounds__(AT_THREADS, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                           const __grid_constant__ CUtensorMap tv, AttnArgs a, unsigned* fault) {
  constexpr int QT = 128 / REP;  // query positions per CTA
  constexpr bool BF = std::is_same<T16, __nv_bfloat16>::value;
  constexpr uint32_t ID_S = tc::idesc_16_mn(128, AT_BK, BF, false, false);
  constexpr uint32_t ID_PV = tc::idesc_16_mn(128, AT_HD, BF, false, true);
  if (tc::fault_pending(fault)) {  // an earlier kernel gave up a wait
    pdl_wait();
    return;
  }
  extern __shared__ __align__(1024) uint8_t sm[];
  const uint32_t sb = tc::smem_u32(sm);
  if (sb & 1023u) {  // the swizzled tiles need a 1024-byte aligned base; never observed otherwise
    if (threadIdx.x == 0) atomicOr(fault, 256u);
    pdl_wait();
    return;
  }
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + AO_BAR);
  uint64_t* q_full = bar;        // [1]
  uint64_t* k_full = bar + 1;    // [KSLOTS]
  uint64_t* k_empty = bar + 7;   // [KSLOTS]
  uint64_t* v_full = bar + 13;   // [VSLOTS]
  uint64_t* v_empty = bar + 15;  // [VSLOTS]
  uint64_t* s_full = bar + 17;   // [2]
  uint64_t* p_full = bar + 19;   // [2]
  uint64_t* pv_done = bar + 21;  // [2]
  uint64_t* drain = bar + 23;    // [1] the issuer's last commit: every MMA of this CTA complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 24);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(sm + AO_RED);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qt = gridDim.x - 1 - blockIdx.x;  // the longest (latest) query tiles first
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int R = a.cache_row0 + b;

  if (tid == 0) {
    tc::mbar_init(q_full, 1);
    for (int i = 0; i < KSLOTS; i++) {
      tc::mbar_init(&k_full[i], 1);
      tc::mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < VSLOTS; i++) {
      tc::mbar_init(&v_full[i], 1);
      tc::mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      tc::mbar_init(&s_full[i], 1);
      tc::mbar_init(&p_full[i], 256);
      tc::mbar_init(&pv_done[i], 1);
    }
    tc::mbar_init(drain, 1);
    *abort = 0;
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tq);
    tc::prefetch_tmap(&tk);
    tc::prefetch_tmap(&tv);
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, TA_COLS);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  pdl_trigger();

  const int p0 = a.start ? a.start[R] : a.len[R] - a.t;
  const int tq0 = qt * QT;
  const int nq = min(QT, a.t - tq0);
  const int n_keys = p0 + tq0 + nq;
  const int ntiles = (n_keys + AT_BK - 1) / AT_BK;

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer: Q; K_0; then K_{j+1} and V_j for j = 0, 1, ...
      // K slab u = 4 j + (head-dim quarter) lives in slot u % KSLOTS; V half v = 2 j + (key half) in slot v % VSLOTS.
      // A slot's barriers complete once per use (parity (u / slots) & 1); its next use waits for the previous one.
      auto load_k = [&](int j) -> bool {
        for (int q = 0; q < 4; q++) {
          const int u = 4 * j + q, sl = u % KSLOTS;
          if (u >= KSLOTS && !tc::mbar_wait(&k_empty[sl], (uint32_t)((u / KSLOTS - 1) & 1))) return false;
          tc::mbar_arrive_expect_tx(&k_full[sl], KSLAB);
          tc::tma_load_4d(sm + AO_K + sl * KSLAB, &tk, q * 64, kvh, j * AT_BK, b, &k_full[sl]);
        }
        return true;
      };
      auto load_v = [&](int j) -> bool {
        for (int h = 0; h < 2; h++) {
          const int v = 2 * j + h, sl = v % VSLOTS;
          if (v >= VSLOTS && !tc::mbar_wait(&v_empty[sl], (uint32_t)((v / VSLOTS - 1) & 1))) return false;
          tc::mbar_arrive_expect_tx(&v_full[sl], VHALF);
          for (int q = 0; q < 4; q++)
            tc::tma_load_4d(sm + AO_V + sl * VHALF + q * 8192, &tv, q * 64, kvh, j * AT_BK + h * 64, b, &v_full[sl]);
        }
        return true;
      };
      tc::mbar_arrive_expect_tx(q_full, 128 * AT_HD * 2);
      for (int hl = 0; hl < REP; hl++)
        for (int qq = 0; qq < 4; qq++)
          tc::tma_load_4d(sm + AO_Q + qq * 16384 + hl * QT * 128, &tq, qq * 64, kvh * REP + hl, tq0, b, q_full);
      int nk = 0, nv = 0;  // tiles requested
      bool ok = load_k(0);
      nk = ok ? 1 : 0;
      for (int j = 0; ok && j < ntiles && !*abort; j++) {
        if (j + 1 < ntiles) {
          if (!(ok = load_k(j + 1))) break;
          nk = j + 2;
        }
        if (!(ok = load_v(j))) break;
        nv = j + 1;
      }
      if (!ok) {
        atomicOr(fault, 128u);
        *abort = 1;
      }
      // no copy may still be landing when the CTA exits: wait (bounded) for Q and every slot's last use
      tc::mbar_wait(q_full, 0);
      for (int u = max(0, 4 * nk - KSLOTS); u < 4 * nk; u++)
        tc::mbar_wait(&k_full[u % KSLOTS], (uint32_t)((u / KSLOTS) & 1));
      for (int v = max(0, 2 * nv - VSLOTS); v < 2 * nv; v++)
        tc::mbar_wait(&v_full[v % VSLOTS], (uint32_t)((v / VSLOTS) & 1));
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer
      // descriptor of each operand base; a byte offset o inside a swizzled region adds o >> 4 (start-address field)
      const uint64_t dq = tc::desc_sw128(sb + AO_Q, 16, 1024);
      const uint64_t dk = tc::desc_sw128(sb + AO_K, 16, 1024);
      const uint64_t dv = tc::desc_sw128(sb + AO_V, 8192, 1024);
      bool ok = tc::mbar_wait(q_full, 0);
      auto pv = [&](int jp) -> bool {
        const int bf = jp & 1;
        if (!tc::mbar_wait(&p_full[bf], (uint32_t)((jp >> 1) & 1))) return false;
        for (int h = 0; h < 2; h++) {
          const int v = 2 * jp + h, sl = v % VSLOTS;
          if (!tc::mbar_wait(&v_full[sl], (uint32_t)((v / VSLOTS) & 1))) return false;
          tc::fence_after_sync();
          const uint64_t d0 = dv + ((sl * VHALF) >> 4);
#pragma unroll
          for (int ks = 0; ks < 4; ks++)  // keys 64 h + 16 ks ..: 2048 bytes of the half per step
            tc::mma_ts(tmem + TA_O, tmem + TA_S + bf * 128 + h * 32 + ks * 8, d0 + ks * 128, ID_PV,
                       (jp > 0 || h > 0 || ks > 0) ? 1u : 0u);
          tc::mma_commit(&v_empty[sl]);
        }
        tc::mma_commit(&pv_done[bf]);
        return true;
      };
      for (int j = 0; ok && j < ntiles && !*abort; j++) {
        const int bf = j & 1;
        // S_j overwrites P_{j-2} (same buffer): P_{j-2} V_{j-2} must have completed
        if (j >= 2 && !tc::mbar_wait(&pv_done[bf], (uint32_t)(((j - 2) >> 1) & 1))) {
          ok = false;
          break;
        }
        for (int q = 0; q < 4 && ok; q++) {
          const int u = 4 * j + q, sl = u % KSLOTS;
          if (!tc::mbar_wait(&k_full[sl], (uint32_t)((u / KSLOTS) & 1))) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint64_t a0 = dq + ((q * 16384) >> 4), b0 = dk + ((sl * KSLAB) >> 4);
#pragma unroll
          for (int ks = 0; ks < 4; ks++)  // 16 head dims = 32 bytes of the K-major rows per step
            tc::mma_bf16(tmem + TA_S + bf * 128, a0 + ks * 2, b0 + ks * 2, ID_S, (q > 0 || ks > 0) ? 1u : 0u);
          tc::mma_commit(&k_empty[sl]);
        }
        if (!ok) break;
        tc::mma_commit(&s_full[bf]);
        if (j >= 1 && !pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && !*abort && ntiles > 0) ok = pv(ntiles - 1);
      if (!ok) {
        atomicOr(fault, 128u);
        *abort = 1;
      }
      tc::mma_commit(drain);  // arrives once every MMA issued above has completed
      tc::mbar_wait(drain, 0);
    }
  } else {  // ---- softmax and epilogue: two threads per query row
    const int qw = warp & 3, half = (warp - 2) >> 2, r = qw * 32 + lane;
    const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
    const int hl = r / QT, qi = r % QT;
    const int pos = p0 + tq0 + qi;
    const int diag = p0 + tq0;  // tiles whose last key is past this (or past n_keys) need the mask
    const float sl2 = a.scale * 1.4426950408889634f;
    float m = -INFINITY, l = 0.f;  // m: running maximum of the scaled scores (log2 units)
    // The two threads of a row meet at one named barrier per tile and one in the epilogue, always the same number of
    // times: a failed wait only marks `bad`, and both leave the loop together right after the barrier that shows it.
    bool bad = false;
    for (int j = 0; j < ntiles; j++) {
      const int bf = j & 1;
      if (!bad && (!tc::mbar_wait(&s_full[bf], (uint32_t)((j >> 1) & 1)) || *abort)) bad = true;
      float x[64];
      float mt = -INFINITY;
      if (!bad) {
        tc::fence_after_sync();
        uint32_t raw0[32], raw1[32];
        tc::tmem_ld32_issue(tmem + TA_S + bf * 128 + half * 64 + lane_off, raw0);
        tc::tmem_ld32_issue(tmem + TA_S + bf * 128 + half * 64 + 32 + lane_off, raw1);
        tc::tmem_ld_wait(raw0);
        tc::tmem_ld_wait(raw1);
#pragma unroll
        for (int c = 0; c < 32; c++) {
          x[c] = __uint_as_float(raw0[c]);
          x[32 + c] = __uint_as_float(raw1[c]);
        }
        const int k0 = j * AT_BK + half * 64;
        if (j * AT_BK + AT_BK - 1 > diag || j * AT_BK + AT_BK > n_keys) {
#pragma unroll
          for (int c = 0; c < 64; c++)
            if (k0 + c > pos || k0 + c >= n_keys) x[c] = -INFINITY;
        }
        float mx[8];
#pragma unroll
        for (int c = 0; c < 8; c++) mx[c] = x[c];
#pragma unroll
        for (int c = 8; c < 64; c++) mx[c & 7] = fmaxf(mx[c & 7], x[c]);
        mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      }
      red[(bf * 2 + half) * 128 + r] = bad ? __uint_as_float(kBad) : mt;
      tc::bar_sync(1 + qw, 64);
      const float mo = red[(bf * 2 + (half ^ 1)) * 128 + r];
      if (bad || __float_as_uint(mo) == kBad) {
        bad = true;
        break;
      }
      mt = fmaxf(mt, mo) * sl2;
      if (mt > m + RESCALE_AT) {  // both threads of the row take this branch together (same m, same mt)
        if (j > 0) {  // O holds P_{<j} V against the old maximum: rescale this half once PV_{j-1} is in
          const float al = ex2(m - mt);
          if (!tc::mbar_wait(&pv_done[(j - 1) & 1], (uint32_t)(((j - 1) >> 1) & 1))) {
            bad = true;
            continue;
          }
          tc::fence_after_sync();
#pragma unroll 1
          for (int c0 = 0; c0 < 128; c0 += 32) {
            float v[32];
            tc::tmem_ld32(tmem + TA_O + half * 128 + c0 + lane_off, v);
#pragma unroll
            for (int e = 0; e < 32; e++) v[e] *= al;
            tc::tmem_st32(tmem + TA_O + half * 128 + c0 + lane_off, v);
          }
          l *= al;
        }
        m = mt;
      }
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const float e0 = ex2(fmaf(x[c], sl2, -m)), e1 = ex2(fmaf(x[c + 1], sl2, -m));
        ls[(c >> 1) & 3] += e0 + e1;
        pk[c >> 1] = pack2_16<T16>(e0, e1);
      }
      l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      // keys 64 half .. + 63 as 16-bit pairs: columns 32 half .. + 31 of this tile's S buffer (both threads of the
      // row have read their S columns: they met at the barrier above)
      tc::tmem_st32(tmem + TA_S + bf * 128 + half * 32 + lane_off, reinterpret_cast<const float*>(pk));
      tc::fence_before_sync();
      tc::mbar_arrive(&p_full[bf]);
    }
    bool ok = !bad;
    // epilogue: O / l * sigmoid(gate); the row's l is the sum of both halves' (through the parity buffer that the
    // last tile did not use: its last reader finished before that tile's barrier)
    red[((ntiles & 1) * 2 + half) * 128 + r] = l;
    tc::bar_sync(1 + qw, 64);
    l += red[((ntiles & 1) * 2 + (half ^ 1)) * 128 + r];
    if (ok && ntiles > 0) ok = tc::mbar_wait(&pv_done[(ntiles - 1) & 1], (uint32_t)(((ntiles - 1) >> 1) & 1));
    if (!ok) {
      atomicOr(fault, 128u);
      *abort = 1;
    } else {
      tc::fence_after_sync();
      const bool valid = qi < nq;
      const int head = kvh * REP + hl;
      const long tok = (long)b * a.t + tq0 + qi;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const T16* gp = a.gate ? static_cast<const T16*>(a.gate) + tok * a.gate_stride + (long)head * a.gate_hstride
                             : nullptr;
      T16* op = static_cast<T16*>(a.o) + (tok * a.nh + head) * AT_HD;
#pragma unroll 1
      for (int c0 = half * 128; c0 < half * 128 + 128; c0 += 32) {
        uint4 graw[4];
        if (gp && valid)
#pragma unroll
          for (int i = 0; i < 4; i++) graw[i] = *reinterpret_cast<const uint4*>(gp + c0 + 8 * i);
        float v[32];
        tc::tmem_ld32(tmem + TA_O + c0 + lane_off, v);
        if (valid) {
#pragma unroll
          for (int i = 0; i < 4; i++) {
            float g[8];
            if (gp) load8(reinterpret_cast<const T16*>(&graw[i]), g);
            uint4 u;
            uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
            for (int e = 0; e < 4; e++) {
              float o0 = v[8 * i + 2 * e] * inv, o1 = v[8 * i + 2 * e + 1] * inv;
              if (gp) {
                o0 /= 1.f + __expf(-g[2 * e]);
                o1 /= 1.f + __expf(-g[2 * e + 1]);
              }
              w[e] = pack2_16<T16>(o0, o1);
            }
            *reinterpret_cast<uint4*>(op + c0 + 8 * i) = u;
          }
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {  // the issuer waited on `drain` above: no MMA reads or writes this CTA's TMEM any more
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, TA_COLS);
  }
}

template <typename T16, int REP>
int run_attn_tc(const AttnArgs& a, int dtype, cudaStream_t st) {
  constexpr int QT = 128 / REP;
  const long hd = AT_HD, es = 2;
  CUtensorMap tq, tk, tv;
  {
    const long dims[4] = {hd, a.nh, a.t, a.b};
    const long strides[3] = {hd * es, a.nh * hd * es, (long)a.t * a.nh * hd * es};
    const int box[4] = {64, 1, QT, 1};
    DUO_TRY(make_tmap_nd_16(&tq, a.q, dtype, 4, dims, strides, box));
  }
  {
    const long dims[4] = {hd, a.nkv, a.max_len, a.b};
    const long strides[3] = {hd * es, a.nkv * hd * es, (long)a.max_len * a.nkv * hd * es};
    const int kbox[4] = {64, 1, AT_BK, 1}, vbox[4] = {64, 1, 64, 1};
    const long row0 = (long)a.cache_row0 * a.max_len * a.nkv * hd;
    DUO_TRY(make_tmap_nd_16(&tk, static_cast<const T16*>(a.kc) + row0, dtype, 4, dims, strides, kbox));
    DUO_TRY(make_tmap_nd_16(&tv, static_cast<const T16*>(a.vc) + row0, dtype, 4, dims, strides, vbox));
  }
  unsigned* fault = tc_fault_ptr();
  if (!fault) return fail(DUO_ECUDA, "tensor-core fault word is not addressable");
  DUO_TRY(ensure_smem_attr(attn_prefill_tc_kernel<T16, REP>, AT_SMEM));
  DUO_CUDA_TRY(::duo::launch_kernel(attn_prefill_tc_kernel<T16, REP>, dim3(cdiv(a.t, QT), a.nkv, a.b), AT_THREADS,
                                    AT_SMEM, st, tq, tk, tv, a, fault));
  DUO_LAUNCH_CHECK("attn_prefill_tc_kernel");
  return DUO_OK;
}

}  // namespace

bool attn_prefill_tc_eligible(const AttnArgs& a, int dtype) {
  if (dtype != DUO_BF16 && dtype != DUO_F16) return false;
  if (a.hd != AT_HD || a.t < 2 || a.nkv <= 0 || a.nh % a.nkv) return false;
  const int rep = a.nh / a.nkv;
  if (rep != 1 && rep != 2 && rep != 4) return false;
  const auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al(a.q) || !al(a.kc) || !al(a.vc) || !al(a.o) || (a.gate && !al(a.gate))) return false;
  if (a.gate && (a.gate_stride % 8 || a.gate_hstride % 8)) return false;
  return true;
}

int launch_attn_prefill_tc(const AttnArgs& a, int dtype, cudaStream_t st) {
  if (a.b == 0 || a.t == 0) return DUO_OK;
  const int rep = a.nh / a.nkv;
  if (dtype == DUO_F16) {
    if (rep == 4) return run_attn_tc<__half, 4>(a, dtype, st);
    if (rep == 2) return run_attn_tc<__half, 2>(a, dtype, st);
    return run_attn_tc<__half, 1>(a, dtype, st);
  }
  if (rep == 4) return run_attn_tc<__nv_bfloat16, 4>(a, dtype, st);
  if (rep == 2) return run_attn_tc<__nv_bfloat16, 2>(a, dtype, st);
  return run_attn_tc<__nv_bfloat16, 1>(a, dtype, st);
}

}  // namespace duo
