// Decode-sized tcgen05 GEMM (8 < M <= 256 rows): C[m, n] = sum_k X[m, k] W[n, k] with the weights on the MMA's M side.
//
// With few rows the cost of a GEMM is streaming the weights, and tiling the row side re-reads the activations once per
// weight tile.  Here a CTA owns 128 weight rows (MMA M = 128) and ALL rows of X (MMA N = NB = 64 / 128 / 256, rows
// past M read as zeros), so X is read once per 128 weight rows, and K is split over a thread-block cluster of KS <= 8
// CTAs (grid y = cluster rank) so that each CTA's K slice is in flight at once.  Each CTA moves its 128 x NB f32
// partial tile TMEM -> shared memory (m-major); after a cluster barrier CTA z sums rows [z R, z R + R) of the KS
// partials over distributed shared memory in rank order (deterministic) and runs the epilogue on them with
// consecutive lanes on consecutive weight rows n, i.e. coalesced along the output row: store (16-bit or f32) or
// SwiGLU (+ pushes) for gate/up packs interleaved per 64 rows.  (The residual-add projections, N = 1024 with long K,
// stay on gemm.cu's per-tile kernel: split 8 ways here, every CTA would pull 128 KB of partials over DSMEM.)
//
// The arithmetic is the reference's matmul (engine/kernels.js:97-151): f32 accumulation of products of the 16-bit
// operands; the per-row int8 scale (colscale) multiplies the reduced sum.
#include <cooperative_groups.h>

#include <algorithm>

#include "kernels.cuh"
#include "tc.cuh"

namespace cg = cooperative_groups;

namespace duo {

namespace {

constexpr int DBM = 128, DBK = 64, DTHREADS = 256, DP = DBM + 4;  // DP: partial-tile row pitch (floats)

template <int NB> struct DCfg {
  static constexpr int W_BYTES = DBM * DBK * 2;
  static constexpr int X_BYTES = NB * DBK * 2;
  static constexpr int STAGE_BYTES = W_BYTES + X_BYTES;
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES;
  static constexpr int RING = STAGES * STAGE_BYTES;
  static constexpr int SMEM = 1024 + RING + 256;
  static_assert(NB * DP * 4 <= RING, "the partial tile must fit in the ring");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

template <int NB, int EPI, bool F16>
__global__ void __launch_bounds__(DTHREADS, 1)
    gemm_dec_kernel(const __grid_constant__ CUtensorMap tma_w, const __grid_constant__ CUtensorMap tma_x, int M,
                    int N, int K, int kper, GemmEpiArgs ep, unsigned* fault) {
  using C = DCfg<NB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sw = smem;
  uint8_t* sx = smem + C::STAGES * C::W_BYTES;
  float* part = reinterpret_cast<float*>(smem);  // [NB][DP], reuses the ring once every MMA has completed
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::RING);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tmem_full = empty + C::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * DBM;
  const int ks = gridDim.y, z = blockIdx.y;
  const int kb0 = z * kper;
  const int num_k = max(0, min(kper, K / DBK - kb0));

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; s++) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(tmem_full, 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tma_w);
    tc::prefetch_tmap(&tma_x);
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, NB);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  // Programmatic launch: constant weight tiles of the first stages stream in while the preceding kernel finishes.
  const int pre = ep.b_const ? min(num_k, C::STAGES) : 0;
  if (warp == 0 && lane == 0) {
    for (int kb = 0; kb < pre; kb++) {
      tc::mbar_arrive_expect_tx(&full[kb], C::STAGE_BYTES);
      tc::tma_load_2d(sw + kb * C::W_BYTES, &tma_w, (kb0 + kb) * DBK, n0, &full[kb]);
    }
  }
  pdl_wait();
  pdl_trigger();

  bool ok = true;
  if (warp == 0 && lane == 0) {
    for (int kb = 0; kb < num_k; kb++) {
      const int s = kb % C::STAGES;
      const uint32_t ph = (kb / C::STAGES) & 1;
      if (kb < pre) {
        tc::tma_load_2d(sx + s * C::X_BYTES, &tma_x, (kb0 + kb) * DBK, 0, &full[s]);
        continue;
      }
      if (kb >= C::STAGES && !tc::mbar_wait(&empty[s], ph ^ 1)) {
        atomicOr(fault, 1u);
        break;
      }
      tc::mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
      tc::tma_load_2d(sw + s * C::W_BYTES, &tma_w, (kb0 + kb) * DBK, n0, &full[s]);
      tc::tma_load_2d(sx + s * C::X_BYTES, &tma_x, (kb0 + kb) * DBK, 0, &full[s]);
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = tc::idesc_16_f32(DBM, NB, F16);
    for (int kb = 0; kb < num_k; kb++) {
      const int s = kb % C::STAGES;
      const uint32_t ph = (kb / C::STAGES) & 1;
      if (!tc::mbar_wait(&full[s], ph)) {
        atomicOr(fault, 2u);
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const uint32_t a0 = tc::smem_u32(sw + s * C::W_BYTES), b0 = tc::smem_u32(sx + s * C::X_BYTES);
#pragma unroll
      for (int k = 0; k < DBK / 16; k++)
        tc::mma_bf16(tmem, tc::desc_kmajor_sw128(a0 + k * 32), tc::desc_kmajor_sw128(b0 + k * 32), idesc,
                     (kb | k) != 0);
      tc::mma_commit(&empty[s]);
    }
    if (ok) tc::mma_commit(tmem_full);
  }
  // partial tile TMEM -> shared memory, m-major, by all 8 warps once the MMAs are done: warp w holds weight rows
  // 32 (w % 4) .. + 31 (its TMEM lane quarter) and columns [(w / 4) NB / 2, + NB / 2)
  bool have = true;
  {
    __syncwarp();  // warps 0 and 1 reconverge after their single-lane roles (tcgen05.ld is warp-wide)
    const int quad = warp & 3, half = warp >> 2;
    const int n = quad * 32 + lane;
    if (num_k > 0) {
      have = tc::mbar_wait(tmem_full, 0);
      if (!have) {
        if (lane == 0) atomicOr(fault, 4u);
      } else {
        tc::fence_after_sync();
        const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
#pragma unroll 1
        for (int c0 = half * (NB / 2); c0 < (half + 1) * (NB / 2); c0 += 32) {
          uint32_t r[32];
          tc::tmem_ld32_issue(trow + c0, r);
          tc::tmem_ld_wait(r);
#pragma unroll
          for (int j = 0; j < 32; j++) part[(c0 + j) * DP + n] = __uint_as_float(r[j]);
        }
      }
    } else {  // an empty K slice contributes zeros
      for (int m = half * (NB / 2); m < (half + 1) * (NB / 2); m++) part[m * DP + n] = 0.f;
    }
  }
  // every partial of the cluster is in shared memory
  if (ks > 1) cg::this_cluster().sync();
  else __syncthreads();

  // reduce rows [z R, z R + R) over the cluster and run the epilogue; 8 warps, one or two rows per warp step
  const int mrows = min(M, NB);
  const int R = (mrows + ks - 1) / ks;
  const int m_lo = z * R, m_hi = min(mrows, m_lo + R);
  const bool v16 = (reinterpret_cast<uintptr_t>(ep.c) & 15) == 0 && ep.ldc % 4 == 0;
  cg::cluster_group cluster = cg::this_cluster();
  // Every partial of a batch of RB rows is loaded (distributed shared memory, all ranks unrolled) before any result
  // is stored, so the remote-load latency is paid about once per batch rather than once per row and rank.
  constexpr int RB = 4;
  auto gather = [&](const int (&ms)[RB], int col, float4 (&out)[RB]) {  // out[i] = sum over ranks of part[ms[i]][col..]
#pragma unroll
    for (int i = 0; i < RB; i++) out[i] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int q = 0; q < 8; q++) {
      if (q < ks) {
        const float* pq = ks > 1 ? cluster.map_shared_rank(part, q) : part;
        float4 v[RB];
#pragma unroll
        for (int i = 0; i < RB; i++)
          if (ms[i] >= 0) v[i] = *reinterpret_cast<const float4*>(pq + ms[i] * DP + col);
#pragma unroll
        for (int i = 0; i < RB; i++) {
          if (ms[i] < 0) continue;
          out[i].x += v[i].x; out[i].y += v[i].y; out[i].z += v[i].z; out[i].w += v[i].w;
        }
      }
    }
  };
  auto store4_16 = [&](long off, const float* o) {  // 4 consecutive 16-bit outputs, one 8-byte store when aligned
    uint32_t w[2];
    for (int i = 0; i < 2; i++) {
      if (ep.c_dtype == DUO_BF16) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
      } else {
        const __half2 h = __floats2half2_rn(o[2 * i], o[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
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
    float cg_[4] = {1.f, 1.f, 1.f, 1.f}, cu_[4] = {1.f, 1.f, 1.f, 1.f};
    if (ep.colscale) {
      for (int i = 0; i < 4; i++) {
        cg_[i] = ep.colscale[n0 + j4 + i];
        cu_[i] = ep.colscale[n0 + 64 + j4 + i];
      }
    }
    for (int mb = m_lo + warp * 2 + (lane >> 4); mb < m_hi; mb += 16 * RB) {
      int ms[RB];
#pragma unroll
      for (int i = 0; i < RB; i++) ms[i] = mb + 16 * i < m_hi ? mb + 16 * i : -1;
      float4 g[RB], u[RB];
      gather(ms, j4, g);
      gather(ms, 64 + j4, u);
#pragma unroll
      for (int i = 0; i < RB; i++) {
        const int m = mb + 16 * i;
        if (m >= m_hi) break;
        const float gv[4] = {g[i].x, g[i].y, g[i].z, g[i].w}, uv[4] = {u[i].x, u[i].y, u[i].z, u[i].w};
        const int r = ep.row_base + m / ep.t;
        float o[4];
#pragma unroll
        for (int c = 0; c < 4; c++) {
          o[c] = siluf_(gv[c] * cg_[c]) * (uv[c] * cu_[c]);
          if (ep.push.count) o[c] = push_apply(ep.push, r, nout + c, o[c]);
        }
        store4_16((long)m * ep.ldc + nout, o);
      }
    }
  } else {
    // one row per warp step: lane -> weight rows n0 + 4 lane .. + 3
    const int n = n0 + lane * 4;
    float cs[4] = {1.f, 1.f, 1.f, 1.f};
    if (ep.colscale) {
      for (int i = 0; i < 4; i++) cs[i] = (n + i < N) ? ep.colscale[n + i] : 0.f;
    }
    for (int mb = m_lo + warp; mb < m_hi; mb += 8 * RB) {
      if (n >= N) break;
      int ms[RB];
#pragma unroll
      for (int i = 0; i < RB; i++) ms[i] = mb + 8 * i < m_hi ? mb + 8 * i : -1;
      float4 a[RB];
      gather(ms, lane * 4, a);
#pragma unroll
      for (int i = 0; i < RB; i++) {
        const int m = mb + 8 * i;
        if (m >= m_hi) break;
        float x[4] = {a[i].x * cs[0], a[i].y * cs[1], a[i].z * cs[2], a[i].w * cs[3]};
        const long off = (long)m * ep.ldc + n;
        const bool full4 = v16 && n + 4 <= N;
        if (ep.c_dtype == DUO_F32) {
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
  if (ks > 1) cg::this_cluster().sync();  // no CTA leaves while a peer may still read its partial
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, NB);
  }
  (void)have;
}

template <int NB, int EPI, bool F16>
int run_dec(const CUtensorMap& tw, const CUtensorMap& tx, int m, int n, int k, const GemmEpiArgs& ep,
            cudaStream_t st) {
  using C = DCfg<NB>;
  static bool attr_set = false;
  auto kern = gemm_dec_kernel<NB, EPI, F16>;
  if (!attr_set) {
    DUO_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr_set = true;
  }
  unsigned* fault = tc_fault_ptr();
  if (!fault) return fail(DUO_ECUDA, "tensor-core fault word is not addressable");
  const int nblocks = cdiv(n, DBM);
  const int num_k = k / DBK;
  // split K so that the grid roughly covers the SMs once (one CTA per SM), at most 8 ways (portable cluster size)
  int ks = std::max(1, std::min({sm_count() / nblocks, 8, num_k}));
  const int kper = cdiv(num_k, ks);
  ks = cdiv(num_k, kper);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nblocks, ks);
  cfg.blockDim = dim3(DTHREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (ks > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = ks;
    attr[na].val.clusterDim.z = 1;
    na++;
  }
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    na++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  DUO_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, tw, tx, m, n, k, kper, ep, fault));
  DUO_LAUNCH_CHECK("gemm_dec_kernel");
  return DUO_OK;
}

template <int NB, bool F16>
int dispatch_dec(const CUtensorMap& tw, const CUtensorMap& tx, int m, int n, int k, const GemmEpiArgs& ep,
                 cudaStream_t st) {
  if (ep.epi == EPI_SWIGLU) return run_dec<NB, EPI_SWIGLU, F16>(tw, tx, m, n, k, ep, st);
  return run_dec<NB, EPI_STORE, F16>(tw, tx, m, n, k, ep, st);
}

}  // namespace

int launch_gemm_dec(const void* x, int m, int k, const void* w, int n, int ab_dtype, const GemmEpiArgs& ep,
                    cudaStream_t st) {
  if (m == 0 || n == 0) return DUO_OK;
  DUO_CHECK_ARG(m <= 256, "gemm_dec: at most 256 rows");
  DUO_CHECK_ARG(k % DBK == 0, "gemm_dec: k must be a multiple of 64");
  DUO_CHECK_ARG(ab_dtype == DUO_BF16 || ab_dtype == DUO_F16, "gemm_dec: operands must be bf16 or f16");
  DUO_CHECK_ARG(ep.epi == EPI_STORE || ep.epi == EPI_SWIGLU, "gemm_dec: store or SwiGLU epilogue only");
  if (ep.epi == EPI_SWIGLU) {
    DUO_CHECK_ARG(n % 128 == 0, "gemm_dec: SwiGLU needs n a multiple of 128");
    DUO_CHECK_ARG(ep.c_dtype == ab_dtype, "gemm_dec: SwiGLU output is 16-bit");
  }
  const int nb = m <= 64 ? 64 : m <= 128 ? 128 : 256;
  CUtensorMap tw, tx;
  DUO_TRY(make_tmap_16(&tw, w, ab_dtype, n, k, k, DBM, DBK));
  DUO_TRY(make_tmap_16(&tx, x, ab_dtype, m, k, k, nb, DBK));
  if (ab_dtype == DUO_F16) {
    if (nb == 64) return dispatch_dec<64, true>(tw, tx, m, n, k, ep, st);
    if (nb == 128) return dispatch_dec<128, true>(tw, tx, m, n, k, ep, st);
    return dispatch_dec<256, true>(tw, tx, m, n, k, ep, st);
  }
  if (nb == 64) return dispatch_dec<64, false>(tw, tx, m, n, k, ep, st);
  if (nb == 128) return dispatch_dec<128, false>(tw, tx, m, n, k, ep, st);
  return dispatch_dec<256, false>(tw, tx, m, n, k, ep, st);
}

}  // namespace duo
