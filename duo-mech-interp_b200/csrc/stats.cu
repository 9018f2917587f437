// Next-token statistics of the push probe: log-softmax normaliser, probability mass and weighted log-probability of a
// set of target ids, and the change against an unsteered row of the same context (KL, mass gain, log-odds gain, the
// per-vocabulary log-probability delta).
//
// Reference: the probe of engine/analysis.js:480-537 (logSoftmax 693-702, lse 665, kl 704-708) and its PyTorch form
// tools/find_steering.py:86-103.  The reference computes them on the host from the logits it reads back; here they
// are two HBM-streaming kernels over the logits on the device:
//   row pass   one CTA per row: online max / sum of exponentials over the vocabulary with 16-byte loads, then the
//              targets (a few dozen gathered values) -> lse, mass, tlse;
//   pair pass  one CTA per row that has a base row: reads both rows once more, sum of p (lp - lb) over p > 1e-12 ->
//              kl, and (optionally) d += lp - lb; thread 0 also writes dp and gain from the two rows' row-pass values.
// Algorithmic bytes: 4 vocab bytes per row (row pass) + 8 vocab bytes per steered row (pair pass) + 8 more with d.
#include <cmath>

#include "kernels.cuh"

namespace duo {
namespace {

constexpr int ST_THREADS = 512;
constexpr float kPMin = 1e-12f;  // the reference's KL ignores terms with p <= 1e-12 (analysis.js:706)

// block-wide (max, sum of exp(x - max)) merge for ST_THREADS threads
__device__ __forceinline__ void merge_ms(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  s = (m == -INFINITY ? 0.f : s * expf(m - mn)) + (m2 == -INFINITY ? 0.f : s2 * expf(m2 - mn));
  m = mn;
}

__global__ void __launch_bounds__(ST_THREADS) stats_row_kernel(const float* __restrict__ logits, long ld, int vocab,
                                                               const int32_t* __restrict__ tid,
                                                               const float* __restrict__ tlw, int nt,
                                                               float* __restrict__ stats) {
  pdl_enter();
  const int r = blockIdx.x;
  const float* x = logits + (long)r * ld;
  float m = -INFINITY, s = 0.f;
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  const int nv = vec ? vocab / 4 : 0;
  for (int i = threadIdx.x; i < nv; i += ST_THREADS) {
    const float4 v = __ldcs(reinterpret_cast<const float4*>(x) + i);
    const float m4 = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
    if (m4 > m) {
      s = (m == -INFINITY) ? 0.f : s * __expf(m - m4);
      m = m4;
    }
    if (m != -INFINITY) s += __expf(v.x - m) + __expf(v.y - m) + __expf(v.z - m) + __expf(v.w - m);
  }
  for (int i = 4 * nv + threadIdx.x; i < vocab; i += ST_THREADS) {
    const float v = x[i];
    if (v > m) {
      s = (m == -INFINITY) ? 0.f : s * __expf(m - v);
      m = v;
    }
    if (m != -INFINITY) s += __expf(v - m);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) merge_ms(m, s, __shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, s, o));
  __shared__ float sm[32], ss[32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) { sm[w] = m; ss[w] = s; }
  __syncthreads();
  __shared__ float lse_s;
  if (w == 0) {
    m = lane < ST_THREADS / 32 ? sm[lane] : -INFINITY;
    s = lane < ST_THREADS / 32 ? ss[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
      merge_ms(m, s, __shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, s, o));
    if (lane == 0) lse_s = m + logf(s);
  }
  __syncthreads();
  const float lse = lse_s;
  // targets: mass = sum exp(lp[t]); tlse = log sum exp(lp[t] + tlw[t]), one warp
  if (w == 0) {
    float mass = 0.f, tm = -INFINITY, ts = 0.f;
    for (int j = lane; j < nt; j += 32) {
      const int id = tid[j];
      const float lp = (id >= 0 && id < vocab) ? x[id] - lse : -INFINITY;
      mass += lp == -INFINITY ? 0.f : expf(lp);
      const float v = lp + (tlw ? tlw[j] : 0.f);
      if (v > tm) {
        ts = (tm == -INFINITY) ? 0.f : ts * expf(tm - v);
        tm = v;
      }
      ts += v == -INFINITY ? 0.f : expf(v - tm);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mass += __shfl_xor_sync(0xffffffffu, mass, o);
      merge_ms(tm, ts, __shfl_xor_sync(0xffffffffu, tm, o), __shfl_xor_sync(0xffffffffu, ts, o));
    }
    if (lane == 0) {
      float* o = stats + (long)r * DUO_STATS_COLS;
      o[0] = lse;
      o[1] = mass;
      o[2] = tm == -INFINITY ? -INFINITY : tm + logf(ts);
    }
  }
}

__global__ void __launch_bounds__(ST_THREADS) stats_pair_kernel(const float* __restrict__ logits, long ld, int vocab,
                                                                const int32_t* __restrict__ base,
                                                                float* __restrict__ stats, float* __restrict__ d,
                                                                long ldd) {
  pdl_enter();
  const int r = blockIdx.x;
  const int b = base[r];
  float* o = stats + (long)r * DUO_STATS_COLS;
  if (b < 0) {
    if (threadIdx.x == 0) o[3] = o[4] = o[5] = 0.f;
    return;
  }
  const float* x = logits + (long)r * ld;
  const float* y = logits + (long)b * ld;
  float* dr = d ? d + (long)r * ldd : nullptr;
  const float lx = stats[(long)r * DUO_STATS_COLS], ly = stats[(long)b * DUO_STATS_COLS];
  float kl = 0.f;
  const bool vec = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0 &&
                   (dr == nullptr || (reinterpret_cast<uintptr_t>(dr) & 15) == 0);
  const int nv = vec ? vocab / 4 : 0;
  for (int i = threadIdx.x; i < nv; i += ST_THREADS) {
    const float4 a = __ldcs(reinterpret_cast<const float4*>(x) + i);
    const float4 c = __ldcs(reinterpret_cast<const float4*>(y) + i);
    const float la[4] = {a.x - lx, a.y - lx, a.z - lx, a.w - lx};
    const float lb[4] = {c.x - ly, c.y - ly, c.z - ly, c.w - ly};
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const float p = __expf(la[e]);
      if (p > kPMin) kl += p * (la[e] - lb[e]);
    }
    if (dr) {
      float4 dd = reinterpret_cast<float4*>(dr)[i];
      dd.x += la[0] - lb[0]; dd.y += la[1] - lb[1]; dd.z += la[2] - lb[2]; dd.w += la[3] - lb[3];
      reinterpret_cast<float4*>(dr)[i] = dd;
    }
  }
  for (int i = 4 * nv + threadIdx.x; i < vocab; i += ST_THREADS) {
    const float la = x[i] - lx, lb = y[i] - ly;
    const float p = __expf(la);
    if (p > kPMin) kl += p * (la - lb);
    if (dr) dr[i] += la - lb;
  }
  __shared__ float red[32];
  kl = block_sum(kl, red);
  if (threadIdx.x == 0) {
    const float* ob = stats + (long)b * DUO_STATS_COLS;
    o[3] = kl;
    o[4] = o[1] - ob[1];
    o[5] = o[2] - ob[2];
  }
}

}  // namespace

int launch_push_stats(const float* logits, int n, int vocab, long ld, const int32_t* base, const int32_t* tid,
                      const float* tlw, int nt, float* stats, float* d, long ldd, cudaStream_t st) {
  if (n == 0) return DUO_OK;
  DUO_CUDA_TRY(::duo::launch_kernel(stats_row_kernel, n, ST_THREADS, 0, st, logits, ld, vocab, tid, tlw, nt, stats));
  DUO_LAUNCH_CHECK("stats_row_kernel");
  DUO_CUDA_TRY(::duo::launch_kernel(stats_pair_kernel, n, ST_THREADS, 0, st, logits, ld, vocab, base, stats, d, ldd));
  DUO_LAUNCH_CHECK("stats_pair_kernel");
  return DUO_OK;
}

}  // namespace duo

using namespace duo;

extern "C" int duo_push_stats(const float* logits, int n, int vocab, const int32_t* base_row, const int32_t* targets,
                              const float* target_logw, int n_targets, float* stats, float* d, duo_stream stream) {
  DUO_CHECK_ARG(n >= 0 && vocab > 0 && n_targets >= 0, "push_stats: bad sizes");
  if (n == 0) return DUO_OK;
  DUO_CHECK_ARG(logits && base_row && stats && (n_targets == 0 || targets), "push_stats: null pointer");
  return launch_push_stats(logits, n, vocab, vocab, base_row, targets, target_logw, n_targets, stats, d, vocab,
                           as_stream(stream));
}
