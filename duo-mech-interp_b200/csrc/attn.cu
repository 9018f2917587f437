// Gated GQA softmax attention with a per-row KV cache.
//
// Reference: engine/kernels_qwen35.js:14-123 (`attnPrep`, `attention`) and, for the arithmetic of its PyTorch path,
// transformers' Qwen3_5Attention (q/k RMSNorm with (1 + w), partial rotate-half RoPE on the first `rot` dims with
// inv_freq = theta^(-2j/rot), softmax(q k^T / sqrt(hd)) v with repeat_kv, output times sigmoid(gate)).
#include <algorithm>
#include <mutex>
#include <type_traits>

#include "kernels.cuh"

namespace duo {

// ---------------------------------------------------------------------------------------------------------------
// prep: block per token, warp per head of q ∪ kv (head dim 256: 8 consecutive dims per lane, 16-byte accesses).  The
// token's RoPE angles are computed once per block; RMSNorm by a warp butterfly; the rotate-half partner of dim i
// (i +- rot / 2) sits rot / 16 lanes away and comes by shuffle.

template <typename T>
__global__ void __launch_bounds__(1024) attn_prep_kernel(AttnPrepArgs a) {
  pdl_enter();
  extern __shared__ float trig[];  // [rot / 2] cos, then [rot / 2] sin
  const int m = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int HD = 256;
  const int rr = m / a.t, R = a.row_base + rr;
  const int pos = a.len[R] + m % a.t;
  const int half = a.rot / 2;
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    float sn, cs;
    sincosf((float)pos * a.inv_freq[j], &sn, &cs);
    trig[j] = cs;
    trig[half + j] = sn;
  }
  __syncthreads();
  const int hh = warp;
  const bool isq = hh < a.nh;
  const T* y = static_cast<const T*>(a.y);
  const long src = isq ? (long)m * a.w + (long)hh * 2 * HD : (long)m * a.w + (long)a.nh * 2 * HD + (long)(hh - a.nh) * HD;
  const int d0 = lane * 8;
  float v[8];
  load8(y + src + d0, v);
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 8; e++) ss += v[e] * v[e];
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)HD + a.eps);
  const float* nw = (isq ? a.q_norm : a.k_norm) + d0;
  float xn[8], out[8];
#pragma unroll
  for (int e = 0; e < 8; e++) xn[e] = v[e] * r * (1.f + nw[e]);
  // rotate-half RoPE on dims [0, rot): lanes [0, rot / 8); partner lane = lane -+ half / 8
  const int hl = half / 8;
  const int rl = a.rot / 8;
  const int partner = lane < hl ? lane + hl : (lane < rl ? lane - hl : lane);
#pragma unroll
  for (int e = 0; e < 8; e++) {
    const float p = __shfl_sync(0xffffffffu, xn[e], partner);
    const int i = d0 + e;
    if (i < a.rot) {
      const int j = i < half ? i : i - half;
      const float cs = trig[j], sn = trig[half + j];
      out[e] = i < half ? xn[e] * cs - p * sn : xn[e] * cs + p * sn;
    } else {
      out[e] = xn[e];
    }
  }
  if (isq) {
    store8(static_cast<T*>(a.q_out) + ((long)m * a.nh + hh) * HD + d0, out);
  } else {
    const int kvh = hh - a.nh;
    const long at = (((long)R * a.max_len + pos) * a.nkv + kvh) * HD + d0;
    store8(static_cast<T*>(a.kc) + at, out);
    float vv[8];
    load8(y + (long)m * a.w + (long)a.nh * 2 * HD + (long)a.nkv * HD + (long)kvh * HD + d0, vv);
    store8(static_cast<T*>(a.vc) + at, vv);
  }
}

int launch_attn_prep(const AttnPrepArgs& a, int dtype, cudaStream_t st) {
  const int m = a.rows * a.t;
  if (m == 0) return DUO_OK;
  if (a.hd != 256 || a.rot > a.hd || a.rot % 16 || a.nh + a.nkv > 32)
    return fail(DUO_EINVAL, "attn_prep: needs head dim 256, rot a multiple of 16, at most 32 heads");
  if (a.w % 8) return fail(DUO_EINVAL, "attn_prep: projection width must be a multiple of 8");
  const int threads = 32 * (a.nh + a.nkv);
  const size_t sm = (size_t)a.rot * sizeof(float);
  return with_act(dtype, [&](auto tag) -> int {
    DUO_CUDA_TRY(::duo::launch_kernel(attn_prep_kernel<decltype(tag)>, dim3(m), threads, sm, st, a));
    DUO_LAUNCH_CHECK("attn_prep_kernel");
    return DUO_OK;
  });
}

// ---------------------------------------------------------------------------------------------------------------
// prefill (t > 1): flash-style online softmax on CUDA cores.  Block = (32-query tile, q head, row); 256 threads.
// Thread (qi = tid / 8, g = tid % 8) computes scores for query qi against keys g*4 .. g*4+3 of each 32-key tile and
// owns output dims g + 8x of query qi.

constexpr int AP_BQ = 32, AP_BK = 32, AP_HD = 256;

__device__ __forceinline__ int q_start(const AttnArgs& a, int b) {
  const int R = a.cache_row0 + b;
  return a.start ? a.start[R] : a.len[R] - a.t;
}

template <typename T>
__global__ void __launch_bounds__(256) attn_prefill_kernel(AttnArgs a) {
  pdl_enter();
  extern __shared__ float sm[];
  float* Qs = sm;                            // [BQ][HD + 1]
  float* Ks = Qs + AP_BQ * (AP_HD + 1);      // [BK][HD + 1]
  float* Vs = Ks + AP_BK * (AP_HD + 1);      // [BK][HD]
  float* Ps = Vs + AP_BK * AP_HD;            // [BQ][BK + 1]
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, qi = tid >> 3, g = tid & 7;
  const int rep = a.nh / a.nkv, kvh = h / rep;
  const int R = a.cache_row0 + b;
  const int p0 = q_start(a, b);
  const int tq0 = qt * AP_BQ;
  const int nq = min(AP_BQ, a.t - tq0);
  const T* q = static_cast<const T*>(a.q);
  const T* kc = static_cast<const T*>(a.kc);
  const T* vc = static_cast<const T*>(a.vc);
  for (int e = tid; e < AP_BQ * AP_HD; e += 256) {
    const int r = e / AP_HD, d = e % AP_HD;
    Qs[r * (AP_HD + 1) + d] = r < nq ? to_f(q[(((long)b * a.t + tq0 + r) * a.nh + h) * AP_HD + d]) * a.scale : 0.f;
  }
  const int my_pos = p0 + tq0 + qi;  // position of this thread's query
  const int n_keys = p0 + tq0 + nq;  // keys 0 .. n_keys-1 are needed by the tile
  float mrow = -INFINITY, lrow = 0.f;
  float o[32];
#pragma unroll
  for (int x = 0; x < 32; x++) o[x] = 0.f;
  for (int k0 = 0; k0 < n_keys; k0 += AP_BK) {
    __syncthreads();
    for (int e = tid; e < AP_BK * AP_HD; e += 256) {
      const int r = e / AP_HD, d = e % AP_HD;
      const int key = k0 + r;
      float kv = 0.f, vv = 0.f;
      if (key < n_keys) {
        const long at = (((long)R * a.max_len + key) * a.nkv + kvh) * AP_HD + d;
        kv = to_f(kc[at]);
        vv = to_f(vc[at]);
      }
      Ks[r * (AP_HD + 1) + d] = kv;
      Vs[r * AP_HD + d] = vv;
    }
    __syncthreads();
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    const float* qrow = Qs + qi * (AP_HD + 1);
    const float* k0p = Ks + (g * 4) * (AP_HD + 1);
#pragma unroll 4
    for (int d = 0; d < AP_HD; d++) {
      const float qv = qrow[d];
#pragma unroll
      for (int x = 0; x < 4; x++) s[x] = fmaf(qv, k0p[x * (AP_HD + 1) + d], s[x]);
    }
    float tmax = -INFINITY;
#pragma unroll
    for (int x = 0; x < 4; x++) {
      const int key = k0 + g * 4 + x;
      if (key > my_pos || key >= n_keys) s[x] = -INFINITY;
      tmax = fmaxf(tmax, s[x]);
    }
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
    const float mnew = fmaxf(mrow, tmax);
    const float alpha = mnew == -INFINITY ? 1.f : expf(mrow - mnew);
    float psum = 0.f;
#pragma unroll
    for (int x = 0; x < 4; x++) {
      const float p = s[x] == -INFINITY ? 0.f : expf(s[x] - mnew);
      Ps[qi * (AP_BK + 1) + g * 4 + x] = p;
      psum += p;
    }
    psum += __shfl_xor_sync(0xffffffffu, psum, 1);
    psum += __shfl_xor_sync(0xffffffffu, psum, 2);
    psum += __shfl_xor_sync(0xffffffffu, psum, 4);
    lrow = lrow * alpha + psum;
    mrow = mnew;
    __syncwarp();
#pragma unroll
    for (int x = 0; x < 32; x++) o[x] *= alpha;
    const float* prow = Ps + qi * (AP_BK + 1);
#pragma unroll 4
    for (int kk = 0; kk < AP_BK; kk++) {
      const float p = prow[kk];
      const float* vr = Vs + kk * AP_HD + g;
#pragma unroll
      for (int x = 0; x < 32; x++) o[x] = fmaf(p, vr[8 * x], o[x]);
    }
  }
  if (qi < nq) {
    const long tok = (long)b * a.t + tq0 + qi;
    const float inv = 1.f / lrow;
    T* op = static_cast<T*>(a.o) + (tok * a.nh + h) * AP_HD;
    const T* gp = a.gate ? static_cast<const T*>(a.gate) + tok * a.gate_stride + (long)h * a.gate_hstride : nullptr;
#pragma unroll
    for (int x = 0; x < 32; x++) {
      const int d = g + 8 * x;
      float v = o[x] * inv;
      if (gp) v *= sigmoidf_(to_f(gp[d]));
      op[d] = from_f<T>(v);
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// decode (t == 1): block = (row, kv head, key split); the `rep` q heads of the kv head share every K / V load.
// 8 warps; warp w takes keys w, w + 8, ... of the split; lane l holds dims 8l .. 8l+7 of q, of each key and of the
// output accumulators for all rep heads.  Partials (m, l, o) of the warps merge in shared memory; with several
// splits they go to `work` and a combine kernel applies the softmax merge and the gate.

constexpr int AD_REP = 4, AD_WARPS = 8;

template <typename T>
__device__ __forceinline__ void ld8f(const T* p, float* o) { load8(p, o); }

template <typename T>
__global__ void __launch_bounds__(256) attn_decode_kernel(AttnArgs a, int nsplit, int split_len) {
  pdl_enter();
  __shared__ float sm_m[AD_WARPS][AD_REP], sm_l[AD_WARPS][AD_REP];
  __shared__ float sm_o[AD_WARPS][AD_REP][AP_HD];
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rep = a.nh / a.nkv;
  const int R = a.cache_row0 + b;
  const int p0 = q_start(a, b);
  const int n_keys = p0 + 1;
  const int kbeg = split * split_len, kend = min(n_keys, kbeg + split_len);
  const T* qp = static_cast<const T*>(a.q);
  const T* kc = static_cast<const T*>(a.kc);
  const T* vc = static_cast<const T*>(a.vc);
  float q[AD_REP][8], o[AD_REP][8], mh[AD_REP], lh[AD_REP];
#pragma unroll
  for (int r = 0; r < AD_REP; r++) {
    if (r < rep) {
      ld8f(qp + ((long)b * a.nh + kvh * rep + r) * AP_HD + lane * 8, q[r]);
#pragma unroll
      for (int x = 0; x < 8; x++) q[r][x] *= a.scale;
    }
#pragma unroll
    for (int x = 0; x < 8; x++) o[r][x] = 0.f;
    mh[r] = -INFINITY;
    lh[r] = 0.f;
  }
  for (int key = kbeg + warp; key < kend; key += AD_WARPS) {
    const long at = (((long)R * a.max_len + key) * a.nkv + kvh) * AP_HD + lane * 8;
    float kv[8], vv[8];
    ld8f(kc + at, kv);
    ld8f(vc + at, vv);
#pragma unroll
    for (int r = 0; r < AD_REP; r++) {
      if (r >= rep) continue;
      float s = 0.f;
#pragma unroll
      for (int x = 0; x < 8; x++) s = fmaf(q[r][x], kv[x], s);
      s = warp_sum(s);
      const float mnew = fmaxf(mh[r], s);
      const float alpha = expf(mh[r] - mnew);
      const float p = expf(s - mnew);
      lh[r] = lh[r] * alpha + p;
      mh[r] = mnew;
#pragma unroll
      for (int x = 0; x < 8; x++) o[r][x] = fmaf(o[r][x], alpha, p * vv[x]);
    }
  }
#pragma unroll
  for (int r = 0; r < AD_REP; r++) {
    if (lane == 0) { sm_m[warp][r] = mh[r]; sm_l[warp][r] = lh[r]; }
#pragma unroll
    for (int x = 0; x < 8; x++) sm_o[warp][r][lane * 8 + x] = o[r][x];
  }
  __syncthreads();
  // merge the warps: thread handles (head r, dim d) pairs
  for (int e = threadIdx.x; e < rep * AP_HD; e += blockDim.x) {
    const int r = e / AP_HD, d = e % AP_HD;
    float M = -INFINITY;
    for (int w = 0; w < AD_WARPS; w++) M = fmaxf(M, sm_m[w][r]);
    float L = 0.f, O = 0.f;
    for (int w = 0; w < AD_WARPS; w++) {
      const float f = sm_m[w][r] == -INFINITY ? 0.f : expf(sm_m[w][r] - M);
      L += sm_l[w][r] * f;
      O += sm_o[w][r][d] * f;
    }
    const int h = kvh * rep + r;
    if (nsplit == 1) {
      float v = O / L;
      if (a.gate) v *= sigmoidf_(to_f(static_cast<const T*>(a.gate)[(long)b * a.gate_stride + (long)h * a.gate_hstride + d]));
      static_cast<T*>(a.o)[((long)b * a.nh + h) * AP_HD + d] = from_f<T>(v);
    } else {
      float* wp = a.work + (((long)b * a.nh + h) * nsplit + split) * (AP_HD + 2);
      wp[2 + d] = O;
      if (d == 0) { wp[0] = M; wp[1] = L; }
    }
  }
}

template <typename T>
__global__ void attn_combine_kernel(AttnArgs a, int nsplit) {
  pdl_enter();
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const float* wp = a.work + ((long)b * a.nh + h) * nsplit * (AP_HD + 2);
  float M = -INFINITY;
  for (int s = 0; s < nsplit; s++) M = fmaxf(M, wp[s * (AP_HD + 2)]);
  float L = 0.f, O = 0.f;
  for (int s = 0; s < nsplit; s++) {
    const float* p = wp + s * (AP_HD + 2);
    const float f = p[0] == -INFINITY ? 0.f : expf(p[0] - M);
    L += p[1] * f;
    O += p[2 + d] * f;
  }
  float v = O / L;
  if (a.gate) v *= sigmoidf_(to_f(static_cast<const T*>(a.gate)[(long)b * a.gate_stride + (long)h * a.gate_hstride + d]));
  static_cast<T*>(a.o)[((long)b * a.nh + h) * AP_HD + d] = from_f<T>(v);
}

// split-K plan for decode: enough blocks to cover the SMs twice, splits of at least 256 keys
static void decode_plan(const AttnArgs& a, int* nsplit, int* split_len) {
  const long blocks = (long)a.b * a.nkv;
  int ns = (int)std::max<long>(1, (2L * sm_count() + blocks - 1) / blocks);
  ns = std::min(ns, std::max(1, cdiv(a.max_len, 256)));
  if (!a.work) ns = 1;
  while (ns > 1 && (long)a.b * a.nh * ns * (AP_HD + 2) > a.work_floats) ns--;
  *nsplit = ns;
  *split_len = cdiv(a.max_len, ns);
}

long attn_decode_scratch_floats(int b, int nh, int nkv, int max_len, int dtype) {
  int ns;
  if (dtype != DUO_F32) {
    ns = attn_decode_mma_plan(b, nkv, max_len, nullptr);
  } else {
    const long blocks = (long)std::max(1, b) * nkv;
    ns = (int)std::max<long>(1, (2L * sm_count() + blocks - 1) / blocks);
    ns = std::min(ns, std::max(1, cdiv(max_len, 256)));
  }
  return ns > 1 ? (long)b * nh * ns * (AP_HD + 2) : 0;
}

int launch_attn_combine(const AttnArgs& a, int dtype, int nsplit, cudaStream_t st) {
  return with_act(dtype, [&](auto tag) -> int {
    DUO_CUDA_TRY(::duo::launch_kernel(attn_combine_kernel<decltype(tag)>, dim3(a.nh, a.b), AP_HD, 0, st, a, nsplit));
    DUO_LAUNCH_CHECK("attn_combine_kernel");
    return DUO_OK;
  });
}

long attn_work_floats(int b, int nh, int max_len) {
  const int ns_max = std::max(1, cdiv(max_len, 256));
  return (long)b * nh * std::min<long>(ns_max, 2L * sm_count()) * (AP_HD + 2);
}

// DUO_ATTN_TC=0 keeps 16-bit prefill on the mma.sync kernel (for comparisons); the default is the tcgen05 kernel
static bool attn_tc_enabled() {
  static const bool on = [] {
    const char* v = getenv("DUO_ATTN_TC");
    return !(v && v[0] == '0');
  }();
  return on;
}

template <typename T>
static int run_attention(const AttnArgs& a, cudaStream_t st) {
  if (!std::is_same<T, float>::value && a.t > 1) {
    const int rep = a.nh / a.nkv;
    const int dt = std::is_same<T, __half>::value ? DUO_F16 : DUO_BF16;
    if (attn_tc_enabled() && attn_prefill_tc_eligible(a, dt)) return launch_attn_prefill_tc(a, dt, st);  // tcgen05
    if (rep == 1 || rep == 2 || rep == 4) return launch_attn_prefill_mma(a, dt, st);  // mma.sync
  }
  if (!std::is_same<T, float>::value && a.t == 1)  // HBM-streaming tensor-core decode
    return launch_attn_decode_mma(a, std::is_same<T, __half>::value ? DUO_F16 : DUO_BF16, st);
  if (a.t == 1) {
    int ns, sl;
    decode_plan(a, &ns, &sl);
    DUO_CUDA_TRY(::duo::launch_kernel(attn_decode_kernel<T>, dim3(ns, a.nkv, a.b), 256, 0, st, a, ns, sl));
    DUO_LAUNCH_CHECK("attn_decode_kernel");
    if (ns > 1) {
      DUO_CUDA_TRY(::duo::launch_kernel(attn_combine_kernel<T>, dim3(a.nh, a.b), AP_HD, 0, st, a, ns));
      DUO_LAUNCH_CHECK("attn_combine_kernel");
    }
    return DUO_OK;
  }
  constexpr size_t smem = sizeof(float) * (AP_BQ * (AP_HD + 1) + AP_BK * (AP_HD + 1) + AP_BK * AP_HD + AP_BQ * (AP_BK + 1));
  DUO_TRY(ensure_smem_attr(attn_prefill_kernel<T>, (int)smem));
  DUO_CUDA_TRY(::duo::launch_kernel(attn_prefill_kernel<T>, dim3(cdiv(a.t, AP_BQ), a.nh, a.b), 256, smem, st, a));
  DUO_LAUNCH_CHECK("attn_prefill_kernel");
  return DUO_OK;
}

int launch_attention(const AttnArgs& a, int dtype, cudaStream_t st) {
  if (a.b == 0 || a.t == 0) return DUO_OK;
  if (a.hd != AP_HD) return fail(DUO_EINVAL, "attention: head dim must be 256");
  if (a.nkv <= 0 || a.nh % a.nkv || a.nh / a.nkv > AD_REP) return fail(DUO_EINVAL, "attention: nh / nkv must be 1..4");
  return with_act(dtype, [&](auto tag) -> int { return run_attention<decltype(tag)>(a, st); });
}

// library-owned split-K workspace for the op-level entry point (grown on demand)
static float* g_op_work = nullptr;
static long g_op_work_floats = 0;
static std::mutex g_op_work_mu;

}  // namespace duo

using namespace duo;

extern "C" int duo_attention(const void* q, const void* kc, const void* vc, const int32_t* start, const void* gate,
                             int gate_stride, void* o, int dtype, int b, int t, int nh, int nkv, int hd, int max_len,
                             float scale, duo_stream stream) {
  DUO_CHECK_ARG(b >= 0 && t >= 0 && nh > 0 && nkv > 0 && max_len > 0, "attention: bad shape");
  DUO_CHECK_ARG(valid_act(dtype), "attention: dtype must be f32, bf16 or f16");
  DUO_CHECK_ARG(b == 0 || t == 0 || (q && kc && vc && start && o), "attention: null pointer");
  AttnArgs a{};
  a.q = q; a.kc = kc; a.vc = vc; a.cache_row0 = 0; a.start = start; a.len = nullptr;
  a.gate = gate; a.gate_stride = gate_stride; a.gate_hstride = hd; a.o = o;
  a.b = b; a.t = t; a.nh = nh; a.nkv = nkv; a.hd = hd; a.max_len = max_len; a.scale = scale;
  if (t == 1) {
    std::lock_guard<std::mutex> lock(g_op_work_mu);
    const long need = attn_work_floats(b, nh, max_len);
    if (need > g_op_work_floats) {
      if (g_op_work) cudaFree(g_op_work);
      g_op_work = nullptr;
      g_op_work_floats = 0;
      if (cudaMalloc(&g_op_work, need * sizeof(float)) != cudaSuccess) return fail(DUO_ENOMEM, "attention: workspace");
      g_op_work_floats = need;
    }
    a.work = g_op_work;
    a.work_floats = g_op_work_floats;
    return launch_attention(a, dtype, as_stream(stream));
  }
  return launch_attention(a, dtype, as_stream(stream));
}
