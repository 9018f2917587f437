// Host-side launchers shared between the kernel files and the engine.  All are stream-ordered and return a duo
// status; none allocates memory.
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace duo {

// Push records of one layer (device arrays): neuron (DUO_ALL_NEURONS for all), mode (DUO_PUSH_ADD / MUL) and one
// value per engine row, vals[i * rows + r].
struct PushTable {
  const int32_t* neuron;
  const int32_t* mode;
  const float* vals;
  int count;
  int rows;
};

// Neuron pushes of the SwiGLU epilogue (the reference's push list, engine/model.js:8, 410-425): every entry whose neuron is n
// (or DUO_ALL_NEURONS) adds its per-row value to, or multiplies it into, activation n of row r, in list order.
__device__ __forceinline__ float push_apply(const PushTable& pt, int r, int n, float v) {
  for (int i = 0; i < pt.count; i++) {
    const int pn = pt.neuron[i];
    if (pn == DUO_ALL_NEURONS || pn == n) {
      const float val = pt.vals[(long)i * pt.rows + r];
      v = pt.mode[i] == DUO_PUSH_MUL ? v * val : v + val;
    }
  }
  return v;
}
// The entries that can touch columns [n, n + w) (bit i: entry i; the table holds at most 32): computed once for a
// thread's columns, so the per-element loop visits only them (usually none) instead of the whole table.
__device__ __forceinline__ unsigned push_mask(const PushTable& pt, int n, int w) {
  unsigned mask = 0u;
  for (int i = 0; i < pt.count; i++) {
    const int pn = pt.neuron[i];
    if (pn == DUO_ALL_NEURONS || (pn >= n && pn < n + w)) mask |= 1u << i;
  }
  return mask;
}
// push_apply over the entries of `mask` (a push_mask covering n), in list order
__device__ __forceinline__ float push_apply_masked(const PushTable& pt, unsigned mask, int r, int n, float v) {
  while (mask) {
    const int i = __ffs(mask) - 1;
    mask &= mask - 1u;
    const int pn = pt.neuron[i];
    if (pn == DUO_ALL_NEURONS || pn == n) {
      const float val = pt.vals[(long)i * pt.rows + r];
      v = pt.mode[i] == DUO_PUSH_MUL ? v * val : v + val;
    }
  }
  return v;
}

// Epilogues of the tensor-core GEMM.
enum GemmEpi {
  EPI_STORE = 0,   // C[m, n] = acc * colscale[n]                   (bf16 or f32 C)
  EPI_ADD_F32 = 1, // X[m, n] += acc * colscale[n] (+ vec[row(m), n])  (f32 residual stream)
  EPI_SWIGLU = 2,  // gate/up interleaved per 64 columns: A[m, j] = silu(g) * u, then pushes   (16-bit A)
  EPI_ARGMAX = 3   // per (row, 256-column tile): max of acc * colscale and its lowest column -> c / idx [m, ldc]
};

struct GemmEpiArgs {
  int epi = EPI_STORE;
  void* c = nullptr;            // output (STORE: C; ADD: X f32; SWIGLU: A)
  int c_dtype = DUO_BF16;
  int ldc = 0;                  // leading dim of the output in elements
  const float* colscale = nullptr;
  const float* vec = nullptr;   // ADD: optional per-row vector table [rows_total, n]
  int t = 1, row_base = 0;      // row(m) = row_base + m / t
  PushTable push{};             // SWIGLU
  int32_t* idx = nullptr;       // ARGMAX: column of each partial maximum (c holds the f32 maxima)
  bool b_const = false;         // B is not written by the kernel launched just before (weight packs): its first
                                // tiles may be fetched before the programmatic-launch wait
  // RMSNorm fused across two tensor-core GEMMs (decode GEMM: blocks of 128 columns, n a multiple of 128; m > 256:
  // the persistent kernel's 256-wide tiles, n a multiple of 256).  The residual add also writes the next norm's input
  // scaled by its weight, nrm_out[m, n] = x_new[m, n] * (1 + nrm_w[n]) in the operand dtype (row stride ldc), and
  // the sum of x_new^2 over each block of columns to nrm_part[m * (n / block) + block index];
  // the consuming GEMM multiplies the accumulator of activation row m by
  // rsqrt(sum_b row_part[m * row_blocks + b] / row_d + row_eps), summed in block order (deterministic).
  const float* nrm_w = nullptr;
  void* nrm_out = nullptr;
  float* nrm_part = nullptr;
  const float* row_part = nullptr;
  int row_blocks = 0, row_d = 0;
  float row_eps = 0.f;
  // SwiGLU on int8 weights in their own order [gate | up] (launch_gemm_dec_q8, inter = cs_inter): colscale holds one
  // entry per int8 row, not per interleaved row
  int cs_inter = 0;
};

// decode-sized tcgen05 GEMM (m <= 256 rows; weights on the MMA's M side, grid = weight blocks x row groups x K
// slices, K split over a cluster where the SMs need it): y = x . w^T
int launch_gemm_dec(const void* x, int m, int k, const void* w, int n, int ab_dtype, const GemmEpiArgs& ep,
                    cudaStream_t st);
// the same kernel reading the int8 weights wq [n, k] (scales ws [n, k / group]; group a multiple of 64 dividing k,
// = k for one scale per row, which the caller passes as ep.colscale) and converting them on chip; inter > 0: SwiGLU
// with wq = [gate (inter rows) | up (inter rows)], n = 2 inter
int launch_gemm_dec_q8(const void* x, int m, int k, const int8_t* wq, const float* ws, int group, int inter, int n,
                       int ab_dtype, const GemmEpiArgs& ep, cudaStream_t st);

// persistent tcgen05 GEMM over prepared tensor maps (A box 128 x 64, B box bn x 64; bn = 256)
int launch_gemm_persist(const CUtensorMap& ta, const CUtensorMap& tb, int bn, int m, int n, int k, int ab_dtype,
                        const GemmEpiArgs& ep, cudaStream_t st);

// Greedy next tokens straight from the LM head: out[i] = argmax_n (A[i, :] . B[n, :]) * colscale[n] (lowest n on
// ties; the values are those the f32 logits would hold), through the persistent GEMM's ARGMAX epilogue and a per-row
// reduction of its partials.  scratch: m * ceil(n / 256) * 2 words.
int launch_lm_argmax(const void* a, int m, int k, const void* b, int n, int ab_dtype, const float* colscale,
                     bool b_const, float* scratch, int32_t* out, cudaStream_t st);

int launch_gemv(const void* x, int x_dtype, int m, int k, const int8_t* q, const float* s, int group, int n, void* y,
                int y_dtype, int accumulate, cudaStream_t st);
int launch_gather(const int32_t* ids, int t, const int8_t* q, const float* s, int group, int k, int vocab, float* y,
                  cudaStream_t st);
int launch_dequant(const int8_t* q, const float* s, int n, int k, int group, void* out, int out_dtype,
                   cudaStream_t st);

// 16-bit tensor-core GEMM (A and B both bf16 or both f16, ab_dtype): acc[m, n] = A[m, k] . B[n, k]^T, then the
// epilogue
int launch_gemm_tc(const void* a, int m, int k, const void* b, int n, int ab_dtype, const GemmEpiArgs& ep,
                   cudaStream_t st);
// f32 CUDA-core GEMM on int8 weights (the f32 engine): acc = A[m, k] . dequant(W)[n, k]^T, then the epilogue
int launch_gemm_f32_q8(const float* a, int m, int k, const int8_t* q, const float* s, int group, int n,
                       const GemmEpiArgs& ep, cudaStream_t st);

int launch_rmsnorm(const float* x, int m, int d, const float* w, float eps, int offset, void* y, int y_dtype,
                   cudaStream_t st);
int launch_swiglu_push(const void* gu, int m, int inter, int t, int row_base, const PushTable& pt, void* a, int dtype,
                       cudaStream_t st);
int launch_vec_add(float* x, int m, int h, int t, int row_base, const float* vec, cudaStream_t st);
int launch_argmax(const float* logits, int m, int v, int32_t* out, cudaStream_t st);
// 16-bit (bf16 / f16) -> f32 copy of n values (n a multiple of 8)
int launch_to_f32(const void* src, int dtype, long n, float* dst, cudaStream_t st);
// push-probe statistics (stats.cu): stats [n, DUO_STATS_COLS]; d [n, ldd] accumulated when not null
int launch_push_stats(const float* logits, int n, int vocab, long ld, const int32_t* base, const int32_t* tid,
                      const float* tlw, int nt, float* stats, float* d, long ldd, cudaStream_t st);
int launch_finish_rows(const float* x, int h, int t, int row_base, int rows, float* last, int32_t* len,
                       cudaStream_t st);
// the greedy tokens am[rows] -> the next forward's ids and column `step` of log[rows][n_steps] (step_ctr != nullptr:
// the step index is read from, and advanced in, that device counter)
int launch_feed_tokens(const int32_t* am, int rows, int32_t* ids, int32_t* log, int n_steps, int step,
                       int32_t* step_ctr, cudaStream_t st);

// ---- Gated DeltaNet
struct GdnConvArgs {
  const void* y;          // fused projection [M, w] = [qkv (conv_dim) | z (vd) | b (hv) | a (hv)]
  int w;                  // its row width
  const float* conv_w;    // [conv_dim, ks]
  float* conv_state;      // [rows_total, ks - 1, conv_dim]
  const float* a_log;
  const float* dt_bias;
  void* qkv_out;          // [M, conv_dim]: l2-normalised q, k (q not yet scaled) and v
  float* g_out;           // [M, hv]
  float* beta_out;        // [M, hv]
  int hk, hv, dk, dv, ks;
  int rows, t, row_base;
};
int launch_gdn_conv(const GdnConvArgs& a, int dtype, cudaStream_t st);

struct GdnScanArgs {
  const void* q; const void* k; const void* v;
  long q_stride, k_stride, v_stride;  // elements between consecutive tokens
  const float* g; const float* beta;  // [M, h]
  float* state;                       // [b_total, h, dk, dv]; this call uses rows state_row0 ..
  int state_row0;
  void* o; long o_stride;
  int b, t, hq, h, dk, dv;            // hq = heads of q/k (h / hq value heads share one q/k head)
  int l2norm_qk;
  // optional fused gated RMSNorm + head scale (the engine path): o = o * rms * w * silu(z) * hs[h]
  const void* z; long z_stride;
  const float* norm_w; const float* head_scale; float eps;
  // chunked scan only: workspace of gdn_chunk_ws_bytes(b, t, h) bytes (per chunk T diag(beta), A and W in f16)
  void* chunk_ws; long chunk_ws_bytes;
};
long gdn_chunk_ws_bytes(int b, int t, int h);
int launch_gdn_recurrent(const GdnScanArgs& a, int dtype, cudaStream_t st);
// short prefill of the 16-bit engines (2 <= t <= 16): token by token with the state held in registers per item
int launch_gdn_short(const GdnScanArgs& a, int dtype, cudaStream_t st);
// decode step (t = 1): conv + gates + l2norm + delta rule + gated norm in one kernel (needs hk == hv)
int launch_gdn_decode(const GdnConvArgs& ca, const GdnScanArgs& a, int dtype, cudaStream_t st);
int launch_gdn_chunk(const GdnScanArgs& a, int dtype, cudaStream_t st);
// the tcgen05 form (gdn_chunk_tc.cu) for 16-bit inputs without the l2norm option; launch_gdn_chunk routes to it
bool gdn_chunk_tc_eligible(const GdnScanArgs& a, int dtype);
int launch_gdn_chunk_tc(const GdnScanArgs& a, int dtype, cudaStream_t st);

// ---- gated attention
struct AttnPrepArgs {
  const void* y;              // fused projection [M, w] = [q+gate (nh * 2hd) | k | v]
  int w;
  const float* q_norm; const float* k_norm;
  const float* inv_freq;      // [rot / 2]
  const int32_t* len;         // per engine row: tokens already in the cache
  void* q_out;                // [M, nh, hd]
  void* kc; void* vc;         // [rows_total, max_len, nkv, hd]
  int nh, nkv, hd, rot, max_len, rows, t, row_base;
  float eps;
};
int launch_attn_prep(const AttnPrepArgs& a, int dtype, cudaStream_t st);

struct AttnArgs {
  const void* q;              // [b, t, nh, hd]
  const void* kc; const void* vc;  // [b_total, max_len, nkv, hd], rows cache_row0 ..
  int cache_row0;
  const int32_t* start;       // per cache row: position of this call's first query (NULL: from len - t)
  const int32_t* len;         // alternative: per cache row tokens held after the prep (start = len - t)
  const void* gate; long gate_stride;  // optional sigmoid gate: head h of token tok at gate + tok * gate_stride
  long gate_hstride;                   //   + h * gate_hstride

  void* o;                    // [b, t, nh, hd]
  int b, t, nh, nkv, hd, max_len;
  float scale;
  float* work;                // split-K scratch for decode (may be NULL: no split)
  long work_floats;
};
int launch_attention(const AttnArgs& a, int dtype, cudaStream_t st);
long attn_work_floats(int b, int nh, int max_len);
// split-K scratch (floats) the decode planner of `dtype` fills when the workspace does not limit it; 0 = no split
long attn_decode_scratch_floats(int b, int nh, int nkv, int max_len, int dtype);
// 16-bit decode (t == 1) on the tensor cores, its split plan (splits; *split_len keys per split) and the combine
int launch_attn_decode_mma(const AttnArgs& a, int dtype, cudaStream_t st);
int attn_decode_mma_plan(int b, int nkv, int max_len, int* split_len);
int launch_attn_combine(const AttnArgs& a, int dtype, int nsplit, cudaStream_t st);
int launch_attn_prefill_mma(const AttnArgs& a, int dtype, cudaStream_t st);  // bf16 / f16, t > 1, hd 256
// bf16 / f16, t > 1, hd 256, nh / nkv in {1, 2, 4}, 16-byte aligned operands: tcgen05 + TMA flash attention
bool attn_prefill_tc_eligible(const AttnArgs& a, int dtype);
int launch_attn_prefill_tc(const AttnArgs& a, int dtype, cudaStream_t st);

// int8 -> 16-bit (bf16 or f16) copy of a weight matrix for the tensor-core GEMM: dst row of src row n is n, or
// (interleave > 0) the gate/up interleaved order [gate 64 | up 64]* with `interleave` = rows of each half.
// apply_scale = 0 writes the int8 values exactly (the per-row scale then goes to the GEMM's column scale).
int launch_pack16(const int8_t* q, const float* s, int n, int k, int group, int interleave, int apply_scale,
                  int out_dtype, void* out, float* colscale_out, cudaStream_t st);

GdnScanArgs op_scan_args(const void* q, const void* k, const void* v, const float* g, const float* beta,
                         float* state, void* o, int b, int t, int h, int l2norm_qk);

}  // namespace duo
