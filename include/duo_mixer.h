/* duo_mixer.h -- C ABI of the B200 (sm_100a) token-mixing engine for Qwen3.5-shaped decoders.
 *
 * This is the drop-in boundary for the hot path of scasella/duo-mech-interp's engine: the Gated DeltaNet and gated
 * attention token mixers, the int8-dequant projections around them and the residual steering-vector add.  In the
 * reference those run as WGSL kernels behind `Model` (engine/model.js:26-509) and are dispatched through
 * `GPU.run(name, wgsl, bindings, workgroups, uniforms)` (engine/gpu.js:109-129).  Each entry point below names the
 * reference function or kernel it replaces.
 *
 * Conventions
 *   - Every call returns a duo status: DUO_OK (0) or a negative code.  No exception or abort crosses the ABI; the
 *     message of the last failure on the calling host thread is returned by duo_last_error().  (The reference
 *     throws JS exceptions on shape limits, model.js:52, 406, 418; gpu.js:127.)
 *   - Pointers named `*_host` are host memory; every other data pointer is device memory of the current CUDA device.
 *   - `duo_stream` is a cudaStream_t (NULL = legacy default stream).  Calls are stream-ordered and asynchronous
 *     unless documented otherwise.
 *   - dtype codes: DUO_F32, DUO_BF16 for activations; weights are int8 + f32 scales ("q8", engine/kernels.js:1-5).
 *   - An engine handle is not thread-safe; use one per stream / process.  Multi-GPU = one handle per process.
 */
#ifndef DUO_MIXER_H
#define DUO_MIXER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* duo_stream;
typedef struct duo_engine duo_engine;

enum duo_status_code {
  DUO_OK = 0,
  DUO_EINVAL = -1,  /* invalid argument or shape */
  DUO_ECUDA = -2,   /* a CUDA runtime / driver call or a kernel launch failed */
  DUO_ESTATE = -3,  /* call out of order (no weights, no state, row past its cache, ...) */
  DUO_ENOMEM = -4   /* device allocation failed */
};

enum duo_dtype { DUO_F32 = 0, DUO_BF16 = 1, DUO_F16 = 2, DUO_I8 = 3, DUO_I32 = 4 };
enum duo_push_mode { DUO_PUSH_ADD = 0, DUO_PUSH_MUL = 1 };
#define DUO_ALL_NEURONS (-1)

/* Message of the last failing call on this host thread ("" if none). */
const char* duo_last_error(void);
/* ABI version of this library (bumped on any signature change). */
int duo_abi_version(void);
/* Number of kernels this library has launched in this process (every entry point counts its launches). */
unsigned long long duo_launch_count(void);
/* Synchronise the current device and read-and-clear the fault word of the bounded-wait kernels (TMA / tcgen05 /
 * TMA-fed conv), its host-mapped mirror and the word set by duo_fault_raise: non-zero means a wait inside a kernel
 * gave up (the kernel unwound instead of hanging; codes 1, 2, 4, 8 tensor-core pipeline, 16 conv prologue).  While the
 * word is set, the tensor-core kernels launched without a cluster skip their work, and every duo_engine_forward /
 * _forward_device / _logits / _argmax / _generate (and each step of _generate) returns DUO_ECUDA before launching
 * anything once the fault is visible on the host (the last kernel of each forward mirrors it there).  Without a CUDA
 * device only the duo_fault_raise word exists.  The reference's analogue is its device-lost check, engine/gpu.js:38,
 * 151. */
int duo_fault_status(unsigned* out);
/* OR `code` into the host-side fault word that the engine calls check, exactly as a mirrored device fault would be
 * seen: exercises the engine's error path without any device fault.  duo_fault_status clears it. */
int duo_fault_raise(unsigned code);

/* ============================================================================================================
 * Op-level entry points (the per-kernel sweeps and the parity tests call these; the engine uses the same kernels)
 * ============================================================================================================ */

/* W[n, k] (f32 / bf16 / f16, row-major) -> q[n, k] int8 + s[n, k / group] f32.  scale = absmax / 127 (1 for an
 * all-zero group), q = round-half-even(v / scale) with IEEE division.  group = 128 is the reference format; group = k
 * gives one scale per output row.  Replaces the `quantize(src)` kernel, engine/kernels.js:16-47 (and its dispatch,
 * model.js:213-216).  Bit-exact contract. */
int duo_q8_quantize(const void* w, int w_dtype, int n, int k, int group, int8_t* q, float* s, duo_stream stream);

/* out[n, k] = f32(q) * scale, written as f32 or bf16 (kernels.js:7-11 unpack, :74-75 dequant). */
int duo_q8_dequantize(const int8_t* q, const float* s, int n, int k, int group, void* out, int out_dtype,
                      duo_stream stream);

/* y[m, n] (+)= x[m, k] . dequant(W)[n, k]^T for m <= 8, streaming the int8 weights once (decode).  x and y are f32 or
 * bf16; accumulate != 0 adds into y.  Replaces `matvec(M, add)`, engine/kernels.js:55-94 (dispatched by
 * model.js:382-392). */
int duo_q8_gemv(const void* x, int x_dtype, int m, int k, const int8_t* q, const float* s, int group, int n, void* y,
                int y_dtype, int accumulate, duo_stream stream);

/* y[t, :] = dequant(E)[ids[t], :] (f32).  Replaces `gather`, engine/kernels.js:205-221. */
int duo_q8_gather(const int32_t* ids, int t, const int8_t* q, const float* s, int group, int k, int vocab, float* y,
                  duo_stream stream);

/* Dense bf16 tensor-core GEMM (tcgen05, accumulators in TMEM):  C[m, n] (+)= (A[m, k] . B[n, k]^T) * col_scale[n].
 * A and B are row-major bf16 with k a multiple of 64; col_scale may be NULL; C is f32 or bf16 with leading dim ldc.
 * The prefill path of `matmul(add)`, engine/kernels.js:97-151, runs on this kernel. */
int duo_gemm_bf16(const void* a, int m, int k, const void* b, int n, const float* col_scale, void* c, int c_dtype,
                  int ldc, int accumulate, duo_stream stream);

/* Fused MLP up-projection: gu = (A[m, k] . B[2 inter, k]^T) * col_scale, then out[i, j] = silu(gate_j) * up_j with the
 * layer's neuron pushes applied in list order to row r = row_base + i / t (row i of A): entry p adds push_vals[p *
 * push_rows + r] to neuron push_neurons[p] (DUO_PUSH_ADD) or multiplies it in (DUO_PUSH_MUL); neuron -1 is every
 * neuron.  B holds gate and up rows interleaved in blocks of 64: B rows [128 b, 128 b + 64) are gate rows 64 b ..
 * 64 b + 63 and B rows [128 b + 64, 128 b + 128) the matching up rows (col_scale in the same order, may be NULL).
 * A and B are bf16 or f16 (ab_dtype); out has the same dtype, leading dim ldo.  k and inter multiples of 64; at most
 * 32 push records.
 * Replaces `_mm(xn, gu)` + `swiglu`, engine/model.js:448-457 and engine/kernels_qwen35.js:250-280. */
int duo_gemm_swiglu(const void* a, int m, int k, const void* b, int inter, int ab_dtype, const float* col_scale,
                    void* out, int ldo, const int32_t* push_neurons, const int32_t* push_modes, const float* push_vals,
                    int push_count, int push_rows, int t, int row_base, duo_stream stream);

/* y[m, n] (+)= x[m, k] . dequant(W)[n, k]^T for 1 <= m <= 256 rows on the tensor cores, streaming the int8 weights
 * q [n, k] (scales s [n, k / group]) and converting them on chip: x bf16 or f16; y f32 (accumulate != 0 adds into
 * it), bf16 or f16 with leading dim ldy.  group is a multiple of 64 that divides k (128: the reference format; k: one
 * scale per row).  The operand the tensor core sees is dequant(W) rounded to x's dtype (exact for one scale per row,
 * whose scale multiplies the f32 sum).  swiglu != 0: q holds [gate (n / 2 rows) | up (n / 2 rows)] and
 * y[m, n / 2] = silu(gate) * up in x's dtype.  The decode path of `matmul(add)` on the int8 format,
 * engine/kernels.js:97-151 (dispatched by model.js:382-392). */
int duo_q8_gemm(const void* x, int x_dtype, int m, int k, const int8_t* q, const float* s, int group, int n,
                int swiglu, void* y, int y_dtype, int ldy, int accumulate, duo_stream stream);

/* y[m, :] = x[m, :] * rsqrt(mean(x^2) + eps) * (1 + w) (offset != 0) or * w.  x f32, y f32 / bf16.
 * Replaces `rmsnorm(offset)`, engine/kernels.js:226-246. */
int duo_rmsnorm(const float* x, int m, int d, const float* w, float eps, int offset, void* y, int y_dtype,
                duo_stream stream);

/* The Gated DeltaNet prologue of a linear-attention layer over b rows x t tokens of its fused projection
 * y [b * t, w] (f32, bf16 or f16; w >= conv_dim + hv dv + 2 hv) = [q k v (conv_dim = 2 hk dk + hv dv) | z (hv dv) |
 * b (hv) | a (hv)]: causal depthwise conv (kernel 4, weights conv_w [conv_dim, 4] f32) over the conv_dim channels,
 * continuing from conv_state [b, 3, conv_dim] (f32, the last 3 inputs of earlier calls, oldest first; updated in
 * place), then SiLU and the l2norm (eps 1e-6) of every q and k head -> qkv [b * t, conv_dim] (same dtype as y);
 * beta = sigmoid(b), g = -exp(a_log) * softplus(a + dt_bias) -> beta, g [b * t, hv] f32.  dk = dv = 128.
 * Replaces `conv` + `convState` (engine/kernels_qwen35.js:129-178) and the gate and l2norm prep of `delta`
 * (kernels_qwen35.js:208-229).  16-bit projections whose rows are 16-byte aligned, called with at least 64 tokens
 * per row, take the TMA-fed kernel, the rest the register-staged one. */
int duo_gdn_conv_fwd(const void* y, int dtype, int w, const float* conv_w, float* conv_state, const float* a_log,
                     const float* dt_bias, void* qkv, float* g, float* beta, int b, int t, int hk, int hv, int dk,
                     int dv, duo_stream stream);

/* Gated DeltaNet scan computed token by token (the recurrent form; t = 1 is one decode step) over b rows x t tokens
 * x h heads:  q, k [b, t, h, dk], v [b, t, h, dv] (f32 or bf16, token-major), g (log decay), beta [b, t, h] f32,
 * state [b, h, dk, dv] f32 read as the initial state and overwritten with the final one, o [b, t, h, dv].
 * l2norm_qk != 0 l2-normalises q and k first (eps 1e-6); q is scaled by 1/sqrt(dk) inside.  dk = dv = 128.
 * Replaces the recurrence of `delta`, engine/kernels_qwen35.js:209-236. */
int duo_gdn_recurrent_fwd(const void* q, const void* k, const void* v, int in_dtype, const float* g,
                          const float* beta, float* state, void* o, int o_dtype, int b, int t, int h, int dk, int dv,
                          int l2norm_qk, duo_stream stream);

/* Same contract as duo_gdn_recurrent_fwd, computed in the chunked WY / UT form (chunk 64) on the tensor cores: bf16
 * operands, f32 accumulation, f32 state.  f32 inputs are rounded to bf16 on load.  This is the prefill form of the
 * reference's PyTorch path (transformers torch_chunk_gated_delta_rule); the reference's own WGSL engine runs prefill
 * token by token in `delta` (engine/kernels_qwen35.js:183-247). */
int duo_gdn_chunk_fwd(const void* q, const void* k, const void* v, int in_dtype, const float* g, const float* beta,
                      float* state, void* o, int o_dtype, int b, int t, int h, int dk, int dv, int l2norm_qk,
                      duo_stream stream);

/* Causal GQA softmax attention of b rows over their caches.  q [b, t, nh, hd] holds the t new queries of each row,
 * which sit at cache positions start[r] .. start[r] + t - 1; kc, vc [b, max_len, nkv, hd] hold keys / values
 * 0 .. start[r] + t - 1.  o[b, t, nh, hd] = softmax(q k^T * scale) v, times sigmoid(gate[b, t, nh, hd]) when gate is
 * not NULL (gate_stride = elements between consecutive tokens' gate rows).  q, kc, vc, gate, o share `dtype`.
 * Replaces `attention`, engine/kernels_qwen35.js:73-123. */
int duo_attention(const void* q, const void* kc, const void* vc, const int32_t* start, const void* gate,
                  int gate_stride, void* o, int dtype, int b, int t, int nh, int nkv, int hd, int max_len, float scale,
                  duo_stream stream);

/* duo_attention for callers that cannot allocate device memory (a serving stack whose pooled allocator owns all of
 * it, or a decode loop where cudaMalloc and the synchronisation it implies are not allowed).  No counterpart in the
 * reference.  Same arguments, kernels and split plan as duo_attention, but the split-K decode scratch is a fixed
 * file-scope device array of 262,144 floats (1 MiB, held on every GPU that loads the library) instead of a
 * library-allocated workspace: nothing is allocated.  A decode call (t == 1) needing more than that
 * (b * nh * splits * (hd + 2) floats) fails with DUO_EINVAL before any launch.  The first call on a device looks up
 * the array's address and should come before any stream capture.  Calls share the array: calls that overlap on the
 * GPU race (order them on one stream); nothing in it needs clearing between calls. */
int duo_attention_noalloc(const void* q, const void* kc, const void* vc, const int32_t* start, const void* gate,
                          int gate_stride, void* o, int dtype, int b, int t, int nh, int nkv, int hd, int max_len,
                          float scale, duo_stream stream);

/* Per (layer, neuron) of a capture cap [layers, t, inter] f32 over tokens t0 .. t - 1: out[(l * inter + n) * 4 + 0..3] =
 * max, its first token, min, its first token (token indices as f32; out 16-byte aligned).  Replaces `tokenExtremes`,
 * engine/kernels.js:288-306 (used on DUO_CAP_ACT captures, analysis.js:612-613). */
int duo_token_extremes(const float* cap, int layers, int t, int inter, int t0, float* out, duo_stream stream);

/* Next-token statistics of the push probe (engine/analysis.js:480-537; its PyTorch form tools/find_steering.py:86-103)
 * over logits [n, vocab] f32 (row-major, from duo_engine_logits).  With lp = logits - lse (log-softmax, analysis.js:
 * 693-702), row r gets stats[r * DUO_STATS_COLS + c]:
 *   DUO_STAT_LSE   lse = log sum_i exp(logits[r, i])
 *   DUO_STAT_MASS  mass = sum_j exp(lp[r, targets[j]])                      (probability on the target ids)
 *   DUO_STAT_TLSE  tlse = log sum_j exp(lp[r, targets[j]] + target_logw[j])  (target_logw may be NULL: zeros)
 * and, when base_row[r] >= 0 (the unsteered row of the same context; its own stats are read, not changed):
 *   DUO_STAT_KL    kl = sum over i with p_i > 1e-12 of p_i (lp[r, i] - lp[base, i])   (analysis.js:704-708)
 *   DUO_STAT_DP    mass[r] - mass[base];   DUO_STAT_GAIN  tlse[r] - tlse[base]
 *   d[r, i] += lp[r, i] - lp[base, i] over the vocabulary when d [n, vocab] is not NULL (analysis.js:523)
 * Rows with base_row[r] < 0 get kl = dp = gain = 0 and leave d alone.  base_row, targets, target_logw, stats and d
 * are device arrays.  Out-of-range target ids count as probability 0. */
enum duo_stat_col {
  DUO_STAT_LSE = 0, DUO_STAT_MASS, DUO_STAT_TLSE, DUO_STAT_KL, DUO_STAT_DP, DUO_STAT_GAIN, DUO_STATS_COLS
};
int duo_push_stats(const float* logits, int n, int vocab, const int32_t* base_row, const int32_t* targets,
                   const float* target_logw, int n_targets, float* stats, float* d, duo_stream stream);

/* ============================================================================================================
 * Engine: mirrors engine/model.js `Model` (alloc, reset, setVectors, setHeadScales, _forward, _logits, argmaxAll)
 * ============================================================================================================ */

typedef struct duo_config {
  int hidden, inter, vocab, layers;
  int nh, nkv, hd, rot;   /* full attention: q heads, kv heads, head dim, rotary dims (partial RoPE) */
  float theta, eps;
  int hk, hv, dk, dv, ks; /* linear attention: key heads, value heads, head dims, conv kernel */
  const uint8_t* full_attention_host; /* [layers], 1 = full attention layer, 0 = Gated DeltaNet (copied) */
  int group;              /* int8 group size along the input dim: 128 (reference), or 0 for one scale per row */
  int act_dtype;          /* DUO_F32 (the reference's f32 engine) or DUO_BF16 (tensor-core path) */
} duo_config;

typedef struct duo_q8_view { const int8_t* q; const float* s; } duo_q8_view;

/* One layer's weights in the reference's fused layouts (model.js:70-116).  Device pointers, owned by the caller. */
typedef struct duo_layer_view {
  const float* in_norm;   /* [hidden], applied as (1 + w) */
  const float* post_norm; /* [hidden] */
  duo_q8_view proj;       /* linear: [qkv | z | b | a] x hidden;  full: [q+gate | k | v] x hidden */
  duo_q8_view out;        /* hidden x (hv * dv) or hidden x (nh * hd) */
  duo_q8_view gu;         /* [gate | up] (2 * inter) x hidden */
  duo_q8_view down;       /* hidden x inter */
  const float* conv;      /* linear: [conv_dim, ks] */
  const float* a_log;     /* linear: [hv] */
  const float* dt_bias;   /* linear: [hv] */
  const float* gnorm;     /* linear: [dv] gated-norm weight (not offset) */
  const float* q_norm;    /* full: [hd] */
  const float* k_norm;    /* full: [hd] */
} duo_layer_view;

typedef struct duo_weights_view {
  duo_q8_view embed;      /* vocab x hidden, tied with the LM head */
  const float* final_norm;
  const duo_layer_view* layers_host; /* [layers] host array of views (copied) */
} duo_weights_view;

/* new Model(cfg) (model.js:27-58). */
int duo_engine_create(const duo_config* cfg, duo_engine** out);
void duo_engine_destroy(duo_engine* e);
/* Model weights (model.js:142-151, 282-302).  Pointers are kept, not copied: the caller keeps them alive.  With
 * act_dtype = DUO_BF16 the engine also builds its own bf16 copy of every projection for the tensor-core GEMM. */
int duo_engine_load(duo_engine* e, const duo_weights_view* w, duo_stream stream);
/* alloc(rows, maxLen, maxT) (model.js:308-342); max_tokens bounds rows * T of one forward call. */
int duo_engine_alloc(duo_engine* e, int rows, int max_len, int max_tokens);
/* reset(r) (model.js:352-360): zero row r's recurrent and conv state and its length. */
int duo_engine_reset(duo_engine* e, int row, duo_stream stream);
/* reset(r) for every row at once. */
int duo_engine_reset_all(duo_engine* e, duo_stream stream);
/* The capture hooks of model.js:7-12, 445-461 (`resid: true`, `resid: "attn"`, `capture` with capLayers / capT /
 * capT0).  For every later forward of M = rows * T token rows (row-major: row_base's T tokens first), the i-th listed
 * layer writes its M rows to out[(i * cap_t + t0 + m) * width], f32, then t0 advances by M (as prefill's chunks
 * advance capT0, model.js:486-491); t0 starts at 0 and duo_engine_set_capture_t0 sets it.  Kinds:
 *   DUO_CAP_RESID       residual stream after the layer's MLP and vector add (width hidden; `resid: true`)
 *   DUO_CAP_RESID_ATTN  residual stream after the layer's mixer out-projection (width hidden; `resid: "attn"`)
 *   DUO_CAP_ACT         down_proj input silu(gate) * up after the pushes (width inter; `capture`)
 * layers_host NULL lists layers 0 .. n_layers - 1; n_layers = 0 turns the kind off.  A forward that would write past
 * cap_t rows fails with DUO_EINVAL before launching anything.  `out` is device memory the caller keeps alive. */
enum duo_capture_kind { DUO_CAP_RESID = 0, DUO_CAP_RESID_ATTN = 1, DUO_CAP_ACT = 2, DUO_CAP_KINDS = 3 };
int duo_engine_set_capture(duo_engine* e, int kind, int n_layers, const int32_t* layers_host, float* out, int cap_t);
int duo_engine_set_capture_t0(duo_engine* e, int kind, int t0);
/* Every later forward runs layers 0 .. layer only (model.js `stopAfter`, 427); -1 runs them all.  Row lengths and
 * last hidden states advance as for a full forward (model.js:463-465). */
int duo_engine_set_stop_after(duo_engine* e, int layer);
/* Shorthand for one DUO_CAP_RESID layer whose rows always start at row 0 of out[rows * T, hidden]; layer = -1 turns
 * it off. */
int duo_engine_capture_resid(duo_engine* e, int layer, float* out);
/* setVectors(rows) (model.js:372-376): vecs_host [n_rows, hidden]; rows >= n_rows get zero vectors.  Synchronises
 * `stream` before returning (vecs_host may be freed then). */
int duo_engine_set_vectors(duo_engine* e, const float* vecs_host, int n_rows, duo_stream stream);
/* setHeadScales (model.js:362-369) for one linear-attention layer; NULL restores all ones. */
int duo_engine_set_head_scales(duo_engine* e, int layer, const float* scales_host, duo_stream stream);
/* Neuron pushes of one layer at the down_proj input (model.js:412-424, kernels_qwen35.js:254-279): n records, each
 * (neuron or DUO_ALL_NEURONS, DUO_PUSH_ADD / DUO_PUSH_MUL, one value per engine row: vals_host[n, rows]).  Records
 * apply in order; n = 0 clears the layer.  They stay in force for every later forward until changed. */
int duo_engine_set_pushes(duo_engine* e, int layer, int n, const int32_t* neurons_host, const int32_t* modes_host,
                          const float* vals_host, duo_stream stream);
/* _forward(ids, rowBase, rows, T, {vec}) (model.js:404-466): ids_host [rows * T] token-major; vec_layer = -1 for
 * none.  The ids are copied into engine-owned pinned memory during the call and from there to the device on
 * `stream` (a few slots in turn; the call waits only if the copy that last used its slot has not run yet), so the
 * caller may reuse ids_host as soon as the call returns.  Leaves each row's final hidden state in the engine. */
int duo_engine_forward(duo_engine* e, const int32_t* ids_host, int row_base, int rows, int t, int vec_layer,
                       duo_stream stream);
/* Same with device-resident ids (no host traffic; capturable in a CUDA graph). */
int duo_engine_forward_device(duo_engine* e, const int32_t* ids, int row_base, int rows, int t, int vec_layer,
                              duo_stream stream);
/* _logits(n, r0) (model.js:472-477): final norm + tied LM head for rows r0..r0+n-1 -> out[n, vocab] f32 (device). */
int duo_engine_logits(duo_engine* e, int row0, int n, float* out, duo_stream stream);
/* argmaxAll (model.js:494-500) for rows r0..r0+n-1 -> out[n] int32 (device); ties go to the lower index. */
int duo_engine_argmax(duo_engine* e, int row0, int n, int32_t* out, duo_stream stream);
/* Greedy decode of every row for n_steps (the reference's loop of argmaxAll + step, analysis.js:127-142), entirely on
 * the device: tokens_out [rows, n_steps] int32 (device).  The first token is the argmax of the current state. */
int duo_engine_generate(duo_engine* e, int n_steps, int vec_layer, int32_t* tokens_out, duo_stream stream);
/* Tokens held so far by row r (this.len[r] in model.js), or a negative status. */
int duo_engine_row_len(duo_engine* e, int row);

/* Live per-kernel-class timing with CUDA events on the launching stream (the reference only times whole steps,
 * tests/profile.html:19-45).  mask = OR of (1 << DUO_PROF_*) classes to time, 0 = off.  Reading synchronises the
 * device, writes the summed milliseconds and launch counts per class (arrays of DUO_PROF_KINDS) and clears them. */
enum duo_prof_kind {
  DUO_PROF_GATHER = 0, DUO_PROF_RMSNORM, DUO_PROF_GEMV, DUO_PROF_GEMM, DUO_PROF_GDN_CONV, DUO_PROF_GDN_SCAN,
  DUO_PROF_ATTN_PREP, DUO_PROF_ATTN, DUO_PROF_SWIGLU, DUO_PROF_OTHER, DUO_PROF_KINDS
};
int duo_engine_profile(duo_engine* e, unsigned mask);
int duo_engine_profile_read(duo_engine* e, double* ms_out, long long* launches_out);

#ifdef __cplusplus
}
#endif
#endif /* DUO_MIXER_H */
