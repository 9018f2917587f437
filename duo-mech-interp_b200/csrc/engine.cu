// The engine: per-row state, weights and the layer-by-layer forward of a Qwen3.5 hybrid decoder, mirroring the
// reference's engine/model.js `Model` (alloc, reset, setVectors, setHeadScales, _forward, _logits, argmaxAll, step).
//
// Activation layout is token-major [M = rows * T, width] as in the reference (kernels_qwen35.js:5-6).  The residual
// stream is f32; GEMM inputs, projections, caches and mixer outputs use the engine's activation dtype (f32 = the
// reference's precision, bf16 = the tensor-core path).  The Gated DeltaNet state and the conv state are f32 always.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "kernels.cuh"
#include "tc.cuh"

using namespace duo;

namespace {

constexpr int kMaxPush = 16;  // push records per layer (the reference allows 8, model.js:415)
constexpr int kStage = 3;     // pinned staging slots for host token ids (duo_engine_forward)
constexpr int kGemvMax = 8;   // rows up to which projections stream int8 weights through the GEMV

struct Pack {
  void* w = nullptr;  // 16-bit (the engine's activation dtype) copy of the int8 matrix
  float* colscale = nullptr;  // per output column when the int8 scale is per row, else null
};

struct LayerState {
  float* conv = nullptr;  // [rows, ks-1, conv_dim]
  float* S = nullptr;     // [rows, hv, dk, dv]
  void* kc = nullptr;     // [rows, max_len, nkv, hd]
  void* vc = nullptr;
  float* head_scale = nullptr;  // [hv]
  int32_t* push_neuron = nullptr;
  int32_t* push_mode = nullptr;
  float* push_vals = nullptr;   // [kMaxPush, rows]
  int push_count = 0;
};

}  // namespace

struct duo_engine {
  duo_config cfg{};
  std::vector<uint8_t> full;
  int kd = 0, vd = 0, conv_dim = 0, w_lin = 0, w_full = 0, wmax = 0, group = 0;
  int act = DUO_F32;
  size_t act_size = 4;
  // weights
  bool loaded = false;
  duo_weights_view w{};
  std::vector<duo_layer_view> lw;
  std::vector<Pack> p_proj, p_out, p_gu, p_down;
  Pack p_embed;
  std::vector<void*> owned;  // device allocations of this engine
  float* inv_freq = nullptr;
  // state
  int rows = 0, max_len = 0, max_tokens = 0;
  float* x = nullptr;
  void* xn = nullptr;
  float* nrm_part[2] = {nullptr, nullptr};  // fused-norm row partials: [rows][hidden / 128 (decode) or / 256]
  void* y = nullptr;
  void* qkv = nullptr;
  float* g = nullptr;
  float* beta = nullptr;
  void* o = nullptr;
  void* q = nullptr;
  void* a = nullptr;
  float* last = nullptr;
  void* xn_last = nullptr;
  float* logits = nullptr;
  int32_t* amax = nullptr;
  int32_t* ids = nullptr;
  int32_t* len_dev = nullptr;
  int32_t* step_ctr = nullptr;
  float* vec = nullptr;
  float* attn_work = nullptr;
  long attn_work_floats_n = 0;
  void* chunk_ws = nullptr;  // chunked DeltaNet scan workspace (16-bit engines)
  long chunk_ws_bytes = 0;
  std::vector<int> len;
  std::vector<LayerState> ls;
  std::vector<void*> state_owned;
  // host token ids are copied into one of kStage pinned slots and from there to the device; a slot is reused only
  // after the copy that last read it has run (its event), so the caller's array is free when the call returns
  int32_t* ids_stage = nullptr;
  cudaEvent_t stage_ev[kStage] = {};
  int stage_next = 0;
  // capture hooks (model.js:7-12, 445-461): per kind, the slot of each layer in `out` (-1: not captured); a forward
  // of M token rows writes its rows to out[(slot * cap_t + t0 + m) * width] (f32) and then advances t0 by M when
  // `advance` (prefill chunks, model.js:486-491)
  struct Capture {
    std::vector<int> slot;
    float* out = nullptr;
    long cap_t = 0, t0 = 0;
    bool advance = true;
    bool on() const { return out != nullptr; }
  } cap[DUO_CAP_KINDS];
  int stop_after = -1;  // last layer a forward runs (-1: all; model.js `stopAfter`)
  // live profiling: per kind, a pool of (start, stop) event pairs recorded around launches on the stream
  unsigned prof_mask = 0;
  struct ProfKind {
    std::vector<cudaEvent_t> ev;  // 2 per recorded launch
    size_t used = 0;
  } prof[DUO_PROF_KINDS];

  ~duo_engine() {
    free_state();
    for (void* p : owned) cudaFree(p);
    for (auto& k : prof)
      for (cudaEvent_t ev : k.ev) cudaEventDestroy(ev);
  }
  // index of a started span, or -1 when this kind is not profiled
  long prof_begin(int kind, cudaStream_t st) {
    if (!(prof_mask & (1u << kind))) return -1;
    ProfKind& k = prof[kind];
    if (k.used + 2 > k.ev.size()) {
      for (int i = 0; i < 256; i++) {
        cudaEvent_t ev;
        if (cudaEventCreate(&ev) != cudaSuccess) return -1;
        k.ev.push_back(ev);
      }
    }
    const long i = (long)k.used;
    k.used += 2;
    cudaEventRecord(k.ev[i], st);
    return i;
  }
  void prof_end(int kind, long i, cudaStream_t st) {
    if (i >= 0) cudaEventRecord(prof[kind].ev[i + 1], st);
  }
  void free_state() {
    for (cudaEvent_t& ev : stage_ev)
      if (ev) {
        cudaEventSynchronize(ev);
        cudaEventDestroy(ev);
        ev = nullptr;
      }
    if (ids_stage) cudaFreeHost(ids_stage);
    ids_stage = nullptr;
    for (void* p : state_owned) cudaFree(p);
    state_owned.clear();
    ls.clear();
    rows = 0;
  }
  int dalloc(void** p, size_t bytes, bool state) {
    if (bytes == 0) bytes = 16;
    if (cudaMalloc(p, bytes) != cudaSuccess) {
      cudaGetLastError();
      return fail(DUO_ENOMEM, "device allocation of " + std::to_string(bytes) + " bytes failed");
    }
    (state ? state_owned : owned).push_back(*p);
    return DUO_OK;
  }
  bool is_full(int l) const { return full[l] != 0; }
  int gsize(int k) const { return group > 0 ? group : k; }
};

namespace {

// DUO_TRY with the launch timed under profiling class `kind`
#define PROF_TRY(kind, expr)                  \
  do {                                        \
    const long _pi = e->prof_begin(kind, st); \
    const int _ps = (expr);                   \
    e->prof_end(kind, _pi, st);               \
    if (_ps != DUO_OK) return _ps;            \
  } while (0)

int check_engine(duo_engine* e, bool need_weights, bool need_state) {
  DUO_CHECK_ARG(e, "null engine");
  if (need_weights && !e->loaded) return fail(DUO_ESTATE, "engine: weights not loaded");
  if (need_state && e->rows == 0) return fail(DUO_ESTATE, "engine: state not allocated (call duo_engine_alloc)");
  return DUO_OK;
}

// Decode projections on the int8 weights converted on chip (DUO_DEC_Q8=1) instead of the 16-bit pack.  Off by
// default: at 256 rows the conversion sits in the MMA's critical path and the pack is faster (8224 x 1024:
// 12.3 us on the pack, 14.8 us converting; 32 rows: 8.1 against 9.1 us).
bool dec_q8_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("DUO_DEC_Q8");
    return v && v[0] == '1';
  }();
  return on;
}

// y[m, n] (+)= x[m, k] . W^T through the GEMV (m <= 8, int8 weights), the f32 GEMM (f32 engine), the decode GEMM
// streaming the int8 weights (m <= 256) or the tensor-core GEMM on the 16-bit pack.
int project(duo_engine* e, const void* xin, int m, int k, const duo_q8_view& wq, const Pack& pk, int n,
            const GemmEpiArgs& ep, cudaStream_t st) {
  const int grp = e->gsize(k);
  if (m <= kGemvMax) {
    if (ep.epi == EPI_STORE) return launch_gemv(xin, e->act, m, k, wq.q, wq.s, grp, n, ep.c, ep.c_dtype, 0, st);
    // residual add into the f32 stream, then the optional vector
    DUO_TRY(launch_gemv(xin, e->act, m, k, wq.q, wq.s, grp, n, ep.c, DUO_F32, 1, st));
    if (ep.vec) DUO_TRY(launch_vec_add(static_cast<float*>(ep.c), m, n, ep.t, ep.row_base, ep.vec, st));
    return DUO_OK;
  }
  if (e->act == DUO_F32) return launch_gemm_f32_q8(static_cast<const float*>(xin), m, k, wq.q, wq.s, grp, n, ep, st);
  if (m <= 256 && dec_q8_enabled()) {
    GemmEpiArgs ep2 = ep;
    ep2.colscale = grp == k ? wq.s : nullptr;  // one scale per row: the epilogue's column scale
    ep2.b_const = true;
    return launch_gemm_dec_q8(xin, m, k, wq.q, wq.s, grp, 0, n, e->act, ep2, st);
  }
  GemmEpiArgs ep2 = ep;
  ep2.colscale = pk.colscale;
  ep2.b_const = true;  // packed once at creation, before any forward
  return launch_gemm_tc(xin, m, k, pk.w, n, e->act, ep2, st);
}

int build_pack(duo_engine* e, const duo_q8_view& v, int n, int k, int interleave, Pack* out, cudaStream_t st) {
  void* w = nullptr;
  DUO_TRY(e->dalloc(&w, (size_t)n * k * 2, false));
  out->w = w;
  const bool per_row = e->group == 0;
  if (per_row) {
    void* cs = nullptr;
    DUO_TRY(e->dalloc(&cs, (size_t)n * 4, false));
    out->colscale = static_cast<float*>(cs);
  }
  return launch_pack16(v.q, v.s, n, k, e->gsize(k), interleave, per_row ? 0 : 1, e->act, out->w, out->colscale, st);
}

// rows [0, M) of src (dtype, row width `width`) -> the capture of `kind` for layer l, as f32
int capture_rows(duo_engine* e, int kind, int l, const void* src, int dtype, int M, int width, cudaStream_t st) {
  const duo_engine::Capture& k = e->cap[kind];
  if (!k.on() || k.slot[l] < 0) return DUO_OK;
  float* dst = k.out + ((long)k.slot[l] * k.cap_t + k.t0) * width;
  if (dtype == DUO_F32) {
    DUO_CUDA_TRY(cudaMemcpyAsync(dst, src, (size_t)M * width * 4, cudaMemcpyDeviceToDevice, st));
    return DUO_OK;
  }
  PROF_TRY(DUO_PROF_OTHER, launch_to_f32(src, dtype, (long)M * width, dst, st));
  return DUO_OK;
}

bool fused_norm_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("DUO_FUSED_NORM");
    return !(v && v[0] == '0');
  }();
  return on;
}

// the residual-add epilogue also writes the next RMSNorm's weighted input (xn) and its row partials
void set_norm_out(GemmEpiArgs& ep, const float* w, void* xn, float* part) {
  ep.nrm_w = w;
  ep.nrm_out = xn;
  ep.nrm_part = part;
}

// the GEMM consumes xn written by set_norm_out: its accumulator rows are scaled by rsqrt(mean x^2 + eps); the
// producer wrote one partial per 128 columns (decode GEMM, m <= 256) or per 256 (persistent GEMM)
void set_row_norm(GemmEpiArgs& ep, const float* part, int m, int d, float eps) {
  ep.row_part = part;
  ep.row_blocks = d / (m <= 256 ? 128 : 256);
  ep.row_d = d;
  ep.row_eps = eps;
}

int forward_impl(duo_engine* e, const int32_t* ids_dev, int row_base, int rows, int T, int vec_layer,
                 cudaStream_t st) {
  const duo_config& c = e->cfg;
  const int M = rows * T;
  const int H = c.hidden;
  const int act = e->act;
  // RMSNorm fused into the tensor-core GEMMs (bf16, M > 8 rows): the residual-add epilogue writes the next norm's
  // weighted input and per-block sums of squares; the consuming GEMM scales its accumulator rows by the rsqrt.  The
  // norm before layer 0's input projection stays a launch.  f16 keeps the launch: the weighted input before the
  // rsqrt could leave the f16 range.
  const bool fuse_norm = act == DUO_BF16 && M > kGemvMax && H % 256 == 0 && fused_norm_enabled();
  PROF_TRY(DUO_PROF_GATHER, launch_gather(ids_dev, M, e->w.embed.q, e->w.embed.s, e->gsize(H), H, c.vocab, e->x, st));
  for (int l = 0; l < c.layers; l++) {
    const duo_layer_view& L = e->lw[l];
    LayerState& S = e->ls[l];
    const bool full = e->is_full(l);
    const int wproj = full ? e->w_full : e->w_lin;
    const bool in_fused = fuse_norm && l > 0;  // the previous layer's down projection wrote xn and the partials
    if (!in_fused) PROF_TRY(DUO_PROF_RMSNORM, launch_rmsnorm(e->x, M, H, L.in_norm, c.eps, 1, e->xn, act, st));
    const void* xin = e->xn;
    {
      GemmEpiArgs ep;
      ep.epi = EPI_STORE;
      ep.c = e->y;
      ep.c_dtype = act;
      ep.ldc = wproj;
      if (in_fused) set_row_norm(ep, e->nrm_part[1], M, H, c.eps);
      PROF_TRY(M <= kGemvMax ? DUO_PROF_GEMV : DUO_PROF_GEMM, project(e, xin, M, H, L.proj, e->p_proj[l], wproj, ep, st));
    }
    int out_k;
    if (!full) {
      GdnConvArgs ca{};
      ca.y = e->y; ca.w = wproj; ca.conv_w = L.conv; ca.conv_state = S.conv; ca.a_log = L.a_log;
      ca.dt_bias = L.dt_bias; ca.qkv_out = e->qkv; ca.g_out = e->g; ca.beta_out = e->beta;
      ca.hk = c.hk; ca.hv = c.hv; ca.dk = c.dk; ca.dv = c.dv; ca.ks = c.ks;
      ca.rows = rows; ca.t = T; ca.row_base = row_base;
      GdnScanArgs sa{};
      const size_t es = e->act_size;
      sa.q = e->qkv;
      sa.k = static_cast<const char*>(e->qkv) + (size_t)e->kd * es;
      sa.v = static_cast<const char*>(e->qkv) + (size_t)2 * e->kd * es;
      sa.q_stride = sa.k_stride = sa.v_stride = e->conv_dim;
      sa.g = e->g; sa.beta = e->beta; sa.state = S.S; sa.state_row0 = row_base;
      sa.o = e->o; sa.o_stride = e->vd;
      sa.b = rows; sa.t = T; sa.hq = c.hk; sa.h = c.hv; sa.dk = c.dk; sa.dv = c.dv;
      sa.l2norm_qk = 0;  // the conv prologue already normalised q and k
      sa.z = static_cast<const char*>(e->y) + (size_t)e->conv_dim * es;
      sa.z_stride = wproj;
      sa.norm_w = L.gnorm; sa.head_scale = S.head_scale; sa.eps = c.eps;
      sa.chunk_ws = e->chunk_ws; sa.chunk_ws_bytes = e->chunk_ws_bytes;
      if (T == 1 && c.hk == c.hv) {
        // decode: one fused kernel from the projection to the gated norm
        PROF_TRY(DUO_PROF_GDN_SCAN, launch_gdn_decode(ca, sa, act, st));
      } else {
        PROF_TRY(DUO_PROF_GDN_CONV, launch_gdn_conv(ca, act, st));
        // prefill of the 16-bit engines: launch_gdn_chunk (up to 16 tokens per row token by token in registers,
        // longer calls the chunked tensor-core scan); the f32 engine: the recurrent form
        if (act != DUO_F32 && T > 1) PROF_TRY(DUO_PROF_GDN_SCAN, launch_gdn_chunk(sa, act, st));
        else PROF_TRY(DUO_PROF_GDN_SCAN, launch_gdn_recurrent(sa, act, st));
      }
      out_k = e->vd;
    } else {
      AttnPrepArgs pa{};
      pa.y = e->y; pa.w = wproj; pa.q_norm = L.q_norm; pa.k_norm = L.k_norm; pa.inv_freq = e->inv_freq;
      pa.len = e->len_dev; pa.q_out = e->q; pa.kc = S.kc; pa.vc = S.vc;
      pa.nh = c.nh; pa.nkv = c.nkv; pa.hd = c.hd; pa.rot = c.rot; pa.max_len = e->max_len;
      pa.rows = rows; pa.t = T; pa.row_base = row_base; pa.eps = c.eps;
      PROF_TRY(DUO_PROF_ATTN_PREP, launch_attn_prep(pa, act, st));
      AttnArgs aa{};
      aa.q = e->q; aa.kc = S.kc; aa.vc = S.vc;
      aa.cache_row0 = row_base;
      aa.start = e->len_dev;  // lengths advance after the last layer: they are this call's start positions
      aa.gate = static_cast<const char*>(e->y) + (size_t)c.hd * e->act_size;
      aa.gate_stride = wproj;
      aa.gate_hstride = 2L * c.hd;
      aa.o = e->o;
      aa.b = rows; aa.t = T; aa.nh = c.nh; aa.nkv = c.nkv; aa.hd = c.hd; aa.max_len = e->max_len;
      aa.scale = 1.f / std::sqrt((float)c.hd);
      aa.work = e->attn_work; aa.work_floats = e->attn_work_floats_n;
      PROF_TRY(DUO_PROF_ATTN, launch_attention(aa, act, st));
      out_k = c.nh * c.hd;
    }
    {
      GemmEpiArgs ep;
      ep.epi = EPI_ADD_F32;
      ep.c = e->x;
      ep.c_dtype = DUO_F32;
      ep.ldc = H;
      if (fuse_norm) set_norm_out(ep, L.post_norm, e->xn, e->nrm_part[0]);
      PROF_TRY(M <= kGemvMax ? DUO_PROF_GEMV : DUO_PROF_GEMM, project(e, e->o, M, out_k, L.out, e->p_out[l], H, ep, st));
    }
    DUO_TRY(capture_rows(e, DUO_CAP_RESID_ATTN, l, e->x, DUO_F32, M, H, st));
    if (!fuse_norm) PROF_TRY(DUO_PROF_RMSNORM, launch_rmsnorm(e->x, M, H, L.post_norm, c.eps, 1, e->xn, act, st));
    PushTable pt{S.push_neuron, S.push_mode, S.push_vals, S.push_count, e->rows};
    if (M > kGemvMax && act != DUO_F32) {
      GemmEpiArgs ep;
      ep.epi = EPI_SWIGLU;
      ep.c = e->a;
      ep.c_dtype = act;
      ep.ldc = c.inter;
      ep.colscale = e->p_gu[l].colscale;
      ep.t = T;
      ep.row_base = row_base;
      ep.push = pt;
      ep.b_const = true;  // weight packs are written once, at creation
      if (fuse_norm) set_row_norm(ep, e->nrm_part[0], M, H, c.eps);
      if (M <= 256 && dec_q8_enabled()) {
        // int8 gate / up rows in their own order: the kernel reads them through the pack's interleave
        const int grp = e->gsize(H);
        ep.colscale = grp == H ? L.gu.s : nullptr;
        ep.cs_inter = c.inter;
        PROF_TRY(DUO_PROF_GEMM, launch_gemm_dec_q8(e->xn, M, H, L.gu.q, L.gu.s, grp, c.inter, 2 * c.inter, act, ep, st));
      } else {
        PROF_TRY(DUO_PROF_GEMM, launch_gemm_tc(e->xn, M, H, e->p_gu[l].w, 2 * c.inter, act, ep, st));
      }
    } else {
      GemmEpiArgs ep;
      ep.epi = EPI_STORE;
      ep.c = e->y;
      ep.c_dtype = act;
      ep.ldc = 2 * c.inter;
      PROF_TRY(M <= kGemvMax ? DUO_PROF_GEMV : DUO_PROF_GEMM, project(e, e->xn, M, H, L.gu, Pack{}, 2 * c.inter, ep, st));
      PROF_TRY(DUO_PROF_SWIGLU, launch_swiglu_push(e->y, M, c.inter, T, row_base, pt, e->a, act, st));
    }
    DUO_TRY(capture_rows(e, DUO_CAP_ACT, l, e->a, act, M, c.inter, st));
    {
      GemmEpiArgs ep;
      ep.epi = EPI_ADD_F32;
      ep.c = e->x;
      ep.c_dtype = DUO_F32;
      ep.ldc = H;
      ep.vec = (vec_layer == l) ? e->vec : nullptr;
      ep.t = T;
      ep.row_base = row_base;
      if (fuse_norm && l + 1 < c.layers && l != e->stop_after) set_norm_out(ep, e->lw[l + 1].in_norm, e->xn, e->nrm_part[1]);
      PROF_TRY(M <= kGemvMax ? DUO_PROF_GEMV : DUO_PROF_GEMM, project(e, e->a, M, c.inter, L.down, e->p_down[l], H, ep, st));
    }
    DUO_TRY(capture_rows(e, DUO_CAP_RESID, l, e->x, DUO_F32, M, H, st));
    if (l == e->stop_after) break;
  }
  PROF_TRY(DUO_PROF_OTHER, launch_finish_rows(e->x, H, T, row_base, rows, e->last, e->len_dev, st));
  for (auto& k : e->cap)
    if (k.on() && k.advance) k.t0 += M;
  return DUO_OK;
}

int logits_impl(duo_engine* e, int row0, int n, float* out, cudaStream_t st) {
  const duo_config& c = e->cfg;
  const int H = c.hidden;
  PROF_TRY(DUO_PROF_RMSNORM, launch_rmsnorm(e->last + (size_t)row0 * H, n, H, e->w.final_norm, c.eps, 1, e->xn_last, e->act, st));
  GemmEpiArgs ep;
  ep.epi = EPI_STORE;
  ep.c = out;
  ep.c_dtype = DUO_F32;
  ep.ldc = c.vocab;
  PROF_TRY(n <= kGemvMax ? DUO_PROF_GEMV : DUO_PROF_GEMM, project(e, e->xn_last, n, H, e->w.embed, e->p_embed, c.vocab, ep, st));
  return DUO_OK;
}

// Greedy tokens of rows row0 .. row0 + n - 1.  On the tensor-core engine the LM head runs with the argmax epilogue
// (the same f32 values the logits would hold, lowest index on ties, no logits written); otherwise logits + argmax.
int greedy_impl(duo_engine* e, int row0, int n, int32_t* out, cudaStream_t st) {
  const duo_config& c = e->cfg;
  if (e->act == DUO_F32 || n <= kGemvMax) {
    DUO_TRY(logits_impl(e, row0, n, e->logits, st));
    PROF_TRY(DUO_PROF_OTHER, launch_argmax(e->logits, n, c.vocab, out, st));
    return DUO_OK;
  }
  const int H = c.hidden;
  PROF_TRY(DUO_PROF_RMSNORM, launch_rmsnorm(e->last + (size_t)row0 * H, n, H, e->w.final_norm, c.eps, 1, e->xn_last, e->act, st));
  PROF_TRY(DUO_PROF_GEMM, launch_lm_argmax(e->xn_last, n, H, e->p_embed.w, c.vocab, e->act, e->p_embed.colscale,
                                           true, e->logits, out, st));
  return DUO_OK;
}

int check_rows(duo_engine* e, int row_base, int rows, int T) {
  DUO_CHECK_ARG(rows >= 1 && T >= 1, "forward: rows and T must be >= 1");
  DUO_CHECK_ARG(row_base >= 0 && row_base + rows <= e->rows, "forward: rows out of range");
  if ((long)rows * T > e->max_tokens)
    return fail(DUO_EINVAL, "forward: rows * T = " + std::to_string((long)rows * T) + " exceeds max_tokens " +
                                std::to_string(e->max_tokens));
  for (int r = row_base; r < row_base + rows; r++)
    if (e->len[r] + T > e->max_len)
      return fail(DUO_ESTATE, "forward: row " + std::to_string(r) + " would exceed max_len " + std::to_string(e->max_len));
  for (const auto& k : e->cap)
    if (k.on() && k.t0 + (long)rows * T > k.cap_t)
      return fail(DUO_EINVAL, "forward: the capture holds " + std::to_string(k.cap_t) + " token rows per layer; this "
                              "call would write rows " + std::to_string(k.t0) + " .. " + std::to_string(k.t0 + (long)rows * T - 1));
  return DUO_OK;
}

}  // namespace

// =================================================================================================================

extern "C" int duo_engine_create(const duo_config* cfg, duo_engine** out) {
  DUO_CHECK_ARG(cfg && out, "engine_create: null pointer");
  const duo_config& c = *cfg;
  DUO_CHECK_ARG(c.hidden > 0 && c.inter > 0 && c.vocab > 0 && c.layers > 0, "engine_create: bad sizes");
  DUO_CHECK_ARG(c.hidden % 128 == 0 && c.inter % 128 == 0, "engine_create: hidden and inter must be multiples of 128");
  DUO_CHECK_ARG(c.dk == 128 && c.dv == 128 && c.ks == 4, "engine_create: linear attention needs dk = dv = 128, ks = 4");
  DUO_CHECK_ARG(c.hd == 256 && c.nkv > 0 && c.nh % c.nkv == 0 && c.nh / c.nkv <= 4,
                "engine_create: full attention needs hd = 256 and nh / nkv in 1..4");
  DUO_CHECK_ARG(c.rot > 0 && c.rot <= c.hd && c.rot % 2 == 0, "engine_create: bad rotary dims");
  DUO_CHECK_ARG(c.hk > 0 && c.hv % c.hk == 0, "engine_create: hv must be a multiple of hk");
  DUO_CHECK_ARG(c.group == 0 || (c.group % 16 == 0 && c.hidden % c.group == 0 && c.inter % c.group == 0),
                "engine_create: group must be 0 or a multiple of 16 dividing hidden and inter");
  DUO_CHECK_ARG(valid_act(c.act_dtype), "engine_create: act_dtype must be DUO_F32, DUO_BF16 or DUO_F16");
  DUO_CHECK_ARG(c.full_attention_host, "engine_create: null layer type array");
  {
    const int fs = fault_mirror_init();  // the host-mapped fault word the forward's last kernel writes
    if (fs != DUO_OK) return fs;
  }
  duo_engine* e = new duo_engine();
  e->cfg = c;
  e->full.assign(c.full_attention_host, c.full_attention_host + c.layers);
  e->cfg.full_attention_host = nullptr;
  e->kd = c.hk * c.dk;
  e->vd = c.hv * c.dv;
  e->conv_dim = 2 * e->kd + e->vd;
  e->w_lin = e->conv_dim + e->vd + 2 * c.hv;
  e->w_full = c.nh * 2 * c.hd + 2 * c.nkv * c.hd;
  e->wmax = std::max(std::max(e->w_lin, e->w_full), 2 * c.inter);
  e->group = c.group;
  e->act = c.act_dtype;
  e->act_size = act_bytes(c.act_dtype);
  // inv_freq[j] = 1 / theta^(2j / rot) in f32, the way transformers computes the default RoPE table
  std::vector<float> inv(c.rot / 2);
  for (int j = 0; j < c.rot / 2; j++) {
    const float ex = (float)(2 * j) / (float)c.rot;
    inv[j] = 1.0f / powf(c.theta, ex);
  }
  void* p = nullptr;
  int s = e->dalloc(&p, inv.size() * 4, false);
  if (s != DUO_OK) { delete e; return s; }
  e->inv_freq = static_cast<float*>(p);
  if (cudaMemcpy(e->inv_freq, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
    delete e;
    return fail(DUO_ECUDA, "engine_create: copy of the rotary table failed");
  }
  *out = e;
  return DUO_OK;
}

extern "C" void duo_engine_destroy(duo_engine* e) { delete e; }

extern "C" int duo_engine_load(duo_engine* e, const duo_weights_view* wv, duo_stream stream) {
  DUO_TRY(check_engine(e, false, false));
  DUO_CHECK_ARG(wv && wv->layers_host && wv->embed.q && wv->embed.s && wv->final_norm, "engine_load: null pointer");
  const duo_config& c = e->cfg;
  e->w = *wv;
  e->lw.assign(wv->layers_host, wv->layers_host + c.layers);
  e->w.layers_host = nullptr;
  for (int l = 0; l < c.layers; l++) {
    const duo_layer_view& L = e->lw[l];
    DUO_CHECK_ARG(L.in_norm && L.post_norm && L.proj.q && L.out.q && L.gu.q && L.down.q, "engine_load: null layer weight");
    if (e->is_full(l)) DUO_CHECK_ARG(L.q_norm && L.k_norm, "engine_load: null q/k norm");
    else DUO_CHECK_ARG(L.conv && L.a_log && L.dt_bias && L.gnorm, "engine_load: null DeltaNet weight");
  }
  cudaStream_t st = as_stream(stream);
  e->p_proj.assign(c.layers, Pack{});
  e->p_out.assign(c.layers, Pack{});
  e->p_gu.assign(c.layers, Pack{});
  e->p_down.assign(c.layers, Pack{});
  if (e->act != DUO_F32) {
    for (int l = 0; l < c.layers; l++) {
      const duo_layer_view& L = e->lw[l];
      const bool full = e->is_full(l);
      DUO_TRY(build_pack(e, L.proj, full ? e->w_full : e->w_lin, c.hidden, 0, &e->p_proj[l], st));
      DUO_TRY(build_pack(e, L.out, c.hidden, full ? c.nh * c.hd : e->vd, 0, &e->p_out[l], st));
      DUO_TRY(build_pack(e, L.gu, 2 * c.inter, c.hidden, c.inter, &e->p_gu[l], st));
      DUO_TRY(build_pack(e, L.down, c.hidden, c.inter, 0, &e->p_down[l], st));
    }
    DUO_TRY(build_pack(e, wv->embed, c.vocab, c.hidden, 0, &e->p_embed, st));
  }
  e->loaded = true;
  return DUO_OK;
}

extern "C" int duo_engine_alloc(duo_engine* e, int rows, int max_len, int max_tokens) {
  DUO_TRY(check_engine(e, false, false));
  DUO_CHECK_ARG(rows >= 1 && max_len >= 1 && max_tokens >= 1, "engine_alloc: sizes must be >= 1");
  e->free_state();
  const duo_config& c = e->cfg;
  const size_t as = e->act_size;
  const long Mx = std::max(max_tokens, rows);
  auto A = [&](void** p, size_t bytes) { return e->dalloc(p, bytes, true); };
  void* p;
  DUO_TRY(A(&p, Mx * c.hidden * 4)); e->x = (float*)p;
  DUO_TRY(A(&e->xn, Mx * c.hidden * as));
  for (auto& np : e->nrm_part) {
    DUO_TRY(A(&p, (size_t)std::max<long>(256L * (c.hidden / 128 + 1), Mx * (c.hidden / 256 + 1)) * 4));
    np = (float*)p;
  }
  DUO_TRY(A(&e->y, Mx * e->wmax * as));
  DUO_TRY(A(&e->qkv, Mx * e->conv_dim * as));
  DUO_TRY(A(&p, Mx * c.hv * 4)); e->g = (float*)p;
  DUO_TRY(A(&p, Mx * c.hv * 4)); e->beta = (float*)p;
  DUO_TRY(A(&e->o, Mx * std::max(e->vd, c.nh * c.hd) * as));
  DUO_TRY(A(&e->q, Mx * c.nh * c.hd * as));
  DUO_TRY(A(&e->a, Mx * c.inter * as));
  DUO_TRY(A(&p, (size_t)rows * c.hidden * 4)); e->last = (float*)p;
  DUO_TRY(A(&e->xn_last, (size_t)rows * c.hidden * as));
  DUO_TRY(A(&p, (size_t)rows * c.vocab * 4)); e->logits = (float*)p;
  DUO_TRY(A(&p, (size_t)rows * 4)); e->amax = (int32_t*)p;
  DUO_TRY(A(&p, Mx * 4)); e->ids = (int32_t*)p;
  DUO_TRY(A(&p, (size_t)rows * 4)); e->len_dev = (int32_t*)p;
  DUO_TRY(A(&p, 16)); e->step_ctr = (int32_t*)p;
  DUO_TRY(A(&p, (size_t)rows * c.hidden * 4)); e->vec = (float*)p;
  e->attn_work_floats_n = attn_work_floats(rows, c.nh, max_len);
  DUO_TRY(A(&p, e->attn_work_floats_n * 4)); e->attn_work = (float*)p;
  // chunk workspace: a forward of r rows x T tokens (r T <= max_tokens, r <= rows) has r ceil(T / 64) <=
  // (max_tokens + 63 rows) / 64 chunks per head
  e->chunk_ws_bytes = 0;
  e->chunk_ws = nullptr;
  if (e->act != DUO_F32 && c.layers > 0) {
    e->chunk_ws_bytes = gdn_chunk_ws_bytes(1, (int)std::min<long>(max_tokens + 63L * rows, 1L << 30), c.hv);
    DUO_TRY(A(&e->chunk_ws, e->chunk_ws_bytes));
  }
  e->ls.assign(c.layers, LayerState{});
  std::vector<float> ones(std::max(c.hv, 1), 1.f);
  for (int l = 0; l < c.layers; l++) {
    LayerState& S = e->ls[l];
    if (e->is_full(l)) {
      const size_t kv = (size_t)rows * max_len * c.nkv * c.hd * as;
      DUO_TRY(A(&S.kc, kv));
      DUO_TRY(A(&S.vc, kv));
      DUO_CUDA_TRY(cudaMemset(S.kc, 0, kv));
      DUO_CUDA_TRY(cudaMemset(S.vc, 0, kv));
    } else {
      const size_t cs = (size_t)rows * (c.ks - 1) * e->conv_dim * 4;
      const size_t ss = (size_t)rows * c.hv * c.dk * c.dv * 4;
      DUO_TRY(A(&p, cs)); S.conv = (float*)p;
      DUO_TRY(A(&p, ss)); S.S = (float*)p;
      DUO_TRY(A(&p, c.hv * 4)); S.head_scale = (float*)p;
      DUO_CUDA_TRY(cudaMemset(S.conv, 0, cs));
      DUO_CUDA_TRY(cudaMemset(S.S, 0, ss));
      DUO_CUDA_TRY(cudaMemcpy(S.head_scale, ones.data(), c.hv * 4, cudaMemcpyHostToDevice));
    }
    DUO_TRY(A(&p, kMaxPush * 4)); S.push_neuron = (int32_t*)p;
    DUO_TRY(A(&p, kMaxPush * 4)); S.push_mode = (int32_t*)p;
    DUO_TRY(A(&p, (size_t)kMaxPush * rows * 4)); S.push_vals = (float*)p;
  }
  {
    void* h = nullptr;
    if (cudaHostAlloc(&h, (size_t)kStage * Mx * 4, cudaHostAllocPortable) != cudaSuccess) {
      cudaGetLastError();
      return fail(DUO_ENOMEM, "engine_alloc: pinned staging of the token ids");
    }
    e->ids_stage = static_cast<int32_t*>(h);
    for (cudaEvent_t& ev : e->stage_ev) DUO_CUDA_TRY(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    e->stage_next = 0;
  }
  DUO_CUDA_TRY(cudaMemset(e->len_dev, 0, rows * 4));
  DUO_CUDA_TRY(cudaMemset(e->vec, 0, (size_t)rows * c.hidden * 4));
  DUO_CUDA_TRY(cudaMemset(e->last, 0, (size_t)rows * c.hidden * 4));
  DUO_CUDA_TRY(cudaDeviceSynchronize());
  e->rows = rows;
  e->max_len = max_len;
  e->max_tokens = max_tokens;
  e->len.assign(rows, 0);
  return DUO_OK;
}

extern "C" int duo_engine_reset_all(duo_engine* e, duo_stream stream) {
  DUO_TRY(check_engine(e, false, true));
  const duo_config& c = e->cfg;
  cudaStream_t st = as_stream(stream);
  for (int l = 0; l < c.layers; l++) {
    if (e->is_full(l)) continue;
    DUO_CUDA_TRY(cudaMemsetAsync(e->ls[l].conv, 0, (size_t)e->rows * (c.ks - 1) * e->conv_dim * 4, st));
    DUO_CUDA_TRY(cudaMemsetAsync(e->ls[l].S, 0, (size_t)e->rows * c.hv * c.dk * c.dv * 4, st));
  }
  DUO_CUDA_TRY(cudaMemsetAsync(e->len_dev, 0, (size_t)e->rows * 4, st));
  for (int& v : e->len) v = 0;
  return DUO_OK;
}

extern "C" int duo_engine_set_capture(duo_engine* e, int kind, int n_layers, const int32_t* layers_host, float* out,
                                      int cap_t) {
  DUO_CHECK_ARG(e, "null engine");
  DUO_CHECK_ARG(kind >= 0 && kind < DUO_CAP_KINDS, "set_capture: bad kind");
  const int L = e->cfg.layers;
  DUO_CHECK_ARG(n_layers >= 0 && n_layers <= L, "set_capture: bad layer count");
  duo_engine::Capture& k = e->cap[kind];
  if (n_layers == 0) {
    k = duo_engine::Capture{};
    return DUO_OK;
  }
  DUO_CHECK_ARG(out && cap_t >= 1, "set_capture: null output or cap_t < 1");
  std::vector<int> slot(L, -1);
  for (int i = 0; i < n_layers; i++) {
    const int l = layers_host ? layers_host[i] : i;
    DUO_CHECK_ARG(l >= 0 && l < L && slot[l] < 0, "set_capture: layer out of range or listed twice");
    slot[l] = i;
  }
  k.slot = std::move(slot);
  k.out = out;
  k.cap_t = cap_t;
  k.t0 = 0;
  k.advance = true;
  return DUO_OK;
}

extern "C" int duo_engine_set_capture_t0(duo_engine* e, int kind, int t0) {
  DUO_CHECK_ARG(e, "null engine");
  DUO_CHECK_ARG(kind >= 0 && kind < DUO_CAP_KINDS && e->cap[kind].on(), "set_capture_t0: that capture is off");
  DUO_CHECK_ARG(t0 >= 0 && t0 < e->cap[kind].cap_t, "set_capture_t0: t0 out of range");
  e->cap[kind].t0 = t0;
  return DUO_OK;
}

extern "C" int duo_engine_set_stop_after(duo_engine* e, int layer) {
  DUO_CHECK_ARG(e, "null engine");
  DUO_CHECK_ARG(layer >= -1 && layer < e->cfg.layers, "set_stop_after: layer out of range");
  e->stop_after = layer == e->cfg.layers - 1 ? -1 : layer;
  return DUO_OK;
}

extern "C" int duo_engine_capture_resid(duo_engine* e, int layer, float* out) {
  DUO_CHECK_ARG(e, "null engine");
  DUO_CHECK_ARG(layer >= -1 && layer < e->cfg.layers, "capture_resid: layer out of range");
  DUO_CHECK_ARG(layer == -1 || out, "capture_resid: null output");
  if (layer < 0) return duo_engine_set_capture(e, DUO_CAP_RESID, 0, nullptr, nullptr, 0);
  const int32_t one = layer;
  DUO_TRY(duo_engine_set_capture(e, DUO_CAP_RESID, 1, &one, out, 1 << 30));
  e->cap[DUO_CAP_RESID].advance = false;  // every forward writes its rows from row 0
  return DUO_OK;
}

extern "C" int duo_engine_reset(duo_engine* e, int row, duo_stream stream) {
  DUO_TRY(check_engine(e, false, true));
  DUO_CHECK_ARG(row >= 0 && row < e->rows, "engine_reset: row out of range");
  const duo_config& c = e->cfg;
  cudaStream_t st = as_stream(stream);
  for (int l = 0; l < c.layers; l++) {
    LayerState& S = e->ls[l];
    if (e->is_full(l)) continue;  // the KV cache is overwritten as positions refill (model.js:352)
    const size_t cs = (size_t)(c.ks - 1) * e->conv_dim * 4, ss = (size_t)c.hv * c.dk * c.dv * 4;
    DUO_CUDA_TRY(cudaMemsetAsync(reinterpret_cast<char*>(S.conv) + row * cs, 0, cs, st));
    DUO_CUDA_TRY(cudaMemsetAsync(reinterpret_cast<char*>(S.S) + row * ss, 0, ss, st));
  }
  DUO_CUDA_TRY(cudaMemsetAsync(e->len_dev + row, 0, 4, st));
  e->len[row] = 0;
  return DUO_OK;
}

extern "C" int duo_engine_set_vectors(duo_engine* e, const float* vecs_host, int n_rows, duo_stream stream) {
  DUO_TRY(check_engine(e, false, true));
  DUO_CHECK_ARG(n_rows >= 0 && n_rows <= e->rows && (n_rows == 0 || vecs_host), "set_vectors: bad rows");
  const size_t H = e->cfg.hidden;
  cudaStream_t st = as_stream(stream);
  DUO_CUDA_TRY(cudaMemsetAsync(e->vec, 0, (size_t)e->rows * H * 4, st));
  if (n_rows) DUO_CUDA_TRY(cudaMemcpyAsync(e->vec, vecs_host, (size_t)n_rows * H * 4, cudaMemcpyHostToDevice, st));
  DUO_CUDA_TRY(cudaStreamSynchronize(st));  // the host array may be freed when this returns
  return DUO_OK;
}

extern "C" int duo_engine_set_head_scales(duo_engine* e, int layer, const float* scales_host, duo_stream stream) {
  DUO_TRY(check_engine(e, false, true));
  DUO_CHECK_ARG(layer >= 0 && layer < e->cfg.layers && !e->is_full(layer), "set_head_scales: not a linear layer");
  std::vector<float> ones(e->cfg.hv, 1.f);
  DUO_CUDA_TRY(cudaMemcpyAsync(e->ls[layer].head_scale, scales_host ? scales_host : ones.data(), e->cfg.hv * 4,
                               cudaMemcpyHostToDevice, as_stream(stream)));
  DUO_CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
  return DUO_OK;
}

extern "C" int duo_engine_set_pushes(duo_engine* e, int layer, int n, const int32_t* neurons_host,
                                     const int32_t* modes_host, const float* vals_host, duo_stream stream) {
  DUO_TRY(check_engine(e, false, true));
  DUO_CHECK_ARG(layer >= 0 && layer < e->cfg.layers, "set_pushes: layer out of range");
  if (n > kMaxPush) return fail(DUO_EINVAL, "set_pushes: at most " + std::to_string(kMaxPush) + " records per layer");
  DUO_CHECK_ARG(n >= 0 && (n == 0 || (neurons_host && modes_host && vals_host)), "set_pushes: null pointer");
  for (int i = 0; i < n; i++) {
    DUO_CHECK_ARG(neurons_host[i] == DUO_ALL_NEURONS || (neurons_host[i] >= 0 && neurons_host[i] < e->cfg.inter),
                  "set_pushes: neuron out of range");
    DUO_CHECK_ARG(modes_host[i] == DUO_PUSH_ADD || modes_host[i] == DUO_PUSH_MUL, "set_pushes: bad mode");
  }
  LayerState& S = e->ls[layer];
  cudaStream_t st = as_stream(stream);
  if (n) {
    DUO_CUDA_TRY(cudaMemcpyAsync(S.push_neuron, neurons_host, n * 4, cudaMemcpyHostToDevice, st));
    DUO_CUDA_TRY(cudaMemcpyAsync(S.push_mode, modes_host, n * 4, cudaMemcpyHostToDevice, st));
    DUO_CUDA_TRY(cudaMemcpyAsync(S.push_vals, vals_host, (size_t)n * e->rows * 4, cudaMemcpyHostToDevice, st));
    DUO_CUDA_TRY(cudaStreamSynchronize(st));  // the host arrays may be freed when this returns
  }
  S.push_count = n;
  return DUO_OK;
}

extern "C" int duo_engine_forward_device(duo_engine* e, const int32_t* ids, int row_base, int rows, int t,
                                         int vec_layer, duo_stream stream) {
  DUO_TRY(fault_gate("forward"));
  DUO_TRY(check_engine(e, true, true));
  DUO_CHECK_ARG(ids, "forward: null ids");
  DUO_CHECK_ARG(vec_layer >= -1 && vec_layer < e->cfg.layers, "forward: vec_layer out of range");
  DUO_TRY(check_rows(e, row_base, rows, t));
  DUO_TRY(forward_impl(e, ids, row_base, rows, t, vec_layer, as_stream(stream)));
  for (int r = row_base; r < row_base + rows; r++) e->len[r] += t;
  return DUO_OK;
}

extern "C" int duo_engine_forward(duo_engine* e, const int32_t* ids_host, int row_base, int rows, int t,
                                  int vec_layer, duo_stream stream) {
  DUO_TRY(fault_gate("forward"));
  DUO_TRY(check_engine(e, true, true));
  DUO_CHECK_ARG(ids_host, "forward: null ids");
  DUO_TRY(check_rows(e, row_base, rows, t));
  cudaStream_t st = as_stream(stream);
  const int s = e->stage_next;
  e->stage_next = (s + 1) % kStage;
  DUO_CUDA_TRY(cudaEventSynchronize(e->stage_ev[s]));  // the copy that last read this slot has run
  int32_t* stage = e->ids_stage + (size_t)s * std::max<long>(e->max_tokens, e->rows);
  std::memcpy(stage, ids_host, (size_t)rows * t * 4);
  DUO_CUDA_TRY(cudaMemcpyAsync(e->ids, stage, (size_t)rows * t * 4, cudaMemcpyHostToDevice, st));
  DUO_CUDA_TRY(cudaEventRecord(e->stage_ev[s], st));
  return duo_engine_forward_device(e, e->ids, row_base, rows, t, vec_layer, stream);
}

extern "C" int duo_engine_logits(duo_engine* e, int row0, int n, float* out, duo_stream stream) {
  DUO_TRY(fault_gate("logits"));
  DUO_TRY(check_engine(e, true, true));
  DUO_CHECK_ARG(out && n >= 1 && row0 >= 0 && row0 + n <= e->rows, "logits: bad rows");
  return logits_impl(e, row0, n, out, as_stream(stream));
}

extern "C" int duo_engine_argmax(duo_engine* e, int row0, int n, int32_t* out, duo_stream stream) {
  DUO_TRY(fault_gate("argmax"));
  DUO_TRY(check_engine(e, true, true));
  DUO_CHECK_ARG(out && n >= 1 && row0 >= 0 && row0 + n <= e->rows, "argmax: bad rows");
  cudaStream_t st = as_stream(stream);
  return greedy_impl(e, row0, n, out, st);
}

namespace {
// step < 0: the step index comes from the device counter (a step captured once and replayed)
int generate_step(duo_engine* e, int vec_layer, int32_t* tokens_out, int n_steps, int step, cudaStream_t st) {
  DUO_TRY(greedy_impl(e, 0, e->rows, e->amax, st));
  PROF_TRY(DUO_PROF_OTHER, launch_feed_tokens(e->amax, e->rows, e->ids, tokens_out, n_steps, step < 0 ? 0 : step,
                                              step < 0 ? e->step_ctr : nullptr, st));
  return forward_impl(e, e->ids, 0, e->rows, 1, vec_layer, st);
}

bool graphs_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("DUO_GRAPH");
    return !(v && v[0] == '0');
  }();
  return on;
}

// The decode steps of one generate call as replays of a CUDA graph of one step, captured on the caller's stream:
// the ~140 launches of a step are submitted once, which saves ~3-4% of a step's device time.  Only on a
// non-default stream that is not already capturing, with no capture hook or profiling active (their host
// bookkeeping changes per step).  Returns DUO_OK with *done = false when the caller should launch directly.
int generate_graphed(duo_engine* e, int n_steps, int vec_layer, int32_t* tokens_out, cudaStream_t st, bool* done) {
  *done = false;
  if (!graphs_enabled() || st == nullptr || n_steps < 2 || e->prof_mask) return DUO_OK;
  for (const auto& k : e->cap)
    if (k.on()) return DUO_OK;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    (void)cudaGetLastError();
    return DUO_OK;
  }
  DUO_CUDA_TRY(cudaMemsetAsync(e->step_ctr, 0, sizeof(int32_t), st));
  const unsigned long long c0 = launch_count();
  DUO_CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
  const int rc = generate_step(e, vec_layer, tokens_out, n_steps, -1, st);
  const long long per_step = (long long)(launch_count() - c0);  // captured, not yet run
  cudaGraph_t g = nullptr;
  const cudaError_t ec = cudaStreamEndCapture(st, &g);
  if (rc != DUO_OK || ec != cudaSuccess || g == nullptr) {  // not capturable here: launch directly
    if (g) cudaGraphDestroy(g);
    (void)cudaGetLastError();
    count_launches(-per_step);
    return DUO_OK;
  }
  cudaGraphExec_t ge = nullptr;
  const cudaError_t ei = cudaGraphInstantiateWithFlags(&ge, g, 0);
  cudaGraphDestroy(g);
  if (ei != cudaSuccess) {
    (void)cudaGetLastError();
    count_launches(-per_step);
    return DUO_OK;
  }
  int status = DUO_OK, launched = 0;
  for (int s = 0; s < n_steps; s++) {
    status = fault_gate("generate");  // a fault seen by an earlier step's last kernel stops the loop
    if (status != DUO_OK) break;
    const cudaError_t el = cudaGraphLaunch(ge, st);
    if (el != cudaSuccess) {
      status = fail(DUO_ECUDA, std::string("generate: graph launch failed: ") + cudaGetErrorString(el));
      break;
    }
    for (int r = 0; r < e->rows; r++) e->len[r] += 1;
    launched++;
  }
  count_launches(per_step * (launched - 1));  // duo_launch_count counts the kernels the replays ran
  cudaGraphExecDestroy(ge);  // released once its launches complete
  *done = true;
  return status;
}
}  // namespace

extern "C" int duo_engine_generate(duo_engine* e, int n_steps, int vec_layer, int32_t* tokens_out, duo_stream stream) {
  DUO_TRY(fault_gate("generate"));
  DUO_TRY(check_engine(e, true, true));
  DUO_CHECK_ARG(n_steps >= 0 && (n_steps == 0 || tokens_out), "generate: bad arguments");
  DUO_CHECK_ARG(vec_layer >= -1 && vec_layer < e->cfg.layers, "generate: vec_layer out of range");
  DUO_CHECK_ARG(e->rows <= e->max_tokens, "generate: rows exceed max_tokens");
  for (int r = 0; r < e->rows; r++)
    if (e->len[r] + n_steps > e->max_len) return fail(DUO_ESTATE, "generate: a row would exceed max_len");
  cudaStream_t st = as_stream(stream);
  bool done = false;
  DUO_TRY(generate_graphed(e, n_steps, vec_layer, tokens_out, st, &done));
  if (done) return DUO_OK;
  for (int s = 0; s < n_steps; s++) {
    DUO_TRY(fault_gate("generate"));  // a fault seen by an earlier step's last kernel stops the loop
    DUO_TRY(generate_step(e, vec_layer, tokens_out, n_steps, s, st));
    for (int r = 0; r < e->rows; r++) e->len[r] += 1;
  }
  return DUO_OK;
}

extern "C" int duo_engine_row_len(duo_engine* e, int row) {
  DUO_TRY(check_engine(e, false, true));
  DUO_CHECK_ARG(row >= 0 && row < e->rows, "row_len: row out of range");
  return e->len[row];
}

extern "C" int duo_engine_profile(duo_engine* e, unsigned mask) {
  DUO_CHECK_ARG(e, "null engine");
  for (auto& k : e->prof) k.used = 0;
  e->prof_mask = mask;
  return DUO_OK;
}

extern "C" int duo_engine_profile_read(duo_engine* e, double* ms_out, long long* launches_out) {
  DUO_CHECK_ARG(e && ms_out && launches_out, "profile_read: null pointer");
  DUO_CUDA_TRY(cudaDeviceSynchronize());
  for (int kind = 0; kind < DUO_PROF_KINDS; kind++) {
    auto& k = e->prof[kind];
    double ms = 0;
    for (size_t i = 0; i + 1 < k.used; i += 2) {
      float t = 0.f;
      DUO_CUDA_TRY(cudaEventElapsedTime(&t, k.ev[i], k.ev[i + 1]));
      ms += t;
    }
    ms_out[kind] = ms;
    launches_out[kind] = (long long)(k.used / 2);
    k.used = 0;
  }
  return DUO_OK;
}
