"""Op-level wrappers over the C ABI (torch tensors in, torch tensors out; torch only allocates and holds memory).

Each function names the reference kernel it replaces; the C entry points in include/duo_mixer.h document the exact
contracts.
"""
import torch

from .lib import (DUO_BF16, DUO_F32, call, dtype_code, ptr, stream_ptr)


def _dev(*ts):
    for t in ts:
        if t is not None and (not t.is_cuda or not t.is_contiguous()):
            raise ValueError("expected contiguous CUDA tensors")


def q8_quantize(w, group=128, stream=None):
    """W[n, k] -> (q int8[n, k], s f32[n, k/group]); group=0 means one scale per row (engine/kernels.js:16-47)."""
    _dev(w)
    n, k = w.shape
    g = k if group == 0 else group
    q = torch.empty(n, k, dtype=torch.int8, device=w.device)
    s = torch.empty(n, k // g, dtype=torch.float32, device=w.device)
    call("duo_q8_quantize", ptr(w), dtype_code(w.dtype), n, k, g, ptr(q), ptr(s), stream_ptr(stream))
    return q, s


def q8_dequantize(q, s, out_dtype=torch.float32, stream=None):
    _dev(q, s)
    n, k = q.shape
    g = k // s.shape[1]
    out = torch.empty(n, k, dtype=out_dtype, device=q.device)
    call("duo_q8_dequantize", ptr(q), ptr(s), n, k, g, ptr(out), dtype_code(out_dtype), stream_ptr(stream))
    return out


def q8_gemv(x, q, s, y=None, accumulate=False, out_dtype=None, stream=None):
    """y[m, n] (+)= x[m, k] . dequant(W)^T for m <= 8 (engine/kernels.js:55-94)."""
    _dev(x, q, s, y)
    m, k = x.shape
    n = q.shape[0]
    g = k // s.shape[1]
    if y is None:
        y = torch.zeros(m, n, dtype=out_dtype or x.dtype, device=x.device)
    call("duo_q8_gemv", ptr(x), dtype_code(x.dtype), m, k, ptr(q), ptr(s), g, n, ptr(y), dtype_code(y.dtype),
         int(accumulate), stream_ptr(stream))
    return y


def q8_gather(ids, q, s, stream=None):
    """y[t, :] = dequant(E)[ids[t], :] (engine/kernels.js:205-221)."""
    _dev(ids, q, s)
    v, k = q.shape
    g = k // s.shape[1]
    y = torch.empty(ids.numel(), k, dtype=torch.float32, device=q.device)
    call("duo_q8_gather", ptr(ids), ids.numel(), ptr(q), ptr(s), g, k, v, ptr(y), stream_ptr(stream))
    return y


def gemm_bf16(a, b, col_scale=None, out=None, out_dtype=torch.bfloat16, accumulate=False, stream=None):
    """C[m, n] (+)= (A[m, k] . B[n, k]^T) * col_scale[n] on the tcgen05 tensor cores."""
    _dev(a, b, col_scale, out)
    m, k = a.shape
    n = b.shape[0]
    if out is None:
        out = torch.zeros(m, n, dtype=out_dtype, device=a.device)
    call("duo_gemm_bf16", ptr(a), m, k, ptr(b), n, ptr(col_scale), ptr(out), dtype_code(out.dtype), out.stride(0),
         int(accumulate), stream_ptr(stream))
    return out


def q8_gemm(x, q, s, y=None, out_dtype=None, accumulate=False, swiglu=False, stream=None):
    """y[m, n] (+)= x[m, k] . dequant(q, s)^T for m <= 256 on the tensor cores, the int8 weights converted on chip
    (engine/kernels.js:97-151); swiglu: q = [gate | up] rows, y = silu(gate) * up [m, n / 2] in x's dtype."""
    _dev(x, q, s, y)
    m, k = x.shape
    n = q.shape[0]
    g = k // s.shape[1]
    if y is None:
        y = torch.zeros(m, n // 2 if swiglu else n, dtype=x.dtype if swiglu else (out_dtype or x.dtype),
                        device=x.device)
    call("duo_q8_gemm", ptr(x), dtype_code(x.dtype), m, k, ptr(q), ptr(s), g, n, int(swiglu), ptr(y),
         dtype_code(y.dtype), y.stride(0), int(accumulate), stream_ptr(stream))
    return y


def interleave_gate_up(gate, up):
    """[inter, k] gate and up weights -> the [2 inter, k] row order duo_gemm_swiglu reads (blocks of 64 rows:
    64 gate rows, then the matching 64 up rows)."""
    inter, k = gate.shape
    if inter % 64:
        raise ValueError("inter must be a multiple of 64")
    return torch.stack([gate.reshape(inter // 64, 64, k), up.reshape(inter // 64, 64, k)], 1).reshape(2 * inter, k)


def gemm_swiglu(a, gu, col_scale=None, pushes=None, t=1, row_base=0, stream=None):
    """silu(gate) * up of (A . GU^T) * col_scale with the neuron pushes of one layer (kernels_qwen35.js:250-280).
    gu is in interleave_gate_up order.  pushes = (neurons int32 [P], modes int32 [P], vals f32 [P, rows])."""
    _dev(a, gu, col_scale)
    m, k = a.shape
    inter = gu.shape[0] // 2
    out = torch.empty(m, inter, dtype=a.dtype, device=a.device)
    if pushes is None:
        pn = pm = pv = None
        count = rows = 0
    else:
        pn, pm, pv = pushes
        _dev(pn, pm, pv)
        count, rows = pv.shape
    call("duo_gemm_swiglu", ptr(a), m, k, ptr(gu), inter, dtype_code(a.dtype), ptr(col_scale), ptr(out), out.stride(0),
         ptr(pn), ptr(pm), ptr(pv), count, rows, t, row_base, stream_ptr(stream))
    return out


def rmsnorm(x, w, eps=1e-6, offset=True, out_dtype=torch.float32, stream=None):
    """y = x * rsqrt(mean(x^2) + eps) * (1 + w) (engine/kernels.js:226-246)."""
    _dev(x, w)
    m, d = x.shape
    y = torch.empty(m, d, dtype=out_dtype, device=x.device)
    call("duo_rmsnorm", ptr(x), m, d, ptr(w), float(eps), int(offset), ptr(y), dtype_code(out_dtype),
         stream_ptr(stream))
    return y


def _gdn(name, q, k, v, g, beta, state, l2norm_qk, stream):
    _dev(q, k, v, g, beta, state)
    b, t, h, dk = q.shape
    dv = v.shape[-1]
    o = torch.empty(b, t, h, dv, dtype=q.dtype, device=q.device)
    call(name, ptr(q), ptr(k), ptr(v), dtype_code(q.dtype), ptr(g), ptr(beta), ptr(state), ptr(o),
         dtype_code(o.dtype), b, t, h, dk, dv, int(l2norm_qk), stream_ptr(stream))
    return o


def gdn_conv(y, conv_w, conv_state, a_log, dt_bias, hk, hv, stream=None):
    """DeltaNet prologue of the fused projection y [b, t, w]: causal conv + SiLU + q/k l2norm with the carried
    conv_state [b, 3, conv_dim] (f32, updated in place), gates beta / g (kernels_qwen35.js:129-178, 208-229).
    Returns qkv [b, t, conv_dim] (y's dtype), g, beta [b, t, hv] f32."""
    _dev(y, conv_w, conv_state, a_log, dt_bias)
    b, t, w = y.shape
    conv_dim = 2 * hk * 128 + hv * 128
    qkv = torch.empty(b, t, conv_dim, dtype=y.dtype, device=y.device)
    g = torch.empty(b, t, hv, dtype=torch.float32, device=y.device)
    beta = torch.empty_like(g)
    call("duo_gdn_conv_fwd", ptr(y), dtype_code(y.dtype), w, ptr(conv_w), ptr(conv_state), ptr(a_log), ptr(dt_bias),
         ptr(qkv), ptr(g), ptr(beta), b, t, hk, hv, 128, 128, stream_ptr(stream))
    return qkv, g, beta


def gdn_recurrent(q, k, v, g, beta, state, l2norm_qk=True, stream=None):
    """Token-by-token gated delta rule; `state` [b, h, 128, 128] f32 is updated in place (kernels_qwen35.js:209-236)."""
    return _gdn("duo_gdn_recurrent_fwd", q, k, v, g, beta, state, l2norm_qk, stream)


def gdn_chunk(q, k, v, g, beta, state, l2norm_qk=True, stream=None):
    """Chunked (64-token WY/UT) gated delta rule on the tensor cores; same contract as gdn_recurrent."""
    return _gdn("duo_gdn_chunk_fwd", q, k, v, g, beta, state, l2norm_qk, stream)


def attention(q, kc, vc, start, gate=None, scale=None, stream=None):
    """Causal GQA attention of q [b, t, nh, hd] over caches [b, L, nkv, hd], optional sigmoid gate [b, t, nh, hd]
    (engine/kernels_qwen35.js:73-123)."""
    _dev(q, kc, vc, start, gate)
    b, t, nh, hd = q.shape
    _, max_len, nkv, _ = kc.shape
    o = torch.empty_like(q)
    scale = hd ** -0.5 if scale is None else scale
    call("duo_attention", ptr(q), ptr(kc), ptr(vc), ptr(start), ptr(gate), nh * hd, ptr(o), dtype_code(q.dtype), b,
         t, nh, nkv, hd, max_len, float(scale), stream_ptr(stream))
    return o


def fault_status():
    """Synchronise the device and read-and-clear the fault word of the tensor-core kernels (0 = no bounded wait gave
    up)."""
    import ctypes as C
    v = C.c_uint(0)
    call("duo_fault_status", C.byref(v))
    return v.value


def push_stats(logits, base, targets, target_logw=None, d=None, stream=None):
    """Next-token statistics of the push probe (engine/analysis.js:480-537) over logits [n, vocab] f32: returns stats
    [n, 6] = (lse, mass, tlse, kl, dp, gain); kl / dp / gain against row base[r] (-1: none); d [n, vocab] (optional)
    is accumulated with lp - lp[base] in place."""
    _dev(logits, base, targets, target_logw, d)
    n, vocab = logits.shape
    stats = torch.empty(n, 6, dtype=torch.float32, device=logits.device)
    call("duo_push_stats", ptr(logits), n, vocab, ptr(base), ptr(targets), ptr(target_logw), targets.numel(),
         ptr(stats), ptr(d), stream_ptr(stream))
    return stats, d
