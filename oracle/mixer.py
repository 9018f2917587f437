"""Gated DeltaNet and gated attention ops, restated in torch fp32 on the CPU (test infrastructure only).

Sources restated (no code copied):
  [HF]  transformers 5.5.0, transformers/models/qwen3_5/modeling_qwen3_5.py, the module the reference's PyTorch tools
        and golden generator run (tests/engine_ref.py:4-8, tools/find_steering.py:89-93).  It is a third-party
        dependency, not vendored in the reference; line numbers below are into that file.
  [WGSL] the reference engine's kernels, engine/kernels_qwen35.js and engine/kernels.js.

Every function works on CPU tensors in float32 (float64 where a caller asks for a tighter reference).
"""
import math

import torch
import torch.nn.functional as F


# ----------------------------------------------------------------------------------------------------------------
# normalisations and gates


def rmsnorm(x, w, eps, offset=True):
    """RMSNorm over the last dim: x * rsqrt(mean(x^2) + eps) * (1 + w) (offset) or * w.

    [HF] 711-724 (Qwen3_5RMSNorm, weight stored as w - 1); [WGSL] kernels.js:226-246 (OFFSET flag)."""
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return xf * r * ((1.0 + w.float()) if offset else w.float())


def swiglu_push(gu, inter, pushes, row_of):
    """a = silu(gate) * up of the fused [M, 2 inter] gate|up projection, then the layer's neuron pushes in record
    order ([WGSL] kernels_qwen35.js:250-280): (neuron or None = every neuron, "add" | "mul", per-row values), row i
    of `gu` taking the value of row row_of[i]."""
    a = F.silu(gu[:, :inter]) * gu[:, inter:]
    for n, mode, vals in pushes:
        v = torch.as_tensor(vals, dtype=a.dtype)[torch.as_tensor(row_of)]
        cols = slice(None) if n is None else n
        v = v[:, None] if n is None else v
        a[:, cols] = a[:, cols] * v if mode == "mul" else a[:, cols] + v
    return a


def l2norm(x, eps=1e-6):
    """x * rsqrt(sum(x^2) + eps) over the last dim.  [HF] 228-231; [WGSL] kernels_qwen35.js:215-223."""
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def gdn_gates(a, b, a_log, dt_bias):
    """beta = sigmoid(b); g = -exp(A_log) * softplus(a + dt_bias) (log-decay per token and head).

    [HF] 490-492; [WGSL] kernels_qwen35.js:208, 227-228.  torch's softplus switches to the identity above 20, as the
    WGSL `softplus` does (kernels_qwen35.js:11)."""
    beta = torch.sigmoid(b.float())
    g = -torch.exp(a_log.float()) * F.softplus(a.float() + dt_bias.float())
    return beta, g


def gated_rmsnorm(o, z, w, eps):
    """Norm-before-gate RMSNorm over the head dim: o * rsqrt(mean(o^2) + eps) * w * silu(z) (w not offset).

    [HF] 175-190 (Qwen3_5RMSNormGated); [WGSL] kernels_qwen35.js:237-243."""
    of = o.float()
    r = torch.rsqrt(of.pow(2).mean(-1, keepdim=True) + eps)
    return of * r * w.float() * F.silu(z.float())


# ----------------------------------------------------------------------------------------------------------------
# causal depthwise conv with carried state


def causal_conv1d(x, weight, state=None):
    """Causal depthwise conv (kernel KS) over channels with a carried state of the previous KS-1 inputs, then SiLU.

    x: [B, T, C] token-major (the qkv columns of the fused projection); weight: [C, KS]; state: [B, KS-1, C] holding
    the last KS-1 inputs of earlier calls, oldest first (zeros for a fresh row).  Returns (out [B, T, C], new_state).

    [HF] 451-476 (prefill: F.conv1d with KS-1 zero padding, then SiLU; the cache keeps the last inputs) and 210-226
    (decode update: concatenate state and input, convolve without padding, keep the tail);
    [WGSL] kernels_qwen35.js:129-178 (same arithmetic per (token, channel) and the state shift).
    """
    bsz, t, c = x.shape
    ks = weight.shape[1]
    if state is None:
        state = torch.zeros(bsz, ks - 1, c, dtype=x.dtype)
    seq = torch.cat([state.to(x.dtype), x], dim=1)  # [B, KS-1+T, C]
    out = torch.zeros(bsz, t, c, dtype=torch.float32)
    for i in range(ks):  # out[t] = sum_i w[:, i] * seq[t + i]   (input at token t - (KS-1) + i)
        out = out + weight[:, i].float()[None, None, :] * seq[:, i:i + t, :].float()
    new_state = seq[:, -(ks - 1):, :].clone()
    return F.silu(out), new_state


# ----------------------------------------------------------------------------------------------------------------
# the delta rule


def recurrent_gated_delta_rule(q, k, v, g, beta, state=None, l2norm_qk=True):
    """Token-by-token gated delta rule.  q, k: [B, T, H, dk]; v: [B, T, H, dv]; g, beta: [B, T, H];
    state: [B, H, dk, dv] or None.  Returns (o [B, T, H, dv] f32, final state [B, H, dk, dv] f32).

    Per token: S *= exp(g); u = S^T k; S += k (beta (v - u))^T; o = S^T (q / sqrt(dk)).
    [HF] 314-353 (torch_recurrent_gated_delta_rule); [WGSL] kernels_qwen35.js:209-236 (the same recurrence).
    """
    dt = torch.float64 if q.dtype == torch.float64 else torch.float32
    q, k, v, g, beta = (x.to(dt) for x in (q, k, v, g, beta))
    if l2norm_qk:
        q, k = l2norm(q), l2norm(k)
    bsz, t, h, dk = k.shape
    dv = v.shape[-1]
    q = q * (1.0 / math.sqrt(dk))
    s = torch.zeros(bsz, h, dk, dv, dtype=dt) if state is None else state.to(dt).clone()
    o = torch.zeros(bsz, t, h, dv, dtype=dt)
    for i in range(t):
        s = s * torch.exp(g[:, i])[:, :, None, None]
        u = torch.einsum("bhkv,bhk->bhv", s, k[:, i])
        d = (v[:, i] - u) * beta[:, i][:, :, None]
        s = s + k[:, i][:, :, :, None] * d[:, :, None, :]
        o[:, i] = torch.einsum("bhkv,bhk->bhv", s, q[:, i])
    return o, s


def chunk_gated_delta_rule(q, k, v, g, beta, state=None, chunk=64, l2norm_qk=True):
    """Chunked (WY / UT-transform) form of the gated delta rule, same signature as recurrent_gated_delta_rule.

    Restates the published chunk algorithm of [HF] 234-311 (torch_chunk_gated_delta_rule), per chunk of C tokens with
    cumulative log-decay G (inclusive cumsum of g inside the chunk):
      L[i, j] = beta_i (k_i . k_j) exp(G_i - G_j) for j < i        (strictly lower)
      T       = (I + L)^-1                                          (unit lower triangular; the UT transform)
      U       = T (beta * v),    W = T (beta * exp(G) * k)
      V'      = U - W S                                             (S: state entering the chunk)
      o       = (q * exp(G)) S + tril(q k^T * exp(G_i - G_j)) V'
      S      <- exp(G_last) S + (k * exp(G_last - G))^T V'
    [HF] solves for T by forward substitution row by row (278-281); this restatement calls a triangular solve, which
    gives the same matrix up to rounding.  T is zero-padded up to a multiple of C ([HF] 253-258).
    """
    dt = torch.float64 if q.dtype == torch.float64 else torch.float32
    q, k, v, g, beta = (x.to(dt) for x in (q, k, v, g, beta))
    if l2norm_qk:
        q, k = l2norm(q), l2norm(k)
    bsz, t, h, dk = k.shape
    dv = v.shape[-1]
    pad = (chunk - t % chunk) % chunk
    q = q * (1.0 / math.sqrt(dk))
    # [B, H, T, d] layout, padded with zeros
    q, k, v = (F.pad(x.transpose(1, 2), (0, 0, 0, pad)) for x in (q, k, v))
    g, beta = (F.pad(x.transpose(1, 2), (0, pad)) for x in (g, beta))
    n = (t + pad) // chunk
    q, k, v = (x.reshape(bsz, h, n, chunk, -1) for x in (q, k, v))
    g, beta = (x.reshape(bsz, h, n, chunk) for x in (g, beta))
    G = g.cumsum(-1)
    diff = G[..., :, None] - G[..., None, :]  # G_i - G_j
    lower_strict = torch.tril(torch.ones(chunk, chunk, dtype=torch.bool), -1)
    lower_incl = torch.tril(torch.ones(chunk, chunk, dtype=torch.bool), 0)
    zero = torch.zeros_like(diff)
    decay = torch.where(lower_incl, torch.exp(torch.where(lower_incl, diff, zero)), zero)  # exp(G_i - G_j), j <= i
    kk = k @ k.transpose(-1, -2)
    L = torch.where(lower_strict, beta[..., :, None] * kk * decay, torch.zeros_like(kk))
    eye = torch.eye(chunk, dtype=dt)
    T = torch.linalg.solve_triangular(eye + L, eye.expand_as(L), upper=False, unitriangular=True)
    U = T @ (v * beta[..., None])
    W = T @ (k * (beta * torch.exp(G))[..., None])
    s = torch.zeros(bsz, h, dk, dv, dtype=dt) if state is None else state.to(dt).clone()
    o = torch.zeros(bsz, h, n, chunk, dv, dtype=dt)
    for c in range(n):
        qc, kc = q[:, :, c], k[:, :, c]
        Gc = G[:, :, c]
        vn = U[:, :, c] - W[:, :, c] @ s
        a = torch.where(lower_incl, (qc @ kc.transpose(-1, -2)) * decay[:, :, c], torch.zeros(chunk, chunk, dtype=dt))
        o[:, :, c] = (qc * torch.exp(Gc)[..., None]) @ s + a @ vn
        glast = Gc[..., -1]
        s = s * torch.exp(glast)[..., None, None] + (kc * torch.exp(glast[..., None] - Gc)[..., None]).transpose(-1, -2) @ vn
    o = o.reshape(bsz, h, n * chunk, dv)[:, :, :t].transpose(1, 2)
    return o, s


# ----------------------------------------------------------------------------------------------------------------
# gated attention


def rope_inv_freq(rot, theta):
    """inv_freq[j] = 1 / theta^(2j / rot), computed in f32 as [HF] 117-122 does (compute_default_rope_parameters)."""
    return 1.0 / (theta ** (torch.arange(0, rot, 2, dtype=torch.int64).to(torch.float32) / rot))


def apply_partial_rope(x, pos, inv_freq):
    """Rotate-half RoPE on the first `rot` = 2 * len(inv_freq) dims of x [..., n, hd] at integer positions pos [...].

    [HF] 544-579 (apply_rotary_pos_emb on q_rot, pass-through for the rest; cos/sin of cat(freqs, freqs));
    [WGSL] kernels_qwen35.js:50-59.  For text positions the interleaved M-RoPE of [HF] 157-171 uses the same
    position on all three sections, so it is plain RoPE."""
    rot = 2 * inv_freq.numel()
    freqs = pos.to(torch.float32)[..., None] * inv_freq  # [..., rot/2]
    emb = torch.cat([freqs, freqs], -1)
    cos, sin = emb.cos()[..., None, :], emb.sin()[..., None, :]
    xr, xp = x[..., :rot], x[..., rot:]
    x1, x2 = xr[..., : rot // 2], xr[..., rot // 2:]
    rh = torch.cat([-x2, x1], -1)
    return torch.cat([xr * cos + rh * sin, xp], -1)


def attn_prep(y, q_norm, k_norm, pos, nh, nkv, hd, inv_freq, eps):
    """Split the fused projection y[M, W] = [q+gate (nh * 2hd) | k (nkv hd) | v (nkv hd)] and prepare q, k, v.

    Per head: q and k RMSNorm with (1 + w), then partial RoPE at positions pos[M].  Returns q [M, nh, hd],
    k [M, nkv, hd], v [M, nkv, hd], gate [M, nh * hd].  [HF] 647-668; [WGSL] kernels_qwen35.js:18-69."""
    m = y.shape[0]
    qg = y[:, : nh * 2 * hd].reshape(m, nh, 2 * hd)
    q, gate = qg[..., :hd], qg[..., hd:].reshape(m, nh * hd)
    k = y[:, nh * 2 * hd: nh * 2 * hd + nkv * hd].reshape(m, nkv, hd)
    v = y[:, nh * 2 * hd + nkv * hd: nh * 2 * hd + 2 * nkv * hd].reshape(m, nkv, hd)
    q = apply_partial_rope(rmsnorm(q, q_norm, eps), pos, inv_freq)
    k = apply_partial_rope(rmsnorm(k, k_norm, eps), pos, inv_freq)
    return q, k, v.float(), gate


def cached_attention(q, kc, vc, n_keys, scale):
    """Causal GQA softmax attention of one row's new queries over its cache.

    q: [T, nh, hd] (query t sits at cache position n_keys[t] - 1); kc, vc: [L, nkv, hd]; n_keys: [T] ints.
    Returns o [T, nh, hd].  [HF] 594-616 (eager_attention_forward with repeat_kv); [WGSL] kernels_qwen35.js:73-123."""
    t, nh, hd = q.shape
    nkv = kc.shape[1]
    rep = nh // nkv
    lmax = int(max(n_keys))
    k = kc[:lmax].float().repeat_interleave(rep, dim=1)  # [L, nh, hd]
    v = vc[:lmax].float().repeat_interleave(rep, dim=1)
    s = torch.einsum("thd,lhd->thl", q.float(), k) * scale
    idx = torch.arange(lmax)[None, :]
    mask = idx < torch.as_tensor(n_keys)[:, None]
    s = s.masked_fill(~mask[:, None, :], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("thl,lhd->thd", p, v)
