"""Full Qwen3.5 text-decoder forward with the reference engine's semantics, on the CPU (test infrastructure only).

Mirrors engine/model.js of the reference:
  * weights in the engine's fused layouts (model.js:70-116): linear attention [qkv | z | b | a], full attention
    [q+gate | k | v], MLP [gate | up];
  * `forward(ids, row_base, rows, T, pushes, vec)` = model.js:404-466 `_forward`: `rows` consecutive sequences
    starting at row_base, each with T new tokens continuing from that row's length; token-major activations
    [M = rows * T, width];
  * neuron pushes at the down_proj input (model.js:7-12, kernels_qwen35.js:254-279): per layer a list of records
    (neuron or None for all, "add" | "mul", per-row values indexed by the absolute row);
  * the residual steering vector `vec` after layer `vec`'s MLP, one vector per absolute row (model.js:372-376, 460;
    kernels.js:190-203);
  * per-head output scales on linear-attention layers (model.js:362-369, kernels_qwen35.js:243).
The arithmetic is the restated [HF] math in oracle.mixer, in float32 (float64 on request).
"""
import math

import torch
import torch.nn.functional as F

from . import mixer


class Cfg:
    """Field names follow transformers' Qwen3_5TextConfig and engine/model.js:27-58."""

    def __init__(self, hidden=1024, inter=3584, vocab=248320, layers=24, nh=8, nkv=2, hd=256, rot=64, theta=1e7,
                 hk=16, hv=16, dk=128, dv=128, ks=4, eps=1e-6, full_interval=4, layer_types=None):
        self.hidden, self.inter, self.vocab, self.layers = hidden, inter, vocab, layers
        self.nh, self.nkv, self.hd, self.rot, self.theta = nh, nkv, hd, rot, theta
        self.hk, self.hv, self.dk, self.dv, self.ks, self.eps = hk, hv, dk, dv, ks, eps
        if layer_types is None:
            layer_types = ["full_attention" if (i + 1) % full_interval == 0 else "linear_attention"
                           for i in range(layers)]
        self.layer_types = list(layer_types)
        self.kd, self.vd = hk * dk, hv * dv
        self.conv_dim = 2 * self.kd + self.vd
        self.w_lin = self.conv_dim + self.vd + 2 * hv
        self.w_full = nh * 2 * hd + 2 * nkv * hd


class OracleModel:
    """CPU restatement of the engine's Model with its per-row state (model.js:308-360)."""

    # Where the 16-bit engines round an intermediate to bf16 / f16 (everything else stays f32): each name marks one
    # such point in forward() / logits().  round_points maps names to a rounding function (empty: pure f32).  Two
    # follow the engine's kernel structure: "conv" (the conv prologue's q / k / v) is not rounded in a decode step
    # (T = 1, hk = hv), whose fused DeltaNet kernel keeps them in registers; "gu" (the gate|up projection stored before
    # a separate SwiGLU kernel) exists only in forwards of at most gemv_max token rows, which run the int8 GEMV --
    # larger ones fuse SwiGLU into the tensor-core GEMM's epilogue.
    ROUND_POINTS = ("norm_in", "proj", "conv", "scan_out", "attn_q", "kv", "attn_out", "norm_post", "gu", "mlp_act",
                    "final")

    def __init__(self, cfg, weights, rows, max_len, dtype=torch.float32, round_points=None, gemm_weights=None,
                 gemv_max=8):
        self.cfg, self.w, self.rows, self.max_len, self.dt = cfg, weights, rows, max_len, dtype
        self.round_points = dict(round_points or {})
        # the matrices a forward of more than gemv_max token rows multiplies with (the 16-bit engines' tensor-core
        # pack, bf16(q * s) for G = 128); forwards of up to gemv_max rows use `weights` (the int8 GEMV's f32(q) * s)
        self.w_gemm, self.gemv_max = gemm_weights, gemv_max
        unknown = set(self.round_points) - set(self.ROUND_POINTS) - {"proj_gates"}
        if unknown:
            raise ValueError(f"unknown rounding points {sorted(unknown)}")
        c = cfg
        self.inv_freq = mixer.rope_inv_freq(c.rot, c.theta)
        self.conv = {}
        self.S = {}
        self.kc = {}
        self.vc = {}
        for l, t in enumerate(c.layer_types):
            if t == "linear_attention":
                self.conv[l] = torch.zeros(rows, c.ks - 1, c.conv_dim, dtype=dtype)
                self.S[l] = torch.zeros(rows, c.hv, c.dk, c.dv, dtype=dtype)
            else:
                self.kc[l] = torch.zeros(rows, max_len, c.nkv, c.hd, dtype=dtype)
                self.vc[l] = torch.zeros(rows, max_len, c.nkv, c.hd, dtype=dtype)
        self.len = [0] * rows
        self.vectors = torch.zeros(rows, c.hidden, dtype=dtype)
        self.head_scales = {l: torch.ones(c.hv, dtype=dtype) for l in self.conv}
        self.last = torch.zeros(rows, c.hidden, dtype=dtype)

    def _r(self, name, x):
        fn = self.round_points.get(name)
        return x if fn is None else fn(x)

    # -- state (model.js:352-376)
    def reset(self, r):
        for l in self.conv:
            self.conv[l][r] = 0
            self.S[l][r] = 0
        self.len[r] = 0

    def set_vectors(self, vecs):
        self.vectors.zero_()
        for r, v in enumerate(vecs):
            if v is not None:
                self.vectors[r] = torch.as_tensor(v, dtype=self.dt)

    def set_head_scales(self, scales):
        for l in self.head_scales:
            s = (scales or {}).get(l)
            self.head_scales[l] = torch.ones(self.cfg.hv, dtype=self.dt) if s is None else torch.as_tensor(s, dtype=self.dt)

    # -- forward (model.js:404-466)
    def forward(self, ids, row_base, rows, T, pushes=None, vec=None, capture_resid=False, capture=None,
                stop_after=None):
        """capture: optional dict that receives, per layer, "resid_attn" (after the mixer's out-projection), "act" (the
        down_proj input after pushes) and "resid" (after the MLP and vector add) as lists of [M, width] tensors
        (model.js:445-461); stop_after: last layer to run (model.js:427)."""
        c, dt = self.cfg, self.dt
        M = rows * T
        w = self.w_gemm if (self.w_gemm is not None and M > self.gemv_max) else self.w
        ids = torch.as_tensor(ids, dtype=torch.int64).reshape(M)
        x = self.w["embed"][ids].to(dt)  # kernels.js:205-221 gather (weights given already dequantised)
        pos = torch.tensor([self.len[row_base + i] + t for i in range(rows) for t in range(T)])
        row_of = torch.tensor([row_base + i for i in range(rows) for _ in range(T)])
        pushes = pushes or {}
        resid = []
        for l, lt in enumerate(c.layer_types):
            L = w["layers"][l]
            xn = self._r("norm_in", mixer.rmsnorm(x, L["in_norm"], c.eps).to(dt))
            y = self._r("proj", xn @ L["proj"].to(dt).T)
            if lt == "linear_attention":
                o = self._deltanet(l, L, y, row_base, rows, T)
            else:
                o = self._attention(l, L, y, row_base, rows, T, pos)
            x = x + o @ L["out"].to(dt).T
            if capture is not None:
                capture.setdefault("resid_attn", []).append(x.clone())
            xn = self._r("norm_post", mixer.rmsnorm(x, L["post_norm"], c.eps).to(dt))
            gu = xn @ L["gu"].to(dt).T
            if M <= self.gemv_max:
                gu = self._r("gu", gu)
            a = F.silu(gu[:, : c.inter]) * gu[:, c.inter:]
            for rec in pushes.get(l, []):  # kernels_qwen35.js:270-276, in record order
                vals = torch.as_tensor([rec["vals"][int(r)] if int(r) < len(rec["vals"]) else
                                        (1.0 if rec.get("mode") == "mul" else 0.0) for r in row_of], dtype=dt)
                cols = slice(None) if rec.get("n") is None else rec["n"]
                if rec.get("mode", "add") == "mul":
                    a[:, cols] = a[:, cols] * (vals[:, None] if rec.get("n") is None else vals)
                else:
                    a[:, cols] = a[:, cols] + (vals[:, None] if rec.get("n") is None else vals)
            a = self._r("mlp_act", a)
            if capture is not None:
                capture.setdefault("act", []).append(a.clone())
            x = x + a @ L["down"].to(dt).T
            if vec == l:  # kernels.js:190-203, one vector per absolute row
                x = x + self.vectors[row_of]
            if capture_resid:
                resid.append(x.clone())
            if capture is not None:
                capture.setdefault("resid", []).append(x.clone())
            if stop_after is not None and l == stop_after:
                break
        for i in range(rows):
            self.last[row_base + i] = x[i * T + T - 1]
            self.len[row_base + i] += T
        return resid if capture_resid else None

    def _deltanet(self, l, L, y, row_base, rows, T):
        c, dt = self.cfg, self.dt
        M = rows * T
        qkv = y[:, : c.conv_dim].reshape(rows, T, c.conv_dim)
        z = y[:, c.conv_dim: c.conv_dim + c.vd].reshape(rows, T, c.hv, c.dv)
        b = self._r("proj_gates", y[:, c.conv_dim + c.vd: c.conv_dim + c.vd + c.hv]).reshape(rows, T, c.hv)
        a = self._r("proj_gates", y[:, c.conv_dim + c.vd + c.hv:]).reshape(rows, T, c.hv)
        rs = slice(row_base, row_base + rows)
        conv_out, new_state = mixer.causal_conv1d(qkv, L["conv"], self.conv[l][rs])
        self.conv[l][rs] = new_state.to(dt)
        conv_out = conv_out.to(dt)
        q = conv_out[..., : c.kd].reshape(rows, T, c.hk, c.dk)
        k = conv_out[..., c.kd: 2 * c.kd].reshape(rows, T, c.hk, c.dk)
        v = conv_out[..., 2 * c.kd:].reshape(rows, T, c.hv, c.dv)
        conv_rounded = "conv" in self.round_points and not (T == 1 and c.hk == c.hv)
        if conv_rounded:  # the engine's conv writes q and k already l2-normalised
            q, k, v = self._r("conv", mixer.l2norm(q)), self._r("conv", mixer.l2norm(k)), self._r("conv", v)
        if c.hv // c.hk > 1:
            q = q.repeat_interleave(c.hv // c.hk, dim=2)
            k = k.repeat_interleave(c.hv // c.hk, dim=2)
        beta, g = mixer.gdn_gates(a, b, L["alog"], L["dtb"])
        rule = mixer.recurrent_gated_delta_rule if T == 1 else mixer.chunk_gated_delta_rule
        o, s = rule(q, k, v, g.to(dt), beta.to(dt), state=self.S[l][rs], l2norm_qk=not conv_rounded)
        self.S[l][rs] = s.to(dt)
        o = mixer.gated_rmsnorm(o, z, L["gnorm"], c.eps).to(dt)
        o = o * self.head_scales[l][None, None, :, None]
        return self._r("scan_out", o.reshape(M, c.vd))

    def _attention(self, l, L, y, row_base, rows, T, pos):
        c, dt = self.cfg, self.dt
        q, k, v, gate = mixer.attn_prep(y, L["qnorm"], L["knorm"], pos, c.nh, c.nkv, c.hd, self.inv_freq, c.eps)
        q, k, v = self._r("attn_q", q.to(dt)), self._r("kv", k.to(dt)), self._r("kv", v.to(dt))
        out = torch.zeros(rows * T, c.nh, c.hd, dtype=dt)
        for i in range(rows):
            r = row_base + i
            p0 = self.len[r]
            if p0 + T > self.max_len:
                raise ValueError("KV cache overflow")
            self.kc[l][r, p0:p0 + T] = k[i * T:(i + 1) * T]
            self.vc[l][r, p0:p0 + T] = v[i * T:(i + 1) * T]
            n_keys = [p0 + t + 1 for t in range(T)]
            out[i * T:(i + 1) * T] = mixer.cached_attention(q[i * T:(i + 1) * T], self.kc[l][r], self.vc[l][r],
                                                            n_keys, 1.0 / math.sqrt(c.hd)).to(dt)
        out = out.reshape(rows * T, c.nh * c.hd) * torch.sigmoid(gate.to(dt))
        return self._r("attn_out", out)

    # -- heads (model.js:472-500)
    def logits(self, rows=None):
        rows = list(range(self.rows)) if rows is None else rows
        w = self.w_gemm if (self.w_gemm is not None and len(rows) > self.gemv_max) else self.w
        h = self._r("final", mixer.rmsnorm(self.last[rows], self.w["final_norm"], self.cfg.eps).to(self.dt))
        return h @ w["embed"].to(self.dt).T

    def argmax(self, rows=None):
        # kernels.js:261-284: ties go to the lower index, which torch.argmax also does on the CPU
        return self.logits(rows).argmax(-1).tolist()


def fuse_state_dict(sd, cfg, prefix="model."):
    """HF state_dict -> the engine's fused float layouts (model.js:70-116)."""
    c = cfg
    g = lambda k: sd[prefix + k].float()
    out = {"embed": g("embed_tokens.weight"), "final_norm": g("norm.weight"), "layers": []}
    for l, lt in enumerate(c.layer_types):
        p = f"layers.{l}."
        L = {"in_norm": g(p + "input_layernorm.weight"), "post_norm": g(p + "post_attention_layernorm.weight"),
             "gu": torch.cat([g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight")]),
             "down": g(p + "mlp.down_proj.weight")}
        if lt == "linear_attention":
            a = p + "linear_attn."
            L["proj"] = torch.cat([g(a + "in_proj_qkv.weight"), g(a + "in_proj_z.weight"), g(a + "in_proj_b.weight"),
                                   g(a + "in_proj_a.weight")])
            L["out"] = g(a + "out_proj.weight")
            L["conv"] = g(a + "conv1d.weight").reshape(c.conv_dim, c.ks)
            L["alog"], L["dtb"], L["gnorm"] = g(a + "A_log"), g(a + "dt_bias"), g(a + "norm.weight")
        else:
            a = p + "self_attn."
            L["proj"] = torch.cat([g(a + "q_proj.weight"), g(a + "k_proj.weight"), g(a + "v_proj.weight")])
            L["out"] = g(a + "o_proj.weight")
            L["qnorm"], L["knorm"] = g(a + "q_norm.weight"), g(a + "k_norm.weight")
        out["layers"].append(L)
    return out


def map_weights(weights, fn):
    """Apply fn to every quantised matrix (embed, proj, out, gu, down) of a fused weight dict."""
    out = {"embed": fn(weights["embed"]), "final_norm": weights["final_norm"], "layers": []}
    for L in weights["layers"]:
        L2 = dict(L)
        for k in ("proj", "out", "gu", "down"):
            L2[k] = fn(L[k])
        out["layers"].append(L2)
    return out
