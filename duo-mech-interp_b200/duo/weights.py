"""Weights in the reference engine's fused int8 layouts (engine/model.js:70-116), quantised on the GPU by the CUDA
quantiser (the reference quantises while streaming the checkpoint, model.js:153-230).

  linear-attention layer: proj = [in_proj_qkv | in_proj_z | in_proj_b | in_proj_a]   (w_lin x hidden)
  full-attention layer:   proj = [q_proj (q and gate interleaved per head) | k_proj | v_proj]   (w_full x hidden)
  every layer:            gu = [gate_proj | up_proj] (2 inter x hidden), down, out
  embed (tied LM head), final norm; f32: norms, conv1d, A_log, dt_bias, gated-norm weight, q/k norms.
"""
import ctypes as C

import torch

from . import ops
from .config import Config
from .lib import duo_layer_view, duo_q8_view, duo_weights_view


class Q8:
    __slots__ = ("q", "s")

    def __init__(self, q, s):
        self.q, self.s = q, s

    def view(self):
        return duo_q8_view(self.q.data_ptr(), self.s.data_ptr())


class Weights:
    """Device tensors of one model, and the C views the engine reads."""

    def __init__(self, cfg: Config):
        self.cfg = cfg
        self.embed = None
        self.final_norm = None
        self.layers = []

    def c_view(self):
        n = self.cfg.num_hidden_layers
        arr = (duo_layer_view * n)()
        for l, L in enumerate(self.layers):
            v = arr[l]
            v.in_norm, v.post_norm = L["in_norm"].data_ptr(), L["post_norm"].data_ptr()
            v.proj, v.out, v.gu, v.down = L["proj"].view(), L["out"].view(), L["gu"].view(), L["down"].view()
            if self.cfg.is_full(l):
                v.q_norm, v.k_norm = L["q_norm"].data_ptr(), L["k_norm"].data_ptr()
            else:
                v.conv, v.a_log, v.dt_bias, v.gnorm = (L["conv"].data_ptr(), L["a_log"].data_ptr(),
                                                       L["dt_bias"].data_ptr(), L["gnorm"].data_ptr())
        self._arr = arr  # keep alive for the call
        return duo_weights_view(self.embed.view(), self.final_norm.data_ptr(), C.cast(arr, C.c_void_p))

    def dequantized(self):
        """Float copies of every matrix (f32(q) * scale), in the fused layouts: the inputs the parity oracle runs on."""
        dq = lambda w: ops.q8_dequantize(w.q, w.s, torch.float32)
        out = {"embed": dq(self.embed), "final_norm": self.final_norm, "layers": []}
        for L in self.layers:
            d = {k: (dq(v) if isinstance(v, Q8) else v) for k, v in L.items()}
            if "q_norm" in d:
                d["qnorm"], d["knorm"] = d.pop("q_norm"), d.pop("k_norm")
            if "a_log" in d:
                d["alog"], d["dtb"] = d.pop("a_log"), d.pop("dt_bias")
            out["layers"].append(d)
        return out


def _q(w, group):
    return Q8(*ops.q8_quantize(w.contiguous(), group))


def from_state_dict(sd, cfg: Config, device="cuda", prefix="model."):
    """Quantise an HF-layout state_dict (float tensors, CPU or GPU) into the fused int8 layouts on `device`."""
    g = cfg.group
    get = lambda k: sd[prefix + k].to(device=device, dtype=torch.float32)
    W = Weights(cfg)
    W.embed = _q(get("embed_tokens.weight"), g)
    W.final_norm = get("norm.weight").contiguous()
    for l in range(cfg.num_hidden_layers):
        p = f"layers.{l}."
        L = {"in_norm": get(p + "input_layernorm.weight").contiguous(),
             "post_norm": get(p + "post_attention_layernorm.weight").contiguous(),
             "gu": _q(torch.cat([get(p + "mlp.gate_proj.weight"), get(p + "mlp.up_proj.weight")]), g),
             "down": _q(get(p + "mlp.down_proj.weight"), g)}
        if cfg.is_full(l):
            a = p + "self_attn."
            L["proj"] = _q(torch.cat([get(a + "q_proj.weight"), get(a + "k_proj.weight"), get(a + "v_proj.weight")]), g)
            L["out"] = _q(get(a + "o_proj.weight"), g)
            L["q_norm"], L["k_norm"] = get(a + "q_norm.weight").contiguous(), get(a + "k_norm.weight").contiguous()
        else:
            a = p + "linear_attn."
            L["proj"] = _q(torch.cat([get(a + "in_proj_qkv.weight"), get(a + "in_proj_z.weight"),
                                      get(a + "in_proj_b.weight"), get(a + "in_proj_a.weight")]), g)
            L["out"] = _q(get(a + "out_proj.weight"), g)
            L["conv"] = get(a + "conv1d.weight").reshape(cfg.conv_dim, cfg.linear_conv_kernel_dim).contiguous()
            L["a_log"], L["dt_bias"] = get(a + "A_log").contiguous(), get(a + "dt_bias").contiguous()
            L["gnorm"] = get(a + "norm.weight").contiguous()
        W.layers.append(L)
    torch.cuda.synchronize()
    return W


def random_weights(cfg: Config, seed=0, device="cuda", std=0.02):
    """Random-init weights with the distributions of transformers' Qwen3.5 init, generated on the GPU (seeded):
    matrices and conv N(0, std), RMSNorm weights 0 (applied as 1 + w), gated-norm weight 1, dt_bias 1,
    A_log = log U(0, 16).  Used for the throughput configs, where the HF CPU init of 752 M parameters is too slow."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    H, I = cfg.hidden_size, cfg.intermediate_size
    g = cfg.group

    def mat(n, k):
        w = torch.empty(n, k, device=device, dtype=torch.float32)
        w.normal_(0.0, std, generator=gen)
        return _q(w, g)

    W = Weights(cfg)
    W.embed = mat(cfg.vocab_size, H)
    W.final_norm = torch.zeros(H, device=device)
    for l in range(cfg.num_hidden_layers):
        L = {"in_norm": torch.zeros(H, device=device), "post_norm": torch.zeros(H, device=device),
             "gu": mat(2 * I, H), "down": mat(H, I)}
        if cfg.is_full(l):
            L["proj"] = mat(cfg.w_full, H)
            L["out"] = mat(H, cfg.num_attention_heads * cfg.head_dim)
            L["q_norm"] = torch.zeros(cfg.head_dim, device=device)
            L["k_norm"] = torch.zeros(cfg.head_dim, device=device)
        else:
            hv = cfg.linear_num_value_heads
            L["proj"] = mat(cfg.w_lin, H)
            L["out"] = mat(H, cfg.value_dim)
            conv = torch.empty(cfg.conv_dim, cfg.linear_conv_kernel_dim, device=device)
            conv.normal_(0.0, std, generator=gen)
            L["conv"] = conv
            u = torch.empty(hv, device=device).uniform_(0, 16, generator=gen)
            L["a_log"] = torch.log(u)
            L["dt_bias"] = torch.ones(hv, device=device)
            L["gnorm"] = torch.ones(cfg.linear_value_head_dim, device=device)
        W.layers.append(L)
    torch.cuda.synchronize()
    return W


def param_bytes(cfg: Config):
    """int8 bytes of every quantised matrix (the weight stream of one full decode step, embed = LM head)."""
    H, I = cfg.hidden_size, cfg.intermediate_size
    n = cfg.vocab_size * H
    for l in range(cfg.num_hidden_layers):
        n += 2 * I * H + H * I
        n += (cfg.w_full * H + H * cfg.num_attention_heads * cfg.head_dim) if cfg.is_full(l) else \
            (cfg.w_lin * H + H * cfg.value_dim)
    return n


def flops_per_token(cfg: Config):
    """2 x the layer matmul parameters (the LM head is counted separately, it only runs on last tokens)."""
    return 2 * (param_bytes(cfg) - cfg.vocab_size * cfg.hidden_size)

