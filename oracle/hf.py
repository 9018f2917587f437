"""Harness around the reference's PyTorch path: Hugging Face transformers' Qwen3.5 in fp32 on the CPU.

Test infrastructure only.  The reference's golden generator and tools drive this module with forward hooks
(tests/engine_ref.py:4-20, 49-53; tools/find_steering.py:104-114; tools/find_scales.py:47-54); this file builds
random-init models of the Qwen3.5-0.8B shape (no checkpoint is available offline) and installs the same hooks, with
per-row values so a batch can carry a different push or vector in every row.

transformers 5.5.0 is the version in this image (the reference pins 5.22.1 only for its Modal jobs,
tools/shapes/modal_app.py:15).  The fla / causal-conv1d fast paths are forced off so the pure-torch functions
(torch_chunk_gated_delta_rule, torch_recurrent_gated_delta_rule, torch_causal_conv1d_update) run.
"""
import torch

from .model import Cfg


def _modeling():
    import transformers.models.qwen3_5.modeling_qwen3_5 as m
    m.FusedRMSNormGated = None
    m.chunk_gated_delta_rule = None
    m.fused_recurrent_gated_delta_rule = None
    m.causal_conv1d_fn = None
    m.causal_conv1d_update = None
    return m


def hf_config(cfg: Cfg):
    from transformers import Qwen3_5TextConfig
    return Qwen3_5TextConfig(
        vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.inter, num_hidden_layers=cfg.layers,
        num_attention_heads=cfg.nh, num_key_value_heads=cfg.nkv, head_dim=cfg.hd, linear_num_key_heads=cfg.hk,
        linear_num_value_heads=cfg.hv, linear_key_head_dim=cfg.dk, linear_value_head_dim=cfg.dv,
        linear_conv_kernel_dim=cfg.ks, rms_norm_eps=cfg.eps, tie_word_embeddings=True, layer_types=cfg.layer_types,
        rope_parameters={"rope_type": "default", "rope_theta": cfg.theta,
                         "partial_rotary_factor": cfg.rot / cfg.hd, "mrope_section": [11, 11, 10]})


def build_model(cfg: Cfg, seed=0):
    """Random-init Qwen3_5ForCausalLM under torch.manual_seed(seed): Linear/Embedding/conv N(0, 0.02), RMSNorm
    weights 0 (applied as 1 + w), gated-norm weight 1, dt_bias 1, A_log = log U(0, 16) ([HF] 801-812)."""
    m = _modeling()
    torch.manual_seed(seed)
    model = m.Qwen3_5ForCausalLM(hf_config(cfg)).eval()
    model.config._attn_implementation = "eager"
    return model


def build_model_fast(cfg: Cfg, seed=0):
    """Same model and distributions as build_model, initialised directly with torch's vectorised samplers (seconds
    instead of a minute at the 0.8B shape); the random stream differs from build_model's.  Used for timing only."""
    m = _modeling()
    with torch.device("meta"):
        model = m.Qwen3_5ForCausalLM(hf_config(cfg))
    model = model.to_empty(device="cpu").eval()
    model.config._attn_implementation = "eager"
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("A_log"):
                p.copy_(torch.empty(p.shape).uniform_(0, 16, generator=g).log())
            elif name.endswith("dt_bias") or name.endswith("linear_attn.norm.weight"):
                p.fill_(1.0)
            elif p.ndim == 1:
                p.zero_()
            else:
                p.normal_(0.0, 0.02, generator=g)
        # non-persistent buffers are left uninitialised by to_empty: recompute the rotary table
        emb = model.model.rotary_emb
        inv, _ = emb.compute_default_rope_parameters(emb.config)
        emb.inv_freq.copy_(inv)
        emb.original_inv_freq.copy_(inv)
    model.tie_weights()
    return model


class Hooks:
    """Push hooks at every down_proj input and a vec hook at every layer output, with per-batch-row values.

    push: {layer: [(neuron or None, "add"|"mul", tensor[B])]}; vec: (layer, tensor[B, H]) or None."""

    def __init__(self, model):
        self.push = {}
        self.vec = None
        self.handles = []
        layers = model.model.layers
        for i, layer in enumerate(layers):
            self.handles.append(layer.mlp.down_proj.register_forward_pre_hook(self._pre(i)))
            self.handles.append(layer.register_forward_hook(self._post(i)))

    def _pre(self, i):
        def f(mod, inp):
            if i not in self.push:
                return None
            h = inp[0].clone()
            for n, mode, vals in self.push[i]:
                v = vals.to(h.dtype)[:, None]
                if n is None:
                    h = h * v[..., None] if mode == "mul" else h + v[..., None]
                elif mode == "mul":
                    h[..., n] = h[..., n] * v
                else:
                    h[..., n] = h[..., n] + v
            return (h,)
        return f

    def _post(self, i):
        def f(mod, inp, out):
            if self.vec is None or self.vec[0] != i:
                return None
            add = self.vec[1][:, None, :].to(torch.float32)
            return ((out[0] + add,) + tuple(out[1:])) if isinstance(out, tuple) else out + add
        return f

    def remove(self):
        for h in self.handles:
            h.remove()


@torch.inference_mode()
def prefill_and_greedy(model, ids, n_new, hooks=None, push=None, vec=None):
    """Prefill a [B, T] batch through the HF cache path, then n_new greedy steps (argmax, lowest index on ties).

    Returns (prefill last-token logits [B, V], list of per-step logits [B, V], tokens [B, n_new])."""
    from transformers import DynamicCache
    if hooks is not None:
        hooks.push = push or {}
        hooks.vec = vec
    ids = torch.as_tensor(ids)
    cache = DynamicCache(config=model.config)
    out = model(input_ids=ids, past_key_values=cache, use_cache=True)
    cache = out.past_key_values
    first = out.logits[:, -1].float().clone()
    lg = first
    toks, step_logits = [], []
    for _ in range(n_new):
        nxt = lg.argmax(-1)
        toks.append(nxt)
        out = model(input_ids=nxt[:, None], past_key_values=cache, use_cache=True)
        cache = out.past_key_values
        lg = out.logits[:, -1].float().clone()
        step_logits.append(lg)
    if hooks is not None:
        hooks.push, hooks.vec = {}, None
    return first, step_logits, (torch.stack(toks, 1) if toks else torch.zeros(ids.shape[0], 0, dtype=torch.long))
