"""Model configuration.  Field names follow transformers' Qwen3_5TextConfig, which the reference's engine reads from
the checkpoint's config.json (engine/model.js:27-58)."""
from dataclasses import dataclass, field
from typing import List, Optional


@dataclass
class Config:
    hidden_size: int = 1024
    intermediate_size: int = 3584
    vocab_size: int = 248320
    num_hidden_layers: int = 24
    num_attention_heads: int = 8
    num_key_value_heads: int = 2
    head_dim: int = 256
    partial_rotary_factor: float = 0.25
    rope_theta: float = 1e7
    linear_num_key_heads: int = 16
    linear_num_value_heads: int = 16
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_conv_kernel_dim: int = 4
    rms_norm_eps: float = 1e-6
    layer_types: Optional[List[str]] = None
    full_attention_interval: int = 4
    # engine options (not in the HF config): int8 group size along K (128 = the reference's q8 format, 0 = one
    # scale per output row) and the activation dtype: "f32" = the reference's precision (CUDA cores), "bf16" or
    # "f16" = the tensor-core path with 16-bit activations (f16 keeps 3 more mantissa bits, bf16 more range)
    group: int = 128
    act_dtype: str = "bf16"

    def __post_init__(self):
        if self.layer_types is None:
            self.layer_types = ["full_attention" if (i + 1) % self.full_attention_interval == 0 else "linear_attention"
                                for i in range(self.num_hidden_layers)]
        if len(self.layer_types) != self.num_hidden_layers:
            raise ValueError("layer_types must have num_hidden_layers entries")
        if self.act_dtype not in ("f32", "bf16", "f16"):
            raise ValueError("act_dtype must be 'f32', 'bf16' or 'f16'")

    # derived sizes (engine/model.js:44-54)
    @property
    def rot(self):
        return int(round(self.head_dim * self.partial_rotary_factor))

    @property
    def key_dim(self):
        return self.linear_num_key_heads * self.linear_key_head_dim

    @property
    def value_dim(self):
        return self.linear_num_value_heads * self.linear_value_head_dim

    @property
    def conv_dim(self):
        return 2 * self.key_dim + self.value_dim

    @property
    def w_lin(self):
        return self.conv_dim + self.value_dim + 2 * self.linear_num_value_heads

    @property
    def w_full(self):
        return self.num_attention_heads * 2 * self.head_dim + 2 * self.num_key_value_heads * self.head_dim

    def is_full(self, l):
        return self.layer_types[l] == "full_attention"

    @classmethod
    def from_hf(cls, hf, **engine_opts):
        """From a transformers Qwen3_5TextConfig / Qwen3_5Config (or its dict)."""
        d = hf if isinstance(hf, dict) else hf.to_dict()
        d = d.get("text_config", d) or d
        rp = d.get("rope_parameters") or {}
        return cls(hidden_size=d["hidden_size"], intermediate_size=d["intermediate_size"], vocab_size=d["vocab_size"],
                   num_hidden_layers=d["num_hidden_layers"], num_attention_heads=d["num_attention_heads"],
                   num_key_value_heads=d["num_key_value_heads"], head_dim=d.get("head_dim", 256),
                   partial_rotary_factor=rp.get("partial_rotary_factor", d.get("partial_rotary_factor", 1.0)),
                   rope_theta=rp.get("rope_theta", d.get("rope_theta", 1e7)),
                   linear_num_key_heads=d["linear_num_key_heads"], linear_num_value_heads=d["linear_num_value_heads"],
                   linear_key_head_dim=d["linear_key_head_dim"], linear_value_head_dim=d["linear_value_head_dim"],
                   linear_conv_kernel_dim=d["linear_conv_kernel_dim"], rms_norm_eps=d["rms_norm_eps"],
                   layer_types=list(d["layer_types"]), **engine_opts)


def qwen35_0p8b(**kw):
    """The Qwen3.5-0.8B text decoder shape (README.md:94 of the reference: 24 layers, 18 DeltaNet + 6 attention)."""
    return Config(**kw)
