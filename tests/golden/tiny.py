"""A tiny Qwen3.5-shaped model for golden fixtures: real head sizes (dk = dv = 128, hd = 256), small everything else.

Weights come from a numpy PCG64 generator (bit-reproducible on every machine), in Hugging Face state_dict naming, so
the fixture generator can load them into transformers and the tests can rebuild them without transformers.
"""
import numpy as np

TINY = dict(hidden=256, inter=512, vocab=2048, layers=4, nh=2, nkv=1, hd=256, rot=64, theta=1e7, hk=2, hv=2, dk=128,
            dv=128, ks=4, eps=1e-6)


def tiny_state_dict(seed=1234):
    c = TINY
    rng = np.random.Generator(np.random.PCG64(seed))
    n = lambda *s: (rng.standard_normal(s) * 0.02).astype(np.float32)
    small = lambda *s: (rng.standard_normal(s) * 0.1).astype(np.float32)
    H, I = c["hidden"], c["inter"]
    kd, vd = c["hk"] * c["dk"], c["hv"] * c["dv"]
    conv_dim = 2 * kd + vd
    sd = {"model.embed_tokens.weight": n(c["vocab"], H), "model.norm.weight": small(H)}
    types = ["full_attention" if (i + 1) % 4 == 0 else "linear_attention" for i in range(c["layers"])]
    for l, t in enumerate(types):
        p = f"model.layers.{l}."
        sd[p + "input_layernorm.weight"] = small(H)
        sd[p + "post_attention_layernorm.weight"] = small(H)
        sd[p + "mlp.gate_proj.weight"] = n(I, H)
        sd[p + "mlp.up_proj.weight"] = n(I, H)
        sd[p + "mlp.down_proj.weight"] = n(H, I)
        if t == "linear_attention":
            a = p + "linear_attn."
            sd[a + "in_proj_qkv.weight"] = n(conv_dim, H) * 10  # larger mixer inputs exercise the delta rule harder
            sd[a + "in_proj_z.weight"] = n(vd, H) * 10
            sd[a + "in_proj_b.weight"] = n(c["hv"], H) * 10
            sd[a + "in_proj_a.weight"] = n(c["hv"], H) * 10
            sd[a + "out_proj.weight"] = n(H, vd)
            sd[a + "conv1d.weight"] = (rng.standard_normal((conv_dim, 1, c["ks"])) * 0.3).astype(np.float32)
            sd[a + "A_log"] = np.log(rng.uniform(0.5, 16, c["hv"])).astype(np.float32)
            sd[a + "dt_bias"] = (1.0 + small(c["hv"])).astype(np.float32)
            sd[a + "norm.weight"] = (1.0 + small(c["dv"])).astype(np.float32)
        else:
            a = p + "self_attn."
            sd[a + "q_proj.weight"] = n(c["nh"] * 2 * c["hd"], H) * 10
            sd[a + "k_proj.weight"] = n(c["nkv"] * c["hd"], H) * 10
            sd[a + "v_proj.weight"] = n(c["nkv"] * c["hd"], H) * 10
            sd[a + "o_proj.weight"] = n(H, c["nh"] * c["hd"])
            sd[a + "q_norm.weight"] = small(c["hd"])
            sd[a + "k_norm.weight"] = small(c["hd"])
    return sd, types


def tiny_workload(seed=7):
    """3 rows x 20 prompt tokens, a per-row add push, a per-row mul-all push and a residual vector."""
    rng = np.random.Generator(np.random.PCG64(seed))
    ids = rng.integers(0, TINY["vocab"], size=(3, 20)).astype(np.int64)
    vecs = (rng.standard_normal((3, TINY["hidden"])) * 0.3).astype(np.float32)
    push = {2: [{"n": 17, "mode": "add", "vals": [0.5, 0.0, -0.5]}],
            1: [{"n": None, "mode": "mul", "vals": [1.1, 1.0, 0.9]}]}
    return ids, push, 2, vecs
