"""The checkpoint loader (duo.checkpoint, the mirror of engine/model.js:60-306): the safetensors format, the plan of
where every tensor of a Qwen3.5 checkpoint lands in the fused layouts, missing-tensor errors, and (GPU) a checkpoint
written here in bf16 and in f32, split over two shards, quantised in small stages into exactly the bytes that
quantising whole tensors gives, an int8 pack that reloads identically, and the engine's logits on it."""
import json

import pytest
import torch

from tiny import TINY, tiny_state_dict


def _cfg(types, group=128, act="f32"):
    from duo import Config
    c = TINY
    return Config(hidden_size=c["hidden"], intermediate_size=c["inter"], vocab_size=c["vocab"],
                  num_hidden_layers=c["layers"], num_attention_heads=c["nh"], num_key_value_heads=c["nkv"],
                  head_dim=c["hd"], partial_rotary_factor=c["rot"] / c["hd"], rope_theta=c["theta"],
                  linear_num_key_heads=c["hk"], linear_num_value_heads=c["hv"], linear_key_head_dim=c["dk"],
                  linear_value_head_dim=c["dv"], linear_conv_kernel_dim=c["ks"], rms_norm_eps=c["eps"],
                  layer_types=types, group=group, act_dtype=act)


def _write(tmp_path, sd, dtype, prefix="model.language_model.", shards=2):
    from duo.checkpoint import write_safetensors
    names = list(sd)
    paths = []
    for i in range(shards):
        part = {prefix + k[len("model."):]: torch.from_numpy(sd[k]).to(dtype) for k in names[i::shards]}
        p = tmp_path / f"model-{i}.safetensors"
        write_safetensors(p, part)
        paths.append(str(p))
    return paths


def test_safetensors_round_trip(tmp_path):
    from duo.checkpoint import read_header, write_safetensors
    t = {"a": torch.arange(6, dtype=torch.float32).reshape(2, 3), "b": torch.tensor([1.5, -2.0], dtype=torch.bfloat16),
         "c": torch.tensor([[-3, 4]], dtype=torch.int8)}
    write_safetensors(tmp_path / "x.safetensors", t, {"k": 1})
    header, meta, base = read_header(tmp_path / "x.safetensors")
    assert meta == {"k": "1"} and base % 8 == 0
    assert header["b"] == {"dtype": "BF16", "shape": [2], "data_offsets": [24, 28]}
    raw = (tmp_path / "x.safetensors").read_bytes()[base:]
    assert torch.equal(torch.frombuffer(bytearray(raw[0:24]), dtype=torch.float32).reshape(2, 3), t["a"])


def test_plan_covers_every_tensor_of_a_qwen35_checkpoint():
    from duo import qwen35_0p8b
    from duo.checkpoint import matrix_shapes, plan
    cfg = qwen35_0p8b()
    pl = plan(cfg)
    n_lin = sum(1 for l in range(24) if not cfg.is_full(l))
    assert len(pl) == 2 + 24 * 5 + n_lin * 9 + (24 - n_lin) * 6
    # the row ranges of each fused matrix tile it exactly (model.js:70-116)
    rows = {}
    for name, d in pl.items():
        if d[0] == "q":
            rows.setdefault(d[1], []).append(d[2])
    shapes = matrix_shapes(cfg)
    assert sorted(rows[(0, "proj")]) == [0, cfg.conv_dim, cfg.conv_dim + cfg.value_dim,
                                         cfg.conv_dim + cfg.value_dim + 16]
    assert sorted(rows[(3, "proj")]) == [0, 8 * 512, 8 * 512 + 512]
    assert shapes[(3, "proj")] == (5120, 1024) and shapes[(0, "proj")] == (8224, 1024)


def test_missing_tensor_is_reported(tmp_path):
    from duo.checkpoint import _locate
    sd, types = tiny_state_dict()
    sd.pop("model.layers.2.mlp.down_proj.weight")
    paths = _write(tmp_path, sd, torch.float32, prefix="model.", shards=1)
    with pytest.raises(ValueError, match="down_proj"):
        _locate(paths, _cfg(types), None)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,group", [(torch.bfloat16, 128), (torch.float32, 0)])
def test_load_checkpoint_matches_whole_tensor_quantisation(cuda, tmp_path, dtype, group):
    from duo import Model, from_state_dict
    from duo.checkpoint import load_checkpoint, load_pack, save_pack
    sd, types = tiny_state_dict()
    cfg = _cfg(types, group)
    paths = _write(tmp_path, sd, dtype)
    # stages of 8 KiB: every matrix is quantised in several pieces
    W = load_checkpoint(paths, cfg, stage_bytes=8192)
    ref = from_state_dict({k: torch.from_numpy(v).to(dtype).float() for k, v in sd.items()}, cfg)
    pairs = [(W.embed, ref.embed)] + [(W.layers[l][k], ref.layers[l][k]) for l in range(cfg.num_hidden_layers)
                                      for k in ("proj", "out", "gu", "down")]
    for a, b in pairs:
        assert torch.equal(a.q, b.q) and torch.equal(a.s, b.s)
    for l in range(cfg.num_hidden_layers):
        for k, v in ref.layers[l].items():
            if not hasattr(v, "q"):
                assert torch.equal(W.layers[l][k], v), (l, k)
    pack = tmp_path / "pack.safetensors"
    save_pack(W, pack)
    W2 = load_pack(pack, cfg)
    assert torch.equal(W2.embed.q, W.embed.q) and torch.equal(W2.layers[3]["down"].s, W.layers[3]["down"].s)
    ids = torch.randint(0, TINY["vocab"], (2, 9), generator=torch.Generator().manual_seed(2))
    out = []
    for w in (W, W2, ref):
        m = Model(cfg, w).alloc(rows=2, max_len=16, max_t=16, max_tokens=32)
        m.forward(ids.reshape(-1), 0, 2, 9)
        out.append(m.logits_all().cpu())
    assert torch.equal(out[0], out[1]) and torch.equal(out[0], out[2])
    with pytest.raises(ValueError, match="group"):
        load_pack(pack, _cfg(types, 128 if group == 0 else 0))
