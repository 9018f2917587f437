"""Checkpoint loading: safetensors files (bf16 / f16 / f32) -> the engine's fused int8 layouts, quantised on the GPU
while the file streams through a fixed-size stage, plus an on-disk int8 pack that later runs load without
quantising again.

The host-side mirror of the reference's loader (engine/model.js:60-306): `plan` is its _plan (where every checkpoint
tensor lands: a row range of a fused int8 matrix, or a small f32 tensor), `load_checkpoint` its _stream (tensors in
file order, rows moved in stages of at most 16 MB, each stage quantised by the library's quantiser straight into its
rows of the destination), `save_pack` / `load_pack` its Cache Storage (_saveCache / _loadCached; a safetensors file
here, since there is no browser).  Works for one file or a list of shards.
"""
import ctypes as C
import json
import os
import struct

import numpy as np
import torch

from . import lib as L
from .config import Config
from .weights import Q8, Weights

DTYPES = {"BF16": (torch.bfloat16, 2, L.DUO_BF16), "F16": (torch.float16, 2, L.DUO_F16),
          "F32": (torch.float32, 4, L.DUO_F32), "I8": (torch.int8, 1, None)}
NAMES = {v[0]: k for k, v in DTYPES.items()}
PACK_FORMAT = "duo-q8"
PACK_VERSION = "1"


# ---------------------------------------------------------------------------------------------------------------
# safetensors: 8-byte little-endian header length, a JSON header {name: {dtype, shape, data_offsets}}, the data


def read_header(path):
    """(header without __metadata__, metadata dict, byte offset of the data) of a safetensors file."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        if n > 1 << 28:
            raise ValueError(f"{path}: implausible safetensors header length {n}")
        header = json.loads(f.read(n).decode("utf-8"))
    meta = header.pop("__metadata__", {}) or {}
    return header, meta, 8 + n


def write_safetensors(path, tensors, metadata=None):
    """Write CPU tensors (dtypes of DTYPES) as one safetensors file, in the order given."""
    header, off = {}, 0
    for name, t in tensors.items():
        nbytes = t.numel() * t.element_size()
        header[name] = {"dtype": NAMES[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + nbytes]}
        off += nbytes
    if metadata:
        header["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    hb = json.dumps(header, separators=(",", ":")).encode("utf-8")
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for t in tensors.values():
            t = t.contiguous()
            f.write((t.view(torch.int16) if t.element_size() == 2 else t).numpy().tobytes())


# ---------------------------------------------------------------------------------------------------------------
# where each checkpoint tensor goes (model.js:68-114)


def matrix_shapes(cfg: Config):
    """{key: (rows, cols)} of the fused int8 matrices; keys "embed" and (layer, "proj" | "out" | "gu" | "down")."""
    H, I = cfg.hidden_size, cfg.intermediate_size
    out = {"embed": (cfg.vocab_size, H)}
    for l in range(cfg.num_hidden_layers):
        full = cfg.is_full(l)
        out[(l, "proj")] = (cfg.w_full if full else cfg.w_lin, H)
        out[(l, "out")] = (H, cfg.num_attention_heads * cfg.head_dim if full else cfg.value_dim)
        out[(l, "gu")] = (2 * I, H)
        out[(l, "down")] = (H, I)
    return out


def plan(cfg: Config, prefix="model.language_model."):
    """{checkpoint name: ("q", matrix key, first row) | ("f", (layer or None, small-tensor key))}."""
    c, p = cfg, prefix
    out = {p + "embed_tokens.weight": ("q", "embed", 0), p + "norm.weight": ("f", (None, "final_norm"))}
    for l in range(c.num_hidden_layers):
        lp = f"{p}layers.{l}."
        out[lp + "input_layernorm.weight"] = ("f", (l, "in_norm"))
        out[lp + "post_attention_layernorm.weight"] = ("f", (l, "post_norm"))
        out[lp + "mlp.gate_proj.weight"] = ("q", (l, "gu"), 0)
        out[lp + "mlp.up_proj.weight"] = ("q", (l, "gu"), c.intermediate_size)
        out[lp + "mlp.down_proj.weight"] = ("q", (l, "down"), 0)
        if c.is_full(l):
            a = lp + "self_attn."
            qd = c.num_attention_heads * 2 * c.head_dim
            out[a + "q_proj.weight"] = ("q", (l, "proj"), 0)
            out[a + "k_proj.weight"] = ("q", (l, "proj"), qd)
            out[a + "v_proj.weight"] = ("q", (l, "proj"), qd + c.num_key_value_heads * c.head_dim)
            out[a + "o_proj.weight"] = ("q", (l, "out"), 0)
            out[a + "q_norm.weight"] = ("f", (l, "q_norm"))
            out[a + "k_norm.weight"] = ("f", (l, "k_norm"))
        else:
            a = lp + "linear_attn."
            out[a + "in_proj_qkv.weight"] = ("q", (l, "proj"), 0)
            out[a + "in_proj_z.weight"] = ("q", (l, "proj"), c.conv_dim)
            out[a + "in_proj_b.weight"] = ("q", (l, "proj"), c.conv_dim + c.value_dim)
            out[a + "in_proj_a.weight"] = ("q", (l, "proj"), c.conv_dim + c.value_dim + c.linear_num_value_heads)
            out[a + "out_proj.weight"] = ("q", (l, "out"), 0)
            out[a + "conv1d.weight"] = ("f", (l, "conv"))
            out[a + "A_log"] = ("f", (l, "a_log"))
            out[a + "dt_bias"] = ("f", (l, "dt_bias"))
            out[a + "norm.weight"] = ("f", (l, "gnorm"))
    return out


def detect_prefix(names):
    """The decoder's name prefix in a checkpoint: Qwen3.5 image-text checkpoints nest it (model.language_model.),
    text-only ones do not (model.)."""
    for p in ("model.language_model.", "model."):
        if p + "embed_tokens.weight" in names:
            return p
    raise ValueError("checkpoint has no embed_tokens.weight under model.language_model. or model.")


def _locate(paths, cfg, prefix):
    """Every planned tensor's (file, header entry, data offset); raises on the missing ones (model.js:184-185)."""
    where = {}
    for path in paths:
        header, _, base = read_header(path)
        for name, ent in header.items():
            where[name] = (path, ent, base)
    prefix = prefix or detect_prefix(where)
    pl = plan(cfg, prefix)
    missing = [k for k in pl if k not in where]
    if missing:
        raise ValueError("checkpoint is missing " + ", ".join(missing[:3]) + (" ..." if len(missing) > 3 else ""))
    return pl, where


# ---------------------------------------------------------------------------------------------------------------
# loading


def _empty_weights(cfg: Config, device):
    W = Weights(cfg)
    shapes = matrix_shapes(cfg)

    def q8(key):
        rows, cols = shapes[key]
        g = cfg.group or cols
        if cols % g:
            raise ValueError(f"{key}: {cols} columns are not a multiple of the group size {g}")
        return Q8(torch.empty(rows, cols, dtype=torch.int8, device=device),
                  torch.empty(rows, cols // g, dtype=torch.float32, device=device))

    W.embed = q8("embed")
    W.layers = [{"proj": q8((l, "proj")), "out": q8((l, "out")), "gu": q8((l, "gu")), "down": q8((l, "down"))}
                for l in range(cfg.num_hidden_layers)]
    return W


def _set_small(W, cfg, key, t):
    layer, name = key
    if layer is None:
        W.final_norm = t
        return
    if name == "conv":
        t = t.reshape(cfg.conv_dim, cfg.linear_conv_kernel_dim)
    W.layers[layer][name] = t.contiguous()


def load_checkpoint(paths, cfg: Config, prefix=None, device="cuda", stage_bytes=16 << 20):
    """Quantise a safetensors checkpoint (one path or a list of shards) into the engine's fused int8 layouts on
    `device`.  Matrices move in file order through a pinned host stage and a device stage of `stage_bytes`, whole
    rows at a time, and each stage is quantised (duo_q8_quantize, group cfg.group or one scale per row) straight into
    its rows of the destination -- the checkpoint is never held whole in memory (model.js:153-230)."""
    paths = [paths] if isinstance(paths, (str, os.PathLike)) else list(paths)
    pl, where = _locate(paths, cfg, prefix)
    W = _empty_weights(cfg, device)
    shapes = matrix_shapes(cfg)
    host = torch.empty(stage_bytes, dtype=torch.uint8, pin_memory=True)
    dev = torch.empty(stage_bytes, dtype=torch.uint8, device=device)
    st = L.stream_ptr(None)  # torch's current stream, which the staging copies use too
    todo = sorted(pl.items(), key=lambda kv: (where[kv[0]][0], where[kv[0]][1]["data_offsets"][0]))
    files = {}
    try:
        for name, dst in todo:
            path, ent, base = where[name]
            f = files.get(path) or files.setdefault(path, open(path, "rb"))
            if ent["dtype"] not in DTYPES or ent["dtype"] == "I8":
                raise ValueError(f"{name}: unsupported dtype {ent['dtype']}")
            tdt, es, code = DTYPES[ent["dtype"]]
            s0, s1 = ent["data_offsets"]
            shape = ent["shape"]
            f.seek(base + s0)
            if dst[0] == "f":
                raw = np.frombuffer(f.read(s1 - s0), dtype=np.uint8).copy()
                t = torch.from_numpy(raw).view(tdt).reshape(shape).to(torch.float32)
                _set_small(W, cfg, dst[1], t.to(device))
                continue
            key, row0 = dst[1], dst[2]
            q8 = W.embed if key == "embed" else W.layers[key[0]][key[1]]
            rows_total, cols_total = shapes[key]
            cols = shape[-1]
            rows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
            if cols != cols_total or row0 + rows > rows_total:
                raise ValueError(f"{name}: shape {shape} does not fit rows {row0}.. of a {rows_total} x {cols_total} "
                                 "fused matrix")
            g = cfg.group or cols
            row_bytes = cols * es
            per = max(1, stage_bytes // row_bytes)
            if per * row_bytes > stage_bytes:
                raise ValueError(f"{name}: one row ({row_bytes} bytes) exceeds the {stage_bytes}-byte stage")
            for r in range(0, rows, per):
                n = min(per, rows - r)
                nb = n * row_bytes
                torch.cuda.current_stream().synchronize()  # the stage's previous rows are quantised
                got = f.readinto(memoryview(host.numpy())[:nb])
                if got != nb:
                    raise ValueError(f"{name}: checkpoint ended early")
                dev[:nb].copy_(host[:nb], non_blocking=True)
                qp = q8.q.data_ptr() + (row0 + r) * cols
                sp = q8.s.data_ptr() + (row0 + r) * (cols // g) * 4
                L.call("duo_q8_quantize", C.c_void_p(dev.data_ptr()), code, n, cols, g, C.c_void_p(qp),
                       C.c_void_p(sp), st)
    finally:
        for f in files.values():
            f.close()
    torch.cuda.synchronize()
    return W


# ---------------------------------------------------------------------------------------------------------------
# the int8 pack (the reference keeps its quantised weights in the browser's Cache Storage, model.js:232-280)

_SMALL = ("in_norm", "post_norm", "conv", "a_log", "dt_bias", "gnorm", "q_norm", "k_norm")


def save_pack(weights: Weights, path):
    """Write the quantised weights (int8 matrices, f32 scales, small f32 tensors) as one safetensors file; the group
    size and the layer types go to its metadata."""
    cfg = weights.cfg
    t = {"embed.q": weights.embed.q.cpu(), "embed.s": weights.embed.s.cpu(), "final_norm": weights.final_norm.cpu()}
    for l, Ly in enumerate(weights.layers):
        for k in ("proj", "out", "gu", "down"):
            t[f"layers.{l}.{k}.q"] = Ly[k].q.cpu()
            t[f"layers.{l}.{k}.s"] = Ly[k].s.cpu()
        for k in _SMALL:
            if k in Ly:
                t[f"layers.{l}.{k}"] = Ly[k].float().cpu()
    write_safetensors(path, t, {"format": PACK_FORMAT, "version": PACK_VERSION, "group": cfg.group,
                                "layer_types": json.dumps(cfg.layer_types)})


def load_pack(path, cfg: Config, device="cuda"):
    """Read a pack written by save_pack for the same configuration and group size (no quantisation)."""
    header, meta, base = read_header(path)
    if meta.get("format") != PACK_FORMAT or meta.get("version") != PACK_VERSION:
        raise ValueError(f"{path}: not a {PACK_FORMAT} v{PACK_VERSION} pack")
    if int(meta.get("group", -1)) != cfg.group:
        raise ValueError(f"{path}: packed with group {meta.get('group')}, the configuration asks for {cfg.group}")
    if json.loads(meta.get("layer_types", "[]")) != list(cfg.layer_types):
        raise ValueError(f"{path}: packed for other layer types")
    with open(path, "rb") as f:
        def get(name):
            ent = header[name]
            tdt = DTYPES[ent["dtype"]][0]
            f.seek(base + ent["data_offsets"][0])
            raw = np.frombuffer(f.read(ent["data_offsets"][1] - ent["data_offsets"][0]), dtype=np.uint8).copy()
            return torch.from_numpy(raw).view(tdt).reshape(ent["shape"]).to(device)

        W = Weights(cfg)
        shapes = matrix_shapes(cfg)
        W.embed = Q8(get("embed.q"), get("embed.s"))
        if tuple(W.embed.q.shape) != shapes["embed"]:
            raise ValueError(f"{path}: embed is {tuple(W.embed.q.shape)}, the configuration needs {shapes['embed']}")
        W.final_norm = get("final_norm")
        for l in range(cfg.num_hidden_layers):
            Ly = {}
            for k in ("proj", "out", "gu", "down"):
                Ly[k] = Q8(get(f"layers.{l}.{k}.q"), get(f"layers.{l}.{k}.s"))
                if tuple(Ly[k].q.shape) != shapes[(l, k)]:
                    raise ValueError(f"{path}: layer {l} {k} has shape {tuple(Ly[k].q.shape)}")
            for k in _SMALL:
                if f"layers.{l}.{k}" in header:
                    Ly[k] = get(f"layers.{l}.{k}")
            W.layers.append(Ly)
    torch.cuda.synchronize()
    return W
