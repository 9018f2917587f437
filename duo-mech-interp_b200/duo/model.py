"""`Model`: the host-side mirror of the reference engine's Model class (engine/model.js:26-509).

Same operations and argument meaning: alloc(rows, maxLen, maxT), reset(r), setVectors(rows), setHeadScales,
_forward(ids, rowBase, rows, T, opts) with opts = {pushes: {layer: [{n, mode, vals}]}, vec: layer, resid: true |
"attn", residBuf, capture, capLayers, capT, capT0, stopAfter} (model.js:7-12, 404-466; the buffers are CUDA f32
tensors [layers, capT, hidden] and [len(capLayers), capT, inter]), prefill(r, ids, opts) chunked by maxT with capT0
advancing per chunk, step(ids, opts), logitsRow(r), logitsAll(), argmaxAll().  Names are snake_case; errors raise
(the reference throws, model.js:52, 406, 418).  All compute runs in libduo_mixer.so; this file only moves arguments.
"""
import ctypes as C

import numpy as np
import torch

from . import lib as L
from .config import Config
from .weights import Weights


class Model:
    def __init__(self, cfg: Config, weights: Weights, stream=None):
        self.cfg = cfg
        self.weights = weights
        self.stream = stream
        c = cfg
        full = (C.c_uint8 * c.num_hidden_layers)(*[1 if c.is_full(l) else 0 for l in range(c.num_hidden_layers)])
        self._c = L.duo_config(
            hidden=c.hidden_size, inter=c.intermediate_size, vocab=c.vocab_size, layers=c.num_hidden_layers,
            nh=c.num_attention_heads, nkv=c.num_key_value_heads, hd=c.head_dim, rot=c.rot, theta=c.rope_theta,
            eps=c.rms_norm_eps, hk=c.linear_num_key_heads, hv=c.linear_num_value_heads, dk=c.linear_key_head_dim,
            dv=c.linear_value_head_dim, ks=c.linear_conv_kernel_dim, full_attention_host=C.cast(full, C.c_void_p),
            group=c.group, act_dtype={"f32": L.DUO_F32, "bf16": L.DUO_BF16, "f16": L.DUO_F16}[c.act_dtype])
        h = C.c_void_p()
        L.call("duo_engine_create", C.byref(self._c), C.byref(h))
        self._h = h
        view = weights.c_view()
        L.call("duo_engine_load", self._h, C.byref(view), self._s())
        torch.cuda.synchronize()
        self.rows = 0
        self._pushes = {}
        self._ids_pinned = None

    def _s(self):
        return L.stream_ptr(self.stream)

    def close(self):
        if getattr(self, "_h", None):
            L.lib().duo_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- state (model.js:308-376)
    def alloc(self, rows=3, max_len=1024, max_t=128, max_tokens=None):
        """rows independent sequences, max_len cache positions per row, max_t tokens per prefill chunk;
        max_tokens bounds rows * T of one forward call (default max(max_t, rows), as model.js:313 sizes it)."""
        self.max_t = max_t
        self.max_len = max_len
        self.max_tokens = max_tokens or max(max_t, rows)
        L.call("duo_engine_alloc", self._h, rows, max_len, self.max_tokens)
        self.rows = rows
        self._pushes = {}
        return self

    def reset(self, r):
        L.call("duo_engine_reset", self._h, r, self._s())

    def reset_all(self):
        L.call("duo_engine_reset_all", self._h, self._s())

    def capture_resid(self, layer=None):
        """The reference's `resid` option for one layer: later forwards copy the residual stream after `layer` into
        the returned [max_tokens, hidden] f32 tensor (rows of the last call first).  None turns it off."""
        if layer is None:
            L.call("duo_engine_capture_resid", self._h, -1, None)
            self._resid = None
            return None
        self._resid = torch.empty(self.max_tokens, self.cfg.hidden_size, dtype=torch.float32, device="cuda")
        L.call("duo_engine_capture_resid", self._h, int(layer), L.ptr(self._resid))
        return self._resid

    def set_vectors(self, rows):
        """One vector (len hidden) per row, None for zero (model.js:372-376)."""
        H = self.cfg.hidden_size
        buf = np.zeros((self.rows, H), dtype=np.float32)
        for r, v in enumerate(rows):
            if v is not None:
                buf[r] = np.asarray(v.detach().cpu() if torch.is_tensor(v) else v, dtype=np.float32)
        L.call("duo_engine_set_vectors", self._h, buf.ctypes.data_as(C.c_void_p), self.rows, self._s())
        torch.cuda.current_stream().synchronize() if self.stream is None else self.stream.synchronize()

    def set_head_scales(self, scales):
        """{layer: [hv scales]} for linear-attention layers; missing layers get ones (model.js:362-369)."""
        for l in range(self.cfg.num_hidden_layers):
            if self.cfg.is_full(l):
                continue
            s = (scales or {}).get(l)
            arr = None if s is None else np.ascontiguousarray(np.asarray(s, dtype=np.float32))
            L.call("duo_engine_set_head_scales", self._h, l, None if arr is None else arr.ctypes.data_as(C.c_void_p),
                   self._s())

    def _set_pushes(self, pushes):
        pushes = pushes or {}
        for l in set(self._pushes) | set(int(k) for k in pushes):
            recs = pushes.get(l, pushes.get(str(l), []))
            key = tuple((r.get("n"), r.get("mode", "add"), tuple(np.asarray(r["vals"], dtype=np.float32).tolist()))
                        for r in recs)
            if self._pushes.get(l) == key:
                continue
            n = len(recs)
            neu = np.array([L.DUO_ALL_NEURONS if r.get("n") is None else int(r["n"]) for r in recs], dtype=np.int32)
            mode = np.array([L.DUO_PUSH_MUL if r.get("mode") == "mul" else L.DUO_PUSH_ADD for r in recs], dtype=np.int32)
            vals = np.zeros((max(n, 1), self.rows), dtype=np.float32)
            for i, r in enumerate(recs):
                v = np.asarray(r["vals"], dtype=np.float32).reshape(-1)
                vals[i, :] = 1.0 if r.get("mode") == "mul" else 0.0  # rows without a value are untouched
                vals[i, : min(len(v), self.rows)] = v[: self.rows]
            L.call("duo_engine_set_pushes", self._h, l, n, neu.ctypes.data_as(C.c_void_p),
                   mode.ctypes.data_as(C.c_void_p), vals.ctypes.data_as(C.c_void_p), self._s())
            self._pushes[l] = key

    # ---- forward (model.js:404-508)
    def _set_hooks(self, opts):
        """The per-call capture / stopAfter options (model.js:427, 445-461); returns the kinds it turned on."""
        on = []
        cap_t = opts.get("capT")
        t0 = int(opts.get("capT0", 0) or 0)
        if opts.get("resid"):
            kind = L.DUO_CAP_RESID_ATTN if opts["resid"] == "attn" else L.DUO_CAP_RESID
            buf = opts["residBuf"]
            L.call("duo_engine_set_capture", self._h, kind, self.cfg.num_hidden_layers, None, L.ptr(buf),
                   int(cap_t or buf.shape[1]))
            on.append(kind)
        if opts.get("capture") is not None:
            buf = opts["capture"]
            layers = opts.get("capLayers")
            arr = None if layers is None else np.ascontiguousarray(np.asarray(layers, dtype=np.int32))
            n = self.cfg.num_hidden_layers if layers is None else len(layers)
            L.call("duo_engine_set_capture", self._h, L.DUO_CAP_ACT, n,
                   None if arr is None else arr.ctypes.data_as(C.c_void_p), L.ptr(buf), int(cap_t or buf.shape[1]))
            on.append(L.DUO_CAP_ACT)
        for kind in on:
            if t0:
                L.call("duo_engine_set_capture_t0", self._h, kind, t0)
        if opts.get("stopAfter") is not None:
            L.call("duo_engine_set_stop_after", self._h, int(opts["stopAfter"]))
        return on

    def _clear_hooks(self, on, opts):
        for kind in on:
            L.call("duo_engine_set_capture", self._h, kind, 0, None, None, 0)
        if opts.get("stopAfter") is not None:
            L.call("duo_engine_set_stop_after", self._h, -1)

    def forward(self, ids, row_base, rows, T, opts=None):
        """_forward: rows consecutive sequences from row_base, T new tokens each (ids token-major, len rows * T)."""
        opts = opts or {}
        self._set_pushes(opts.get("pushes"))
        hooks = self._set_hooks(opts)
        try:
            self._forward(ids, row_base, rows, T, opts)
        finally:
            self._clear_hooks(hooks, opts)

    def _forward(self, ids, row_base, rows, T, opts):
        vec = opts.get("vec")
        vec = -1 if vec is None else int(vec)
        if torch.is_tensor(ids) and ids.is_cuda:
            ids = ids.to(torch.int32).contiguous()
            L.call("duo_engine_forward_device", self._h, L.ptr(ids), row_base, rows, T, vec, self._s())
            return
        host = np.ascontiguousarray(np.asarray(ids, dtype=np.int32).reshape(-1))
        if host.size != rows * T:
            raise L.DuoError(L.DUO_EINVAL, f"forward: {host.size} ids for rows * T = {rows * T}")
        # the engine copies the ids into its own pinned staging before returning: `host` may go away after the call
        L.call("duo_engine_forward", self._h, host.ctypes.data_as(C.c_void_p), row_base, rows, T, vec, self._s())

    def prefill(self, r, ids, opts=None):
        """Prefill row r with ids from its current length, in chunks of max_t tokens (model.js:486-491)."""
        ids = list(ids) if not torch.is_tensor(ids) else ids
        opts = opts or {}
        for i in range(0, len(ids), self.max_t):
            chunk = ids[i:i + self.max_t]
            self.forward(chunk, r, 1, len(chunk), {**opts, "capT0": int(opts.get("capT0", 0) or 0) + i})

    def step(self, ids, opts=None):
        """Decode one token for every row (ids[r] for row r) (model.js:508)."""
        self.forward(ids, 0, self.rows, 1, opts)

    def row_len(self, r):
        return L.check(L.lib().duo_engine_row_len(self._h, r))

    # ---- live profiling (CUDA events around each launch of the selected kernel classes)
    def profile(self, kinds=None):
        """Start timing the given classes (names of lib.PROF_KINDS; None = all, [] = off)."""
        kinds = L.PROF_KINDS if kinds is None else kinds
        mask = 0
        for k in kinds:
            mask |= 1 << L.PROF_KINDS.index(k)
        L.call("duo_engine_profile", self._h, mask)

    def profile_read(self):
        """{class: (milliseconds, launches)} since the last read; synchronises the device."""
        n = len(L.PROF_KINDS)
        ms = (C.c_double * n)()
        cnt = (C.c_longlong * n)()
        L.call("duo_engine_profile_read", self._h, ms, cnt)
        return {k: (ms[i], cnt[i]) for i, k in enumerate(L.PROF_KINDS) if cnt[i]}

    # ---- heads (model.js:472-505)
    def logits(self, row0=0, n=None):
        n = self.rows - row0 if n is None else n
        out = torch.empty(n, self.cfg.vocab_size, dtype=torch.float32, device="cuda")
        L.call("duo_engine_logits", self._h, row0, n, L.ptr(out), self._s())
        return out

    def logits_row(self, r):
        return self.logits(r, 1)[0]

    def logits_all(self):
        return self.logits(0, self.rows)

    def argmax_all(self, device_out=False):
        out = torch.empty(self.rows, dtype=torch.int32, device="cuda")
        L.call("duo_engine_argmax", self._h, 0, self.rows, L.ptr(out), self._s())
        return out if device_out else out.tolist()

    def generate(self, n_steps, vec=None):
        """Greedy decode of every row for n_steps on the device (the reference's argmaxAll + step loop,
        analysis.js:127-142); returns the tokens [rows, n_steps] (int32, CUDA)."""
        out = torch.empty(self.rows, max(n_steps, 1), dtype=torch.int32, device="cuda")
        L.call("duo_engine_generate", self._h, n_steps, -1 if vec is None else int(vec), L.ptr(out), self._s())
        return out[:, :n_steps]
