"""CPU tests of the oracle: pinned against the golden fixtures made from the reference's PyTorch path
(tests/golden/make_golden.py) and against known answers of the reference's int8 format (engine/kernels.js:16-47)."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, rel_max
from oracle import mixer, q8
from oracle.model import Cfg, OracleModel, fuse_state_dict
from tiny import TINY, tiny_state_dict, tiny_workload


# ---------------------------------------------------------------------------------------------------------------
# int8 format: known answers that follow the WGSL semantics


def test_q8_known_answers():
    # one 128-group: absmax 2.54 -> scale 0.02; v / scale rounds half to even
    row = np.zeros(128, dtype=np.float32)
    row[0] = 2.54
    row[1] = -2.54
    row[2] = 0.03   # 1.5 -> 2 (ties to even)
    row[3] = 0.05   # 2.5 -> 2 (ties to even)
    row[4] = -0.05  # -2.5 -> -2
    row[5] = 0.07   # 3.5 -> 4
    q, s = q8.quantize(row[None, :], 128)
    scale = np.float32(2.54) / np.float32(127)
    assert s[0, 0] == scale
    expect = np.rint(row / scale).astype(np.int8)
    assert np.array_equal(q[0], expect)
    assert q[0, 0] == 127 and q[0, 1] == -127
    # the ties land exactly on .5 only if the f32 quotient is exact; check the rounding mode on exact halves
    half = np.array([[0.5, 1.5, 2.5, -0.5, -1.5, -2.5] + [0.0] * 121 + [127.0]], dtype=np.float32)
    qh, sh = q8.quantize(half, 128)
    assert sh[0, 0] == np.float32(1.0)
    assert qh[0, :6].tolist() == [0, 2, 2, 0, -2, -2]


def test_q8_zero_group_scale_is_one():
    w = np.zeros((2, 256), dtype=np.float32)
    w[1, 200] = -3.0
    q, s = q8.quantize(w, 128)
    assert s.tolist() == [[1.0, 1.0], [1.0, np.float32(3.0) / np.float32(127)]]
    assert q[1, 200] == -127 and np.count_nonzero(q) == 1


def test_q8_per_row_group_and_roundtrip():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((64, 384)) * 0.02).astype(np.float32)
    for g in (128, 384):
        q, s = q8.quantize(w, g)
        assert s.shape == (64, 384 // g)
        d = q8.dequantize(q, s, g)
        # error of a symmetric 8-bit quantiser is at most half a step
        step = np.repeat(s, g, axis=1)
        assert np.all(np.abs(d - w) <= 0.5 * step * (1 + 1e-6))


def test_q8_gather_and_matvec():
    rng = np.random.default_rng(1)
    w = rng.standard_normal((50, 256)).astype(np.float32)
    q, s = q8.quantize(w, 128)
    ids = [3, 0, 49, 3]
    g = q8.gather(ids, q, s, 128)
    assert np.array_equal(g, q8.dequantize(q, s, 128)[ids])
    x = rng.standard_normal((3, 256)).astype(np.float32)
    y = q8.matvec(x, q, s, 128)
    ref = x.astype(np.float64) @ q8.dequantize(q, s, 128).astype(np.float64).T
    assert np.allclose(y, ref, rtol=1e-6, atol=1e-6)


# ---------------------------------------------------------------------------------------------------------------
# DeltaNet ops vs the reference's PyTorch functions (fixtures)


@pytest.fixture(scope="module")
def gdn():
    return dict(np.load(os.path.join(GOLDEN, "gdn_ops.npz")))


def _t(a):
    return torch.from_numpy(a)


def test_chunk_rule_matches_fixture(gdn):
    o, s = mixer.chunk_gated_delta_rule(_t(gdn["q"]), _t(gdn["k"]), _t(gdn["v"]), _t(gdn["g"]), _t(gdn["beta"]),
                                        state=_t(gdn["s0"]))
    assert rel_max(o, gdn["o_chunk"]) < 1e-5
    assert rel_max(s, gdn["s_chunk"]) < 1e-5


def test_recurrent_rule_matches_fixture(gdn):
    o, s = mixer.recurrent_gated_delta_rule(_t(gdn["q"]), _t(gdn["k"]), _t(gdn["v"]), _t(gdn["g"]), _t(gdn["beta"]),
                                            state=_t(gdn["s0"]))
    assert rel_max(o, gdn["o_rec"]) < 1e-5
    assert rel_max(s, gdn["s_rec"]) < 1e-5
    # the two forms agree with each other (chunk vs token-by-token), as in the reference
    assert rel_max(gdn["o_chunk"], gdn["o_rec"]) < 1e-4


def test_conv_update_matches_fixture(gdn):
    x = _t(gdn["conv_x"]).transpose(1, 2)          # [B, T, C]
    st = _t(gdn["conv_state_in"])[:, :, 1:].transpose(1, 2)  # the last KS-1 inputs, oldest first
    out, ns = mixer.causal_conv1d(x, _t(gdn["conv_w"]), st)
    assert rel_max(out.transpose(1, 2), gdn["conv_out"]) < 1e-6
    assert rel_max(ns.transpose(1, 2), _t(gdn["conv_state_out"])[:, :, 1:]) == 0.0


def test_rope_table_matches_fixture():
    r = np.load(os.path.join(GOLDEN, "rope.npz"))
    inv = mixer.rope_inv_freq(64, 1e7)
    pos = torch.from_numpy(r["pos"][0])
    freqs = pos.float()[:, None] * inv
    emb = torch.cat([freqs, freqs], -1)
    assert rel_max(emb.cos(), r["cos"][0]) < 1e-6
    assert rel_max(emb.sin(), r["sin"][0]) < 1e-6


# ---------------------------------------------------------------------------------------------------------------
# full tiny model (pushes, vec, greedy decode) vs the fixture from Qwen3_5ForCausalLM


def tiny_oracle(dtype=torch.float32, rows=3, max_len=64):
    sd, types = tiny_state_dict()
    c = TINY
    cfg = Cfg(hidden=c["hidden"], inter=c["inter"], vocab=c["vocab"], layers=c["layers"], nh=c["nh"], nkv=c["nkv"],
              hd=c["hd"], rot=c["rot"], theta=c["theta"], hk=c["hk"], hv=c["hv"], dk=c["dk"], dv=c["dv"], ks=c["ks"],
              eps=c["eps"], layer_types=types)
    W = fuse_state_dict({k: torch.from_numpy(v) for k, v in sd.items()}, cfg)
    return cfg, OracleModel(cfg, W, rows=rows, max_len=max_len, dtype=dtype)


@pytest.mark.parametrize("with_hooks", [True, False])
def test_tiny_model_matches_fixture(with_hooks):
    f = np.load(os.path.join(GOLDEN, "tiny_model.npz"))
    ids, push, vec_layer, vecs = tiny_workload()
    cfg, om = tiny_oracle()
    pre = "" if with_hooks else "plain_"
    if with_hooks:
        om.set_vectors(list(vecs))
    kw = dict(pushes=push, vec=vec_layer) if with_hooks else {}
    om.forward(ids.reshape(-1), 0, 3, ids.shape[1], **kw)
    assert rel_max(om.logits(), f[pre + "logits_prefill"]) < 1e-5
    toks = []
    cur = om.logits().argmax(-1)
    for s in range(f[pre + "tokens"].shape[1]):
        toks.append(cur)
        om.forward(cur.tolist(), 0, 3, 1, **kw)
        lg = om.logits()
        assert rel_max(lg, f[pre + "logits_steps"][s]) < 1e-5
        cur = lg.argmax(-1)
    assert torch.stack(toks, 1).tolist() == f[pre + "tokens"].tolist()


def test_batched_equals_single_row():
    """steerfind.html:25-38 of the reference: a batched multi-row prefill equals single-row prefills."""
    ids, push, vec_layer, vecs = tiny_workload()
    cfg, om = tiny_oracle()
    om.forward(ids.reshape(-1), 0, 3, ids.shape[1], pushes=push)
    batched = om.logits()
    for r in range(3):
        _, single = tiny_oracle()
        single.forward(ids[r], r, 1, ids.shape[1], pushes=push)
        assert rel_max(single.logits([r]), batched[r:r + 1]) < 1e-5


def test_chunked_prefill_equals_one_call():
    """model.js:486-491 prefill chunks by maxT: the state carried across chunks gives the same logits."""
    ids, _, _, _ = tiny_workload()
    _, a = tiny_oracle(rows=1)
    a.forward(ids[0], 0, 1, 20)
    _, b = tiny_oracle(rows=1)
    for i in range(0, 20, 7):
        chunk = ids[0][i:i + 7]
        b.forward(chunk, 0, 1, len(chunk))
    assert rel_max(b.logits(), a.logits()) < 1e-5
