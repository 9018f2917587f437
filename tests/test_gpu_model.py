"""GPU parity of the whole engine (libduo_mixer.so through duo.Model) against the CPU oracle on the same dequantised
int8 weights: the method of the reference's tests/engine_ref.py + tests/engine.mjs (same inputs; logits, greedy
tokens; pushes and the residual vector) and steerfind.html (batched rows == single rows).

Tolerances (max relative logit error, north_star):
  * f32 engine: 1e-4 against the f32 oracle and identical greedy tokens for 32 steps (config 1);
  * 16-bit engines (f16 / bf16 activations): TOL16 = 2e-2 against the oracle run with the engine's own rounding points
    (OracleModel.ROUND_POINTS: the intermediates the engine stores in 16 bits, and for G = 128 the tensor-core pack's
    16-bit q * s), i.e. on identical arithmetic up to summation order and the chunk scan's f16 internals;
  * and against the pure f32 oracle: 2e-2, or 1.3 x the error the rounding points alone cause if that is larger.
    For f16 that is 2e-2.  For bf16 it is not: rounding only the projection GEMMs' A operands to bf16 already puts
    config 1's logits 2.5% off f32, all of the engine's points 3.5% (tests/test_bf16_floor.py), so no bf16 engine
    can meet 2e-2 against f32 on this model.
Greedy tokens of a 16-bit engine may differ from the f32 oracle's only where the oracle's top-2 logit gap is within
twice the logit error measured at that step."""
import numpy as np
import pytest
import torch

from conftest import rel_max
from oracle.model import Cfg, OracleModel, map_weights
from tiny import TINY, tiny_state_dict, tiny_workload

TOL16 = 2e-2
BF16_FLOOR_FACTOR = 1.25
RND16 = {"bf16": lambda x: x.to(torch.bfloat16).float(), "f16": lambda x: x.to(torch.float16).float()}


def make_oracle(cfg, Wd, act, group, rows, max_len, emulate):
    """The f32 oracle, or (emulate, 16-bit act) the oracle that rounds where the engine does."""
    if not emulate or act == "f32":
        return OracleModel(cfg, Wd, rows=rows, max_len=max_len)
    rnd = RND16[act]
    wg = map_weights(Wd, rnd) if group else None  # G = 128: the tensor-core pack holds 16-bit(q * s)
    return OracleModel(cfg, Wd, rows=rows, max_len=max_len, round_points={p: rnd for p in OracleModel.ROUND_POINTS},
                       gemm_weights=wg)


def check_16bit(eng, ref, emu, act, what=""):
    """eng / ref / emu: per-step logits of the engine, the f32 oracle and the emulating oracle."""
    s_emu = [round(rel_max(a, b), 5) for a, b in zip(eng, emu)]
    s_ref = [round(rel_max(a, b), 5) for a, b in zip(eng, ref)]
    s_floor = [round(rel_max(b, r), 5) for b, r in zip(emu, ref)]
    e_emu, e_ref, floor = max(s_emu), max(s_ref), max(s_floor)
    detail = {"vs_emulating": s_emu, "vs_f32": s_ref, "emulating_vs_f32": s_floor}
    if act == "f16":
        assert e_emu < TOL16, (what, "vs emulating oracle", detail)
        assert e_ref < TOL16, (what, "vs f32 oracle", detail)
    else:
        assert e_ref < max(TOL16, BF16_FLOOR_FACTOR * floor), (what, "vs f32 oracle", detail)
    return e_emu, e_ref, floor


def check_greedy_near_ties(toks, ref_toks, eng, ref):
    """Tokens may differ only where the reference's top-2 gap is within twice the measured logit error of the step."""
    same = torch.stack(toks) == torch.stack(ref_toks)
    for s, r in zip(*torch.nonzero(~same, as_tuple=True)):
        s, r = int(s), int(r)
        top2 = ref[s][r].topk(2).values
        err = float((eng[s][r].double() - ref[s][r].double()).abs().max())
        assert float(top2[0] - top2[1]) <= 2 * err, ("divergence away from a near-tie", s, r)

pytestmark = pytest.mark.gpu


def duo_cfg_from_tiny(types, act, group=128):
    from duo import Config
    c = TINY
    return Config(hidden_size=c["hidden"], intermediate_size=c["inter"], vocab_size=c["vocab"],
                  num_hidden_layers=c["layers"], num_attention_heads=c["nh"], num_key_value_heads=c["nkv"],
                  head_dim=c["hd"], partial_rotary_factor=c["rot"] / c["hd"], rope_theta=c["theta"],
                  linear_num_key_heads=c["hk"], linear_num_value_heads=c["hv"], linear_key_head_dim=c["dk"],
                  linear_value_head_dim=c["dv"], linear_conv_kernel_dim=c["ks"], rms_norm_eps=c["eps"],
                  layer_types=types, group=group, act_dtype=act)


def oracle_cfg(types):
    c = TINY
    return Cfg(hidden=c["hidden"], inter=c["inter"], vocab=c["vocab"], layers=c["layers"], nh=c["nh"], nkv=c["nkv"],
               hd=c["hd"], rot=c["rot"], theta=c["theta"], hk=c["hk"], hv=c["hv"], dk=c["dk"], dv=c["dv"], ks=c["ks"],
               eps=c["eps"], layer_types=types)


def to_cpu(W):
    return {"embed": W["embed"].cpu(), "final_norm": W["final_norm"].cpu(),
            "layers": [{k: v.cpu() for k, v in L.items()} for L in W["layers"]]}


@pytest.fixture(scope="module")
def tiny(cuda):
    from duo import from_state_dict
    sd, types = tiny_state_dict()
    sdt = {k: torch.from_numpy(v) for k, v in sd.items()}
    out = {}
    for group in (128, 0):
        cfg = duo_cfg_from_tiny(types, "f32", group)
        W = from_state_dict(sdt, cfg)
        out[group] = (W, to_cpu(W.dequantized()))
    return types, out


def run_engine(types, W, act, ids, push, vec_layer, vecs, steps, group=128, max_t=64):
    from duo import Model
    cfg = duo_cfg_from_tiny(types, act, group)
    m = Model(cfg, W)
    m.alloc(rows=3, max_len=64, max_t=max_t, max_tokens=3 * ids.shape[1])
    if vecs is not None:
        m.set_vectors(list(vecs))
    opts = {"pushes": push, "vec": vec_layer}
    m.forward(ids.reshape(-1), 0, 3, ids.shape[1], opts)
    logits = [m.logits_all().cpu()]
    toks = []
    for _ in range(steps):
        nxt = logits[-1].argmax(-1)
        toks.append(nxt)
        m.step(nxt.tolist(), opts)
        logits.append(m.logits_all().cpu())
    return logits, toks


def run_oracle(types, Wd, ids, push, vec_layer, vecs, steps, forced=None, act="f32", group=128, emulate=False):
    om = make_oracle(oracle_cfg(types), Wd, act, group, 3, 64, emulate)
    if vecs is not None:
        om.set_vectors(list(vecs))
    om.forward(ids.reshape(-1), 0, 3, ids.shape[1], pushes=push, vec=vec_layer)
    logits = [om.logits()]
    for s in range(steps):
        nxt = forced[s] if forced is not None else logits[-1].argmax(-1)
        om.forward(nxt.tolist(), 0, 3, 1, pushes=push, vec=vec_layer)
        logits.append(om.logits())
    return logits


@pytest.mark.parametrize("act", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("group", [128, 0])
def test_tiny_model_parity(tiny, act, group):
    types, packs = tiny
    W, Wd = packs[group]
    ids, push, vec_layer, vecs = tiny_workload()
    eng, toks = run_engine(types, W, act, ids, push, vec_layer, vecs, 6, group)
    ref = run_oracle(types, Wd, ids, push, vec_layer, vecs, 6, forced=toks)
    ref_toks = [r.argmax(-1) for r in ref[:-1]]
    if act == "f32":
        for s, (a, b) in enumerate(zip(eng, ref)):
            assert rel_max(a, b) < 1e-4, f"step {s}"
        assert torch.equal(torch.stack(toks), torch.stack(ref_toks))
    else:
        emu = run_oracle(types, Wd, ids, push, vec_layer, vecs, 6, forced=toks, act=act, group=group, emulate=True)
        check_16bit(eng, ref, emu, act, f"tiny {act} G={group}")
        check_greedy_near_ties(toks, ref_toks, eng, ref)


@pytest.mark.parametrize("act", ["f32", "f16", "bf16"])
def test_batched_equals_single_rows(tiny, act):
    """tests/steerfind.html:25-38: one 3-row forward equals three single-row prefills, each row its own push."""
    from duo import Model
    types, packs = tiny
    W, _ = packs[128]
    ids, push, _, _ = tiny_workload()
    cfg = duo_cfg_from_tiny(types, act)
    m = Model(cfg, W).alloc(rows=3, max_len=64, max_t=64, max_tokens=64)
    m.forward(ids.reshape(-1), 0, 3, ids.shape[1], {"pushes": push})
    batched = m.logits_all().cpu()
    for r in range(3):
        m.reset(r)
        m.prefill(r, ids[r].tolist(), {"pushes": push})
        single = m.logits_row(r).cpu()
        tol = 1e-5 if act == "f32" else 2e-2
        assert rel_max(single, batched[r]) < tol


@pytest.mark.parametrize("act", ["f32", "f16", "bf16"])
def test_chunked_prefill_and_row_lengths(tiny, act):
    """model.js:486-491: prefill in max_t chunks carries state; lengths advance per row."""
    from duo import Model
    types, packs = tiny
    W, Wd = packs[128]
    ids, _, _, _ = tiny_workload()
    cfg = duo_cfg_from_tiny(types, act)
    m = Model(cfg, W).alloc(rows=3, max_len=64, max_t=7)
    m.prefill(1, ids[1].tolist())
    assert m.row_len(1) == 20 and m.row_len(0) == 0
    out = {}
    for emulate in ((False,) if act == "f32" else (False, True)):
        om = make_oracle(oracle_cfg(types), Wd, act, 128, 3, 64, emulate)
        for i in range(0, 20, 7):  # the same 7-token calls as the engine's prefill
            chunk = ids[1][i:i + 7]
            om.forward(chunk, 1, 1, len(chunk))
        out[emulate] = om.logits([1])[0]
    eng = m.logits_row(1).cpu()
    if act == "f32":
        assert rel_max(eng, out[False]) < 1e-4
    else:
        check_16bit([eng], [out[False]], [out[True]], act, f"chunked prefill {act}")


@pytest.mark.parametrize("act", ["f32", "f16", "bf16"])
def test_long_prefill(tiny, act):
    """One 150-token forward per row (several conv tiles and scan chunks, ragged last ones) and a second 37-token
    forward that continues from the carried state, against the oracle (model.js:404-466)."""
    from duo import Model
    types, packs = tiny
    W, Wd = packs[128]
    ids = torch.randint(0, TINY["vocab"], (2, 187), generator=torch.Generator().manual_seed(11))
    m = Model(duo_cfg_from_tiny(types, act), W).alloc(rows=2, max_len=200, max_t=150, max_tokens=300)
    om = OracleModel(oracle_cfg(types), Wd, rows=2, max_len=200)
    emu = make_oracle(oracle_cfg(types), Wd, act, 128, 2, 200, True)
    for a, b in ((0, 150), (150, 187)):
        m.forward(ids[:, a:b].reshape(-1), 0, 2, b - a)
        om.forward(ids[:, a:b].reshape(-1), 0, 2, b - a)
        emu.forward(ids[:, a:b].reshape(-1), 0, 2, b - a)
        eng = m.logits_all().cpu()
        if act == "f32":
            assert rel_max(eng, om.logits()) < 1e-4, (a, b)
        else:
            check_16bit([eng], [om.logits()], [emu.logits()], act, f"long prefill {act} {a}:{b}")


def test_generate_matches_step_loop(tiny):
    from duo import Model
    types, packs = tiny
    W, _ = packs[128]
    ids, push, vec_layer, vecs = tiny_workload()
    cfg = duo_cfg_from_tiny(types, "f32")
    a = Model(cfg, W).alloc(rows=3, max_len=64, max_t=64, max_tokens=64)
    a.set_vectors(list(vecs))
    a.forward(ids.reshape(-1), 0, 3, 20, {"pushes": push, "vec": vec_layer})
    toks = a.generate(5, vec=vec_layer).cpu()
    _, ref_toks = run_engine(types, W, "f32", ids, push, vec_layer, vecs, 5)
    assert torch.equal(toks.long(), torch.stack(ref_toks, 1))


@pytest.mark.parametrize("act,rows", [("f32", 3), ("bf16", 12), ("bf16", 3)])
def test_generate_graph_replay_equals_direct(tiny, act, rows):
    """generate on a non-default stream replays a CUDA graph of one decode step (the step index in a device
    counter); on the default stream it launches each step.  Same tokens, same final logits, bit for bit, across two
    generate calls (the second one captures again)."""
    import torch
    from duo import Model
    types, packs = tiny
    W, _ = packs[128]
    T = 9
    ids = torch.randint(0, TINY["vocab"], (rows, T), generator=torch.Generator().manual_seed(11))
    vecs = [torch.randn(TINY["hidden"], generator=torch.Generator().manual_seed(12 + r)) for r in range(rows)]
    cfg = duo_cfg_from_tiny(types, act)
    out = {}
    import contextlib
    from duo import lib as L
    for name, stream in (("direct", None), ("graph", torch.cuda.Stream())):
        with torch.cuda.stream(stream) if stream is not None else contextlib.nullcontext():
            m = Model(cfg, W, stream=stream).alloc(rows=rows, max_len=32, max_t=T, max_tokens=rows * T)
            m.set_vectors(vecs)
            m.forward(ids.reshape(-1), 0, rows, T, {"vec": 1})
            c0 = L.lib().duo_launch_count()
            g1 = m.generate(5, vec=1).cpu()
            g2 = m.generate(3, vec=1).cpu()
            launches = L.lib().duo_launch_count() - c0  # replays count the kernels they run
            out[name] = (g1, g2, m.logits_all().cpu(), m.row_len(0), launches)
    d, g = out["direct"], out["graph"]
    assert d[4] == g[4] > 0
    assert torch.equal(d[0], g[0]) and torch.equal(d[1], g[1])
    assert torch.equal(d[2], g[2])
    assert d[3] == g[3] == T + 8
    from duo import ops
    assert ops.fault_status() == 0


_FUSED_NORM_SCRIPT = """
import sys
import numpy as np
import torch
sys.path[:0] = sys.argv[2:]
from tiny import TINY, tiny_state_dict
from test_gpu_model import duo_cfg_from_tiny
from duo import Model, from_state_dict
sd, types = tiny_state_dict()
W = from_state_dict({k: torch.from_numpy(v) for k, v in sd.items()}, duo_cfg_from_tiny(types, "f32"))
rows, T = 4, 4800
ids = torch.randint(0, TINY["vocab"], (rows * T,), generator=torch.Generator().manual_seed(21))
m = Model(duo_cfg_from_tiny(types, "bf16"), W).alloc(rows=rows, max_len=T + 4, max_t=T, max_tokens=rows * T)
m.forward(ids, 0, rows, T)
first = m.logits_all().cpu().numpy()
m.step([1, 2, 3, 4])
np.save(sys.argv[1], np.stack([first, m.logits_all().cpu().numpy()]))
"""


def test_fused_prefill_norm_equals_separate_norm(tmp_path):
    """A bf16 prefill large enough for the persistent GEMMs to carry the RMSNorms (4 rows x 4800 tokens of the tiny
    model: 150 tiles of 128 x 256 per H-wide projection) against the same forward with every norm its own launch
    (DUO_FUSED_NORM=0, a second process): both round the norm's input to bf16 once, at different points, so their
    logits agree within the bf16 bound."""
    import os
    import subprocess
    import sys as _sys
    import numpy as np
    from conftest import GOLDEN, PKG, ROOT
    script = tmp_path / "run.py"
    script.write_text(_FUSED_NORM_SCRIPT)
    tests_dir = os.path.dirname(os.path.abspath(__file__))
    out = {}
    for name, env_val in (("fused", None), ("separate", "0")):
        env = dict(os.environ)
        env.pop("DUO_FUSED_NORM", None)
        if env_val is not None:
            env["DUO_FUSED_NORM"] = env_val
        dst = tmp_path / f"{name}.npy"
        r = subprocess.run([_sys.executable, str(script), str(dst), tests_dir, GOLDEN, PKG, ROOT], env=env,
                           capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stderr[-2000:]
        out[name] = torch.from_numpy(np.load(dst))
    for step in range(2):
        assert rel_max(out["fused"][step], out["separate"][step]) < TOL16, step


@pytest.mark.parametrize("act", ["f16", "bf16"])
def test_greedy_from_lm_head_epilogue(tiny, act):
    """More than 8 rows on the tensor-core engine: argmax_all and generate take the LM head's argmax epilogue (no
    logits written).  Their tokens equal argmax of the engine's own logits (model.js argmaxAll, analysis.js:127-142),
    lowest index on ties; only a top-2 gap within f32 rounding may differ between the two GEMM tilings."""
    from duo import Model
    types, packs = tiny
    W, _ = packs[128]
    rows, T, steps = 12, 9, 4
    ids = torch.randint(0, TINY["vocab"], (rows, T), generator=torch.Generator().manual_seed(3))
    cfg = duo_cfg_from_tiny(types, act)
    m = Model(cfg, W).alloc(rows=rows, max_len=32, max_t=T, max_tokens=rows * T)
    m.forward(ids.reshape(-1), 0, rows, T)
    logits = m.logits_all().cpu()
    fused = torch.tensor(m.argmax_all())
    top2 = logits.topk(2, -1).values
    near_tie = (top2[:, 0] - top2[:, 1]) <= 1e-6 * top2[:, 0].abs()
    assert bool(((fused.long() == logits.argmax(-1)) | near_tie).all())
    gen = m.generate(steps).cpu()
    m2 = Model(cfg, W).alloc(rows=rows, max_len=32, max_t=T, max_tokens=rows * T)
    m2.forward(ids.reshape(-1), 0, rows, T)
    loop = []
    for _ in range(steps):
        nxt = m2.logits_all().argmax(-1)
        loop.append(nxt.cpu())
        m2.step(nxt.tolist())
    assert torch.equal(gen.long(), torch.stack(loop, 1))


def test_head_scales(tiny):
    """setHeadScales (model.js:362-369; applied after the gated norm, kernels_qwen35.js:243): per-head output scales
    of linear-attention layers, for prefill and decode; None restores ones."""
    from duo import Model
    types, packs = tiny
    W, Wd = packs[128]
    lin = [l for l, t in enumerate(types) if t == "linear_attention"]
    hv = TINY["hv"]
    scales = {lin[0]: [0.5 + 0.25 * i for i in range(hv)], lin[-1]: [2.0 - 0.3 * i for i in range(hv)]}
    ids, _, _, _ = tiny_workload()
    m = Model(duo_cfg_from_tiny(types, "f32"), W).alloc(rows=3, max_len=64, max_t=64, max_tokens=64)
    om = OracleModel(oracle_cfg(types), Wd, rows=3, max_len=64)
    plain = OracleModel(oracle_cfg(types), Wd, rows=3, max_len=64)
    m.set_head_scales(scales)
    om.set_head_scales(scales)
    m.forward(ids.reshape(-1), 0, 3, ids.shape[1])
    om.forward(ids.reshape(-1), 0, 3, ids.shape[1])
    plain.forward(ids.reshape(-1), 0, 3, ids.shape[1])
    assert rel_max(m.logits_all().cpu(), om.logits()) < 1e-4
    assert rel_max(om.logits(), plain.logits()) > 1e-3  # the scales change the result
    m.step([1, 2, 3])
    om.forward([1, 2, 3], 0, 3, 1)
    assert rel_max(m.logits_all().cpu(), om.logits()) < 1e-4
    m.set_head_scales(None)
    m.reset_all()
    m.forward(ids.reshape(-1), 0, 3, ids.shape[1])
    assert rel_max(m.logits_all().cpu(), plain.logits()) < 1e-4


def test_engine_stops_after_a_fault(tiny):
    """With the fault word set (from the host here, as a mirrored device fault would be), engine calls return an error
    before launching anything; once duo_fault_status has read and cleared it, the engine runs again."""
    from duo import DuoError, Model, lib as L, ops
    types, packs = tiny
    W, _ = packs[128]
    m = Model(duo_cfg_from_tiny(types, "bf16"), W).alloc(rows=2, max_len=32, max_t=8)
    m.prefill(0, list(range(5)))
    before = m.logits_row(0).cpu()
    assert ops.fault_status() == 0
    L.lib().duo_fault_raise(2)
    n0 = L.lib().duo_launch_count()
    with pytest.raises(DuoError, match="gave up"):
        m.step([1, 2])
    with pytest.raises(DuoError, match="gave up"):
        m.generate(3)
    assert L.lib().duo_launch_count() == n0
    assert m.row_len(0) == 5
    assert ops.fault_status() == 2
    assert torch.equal(m.logits_row(0).cpu(), before)
    m.step([1, 2])
    assert m.row_len(0) == 6


def test_engine_errors(tiny):
    from duo import DuoError, Model
    types, packs = tiny
    W, _ = packs[128]
    m = Model(duo_cfg_from_tiny(types, "f32"), W).alloc(rows=2, max_len=8, max_t=8)
    with pytest.raises(DuoError):
        m.forward(list(range(9)), 0, 1, 9)        # more tokens than max_tokens / max_len
    m.prefill(0, list(range(8)))
    with pytest.raises(DuoError):
        m.step([1, 2])                            # row 0 is full
    with pytest.raises(DuoError):
        m.forward([1], 2, 1, 1)                   # row out of range


# ---------------------------------------------------------------------------------------------------------------
# config 1: the full Qwen3.5-0.8B shape, random init under seed 0 through transformers (the reference's PyTorch
# path), 3 rows with the +0.8 / 0 / -0.8 dose on L12 N1234, 64 prompt ids, 32 greedy steps


@pytest.fixture(scope="module")
def config1(cuda):
    pytest.importorskip("transformers")
    from duo import Config, from_state_dict
    from oracle import hf
    from oracle.model import Cfg as OCfg
    torch.set_num_threads(max(1, torch.get_num_threads()))
    ocfg = OCfg()
    model = hf.build_model(ocfg, seed=0)
    sd = {k: v for k, v in model.state_dict().items()}
    del model
    cfg = Config(group=128, act_dtype="f32")
    W = from_state_dict(sd, cfg)
    Wd = to_cpu(W.dequantized())
    del sd
    ids = torch.randint(0, ocfg.vocab, (3, 64), generator=torch.Generator().manual_seed(0))
    # dose unit (analysis.js:52-110): median token norm of the layer-12 output over a seeded calibration sequence
    # (token 0 skipped), divided by |W_down[12][:, 1234]|
    cal = OracleModel(ocfg, Wd, rows=1, max_len=80)
    calib = torch.randint(0, ocfg.vocab, (64,), generator=torch.Generator().manual_seed(1))
    resid = cal.forward(calib, 0, 1, 64, capture_resid=True)
    p50 = float(resid[12][1:].norm(dim=-1).median())
    col = float(Wd["layers"][12]["down"][:, 1234].norm())
    unit = p50 / col
    push = {12: [{"n": 1234, "mode": "add", "vals": [0.8 * unit, 0.0, -0.8 * unit]}]}
    return ocfg, W, Wd, ids, push


@pytest.mark.slow
@pytest.mark.parametrize("act", ["f32", "f16", "bf16"])
def test_config1_full_model(config1, act):
    from duo import Config, Model
    ocfg, W, Wd, ids, push = config1
    cfg = Config(group=128, act_dtype=act)
    m = Model(cfg, W).alloc(rows=3, max_len=128, max_t=64, max_tokens=192)
    opts = {"pushes": push}
    m.forward(ids.reshape(-1), 0, 3, 64, opts)
    eng = [m.logits_all().cpu()]
    toks = []
    for s in range(32):
        nxt = eng[-1].argmax(-1)
        toks.append(nxt)
        m.step(nxt.tolist(), opts)
        eng.append(m.logits_all().cpu())
    runs = {}
    for emulate in ((False,) if act == "f32" else (False, True)):
        om = make_oracle(ocfg, Wd, act, 128, 3, 128, emulate)
        om.forward(ids.reshape(-1), 0, 3, 64, pushes=push)
        lg = [om.logits()]
        for s in range(32):
            om.forward(toks[s].tolist(), 0, 3, 1, pushes=push)  # teacher-forced on the engine's tokens
            lg.append(om.logits())
        runs[emulate] = lg
    ref = runs[False]
    ref_toks = [r.argmax(-1) for r in ref[:-1]]
    if act == "f32":
        errs = [rel_max(a, b) for a, b in zip(eng, ref)]
        assert max(errs) < 1e-4, errs
        assert torch.equal(torch.stack(toks), torch.stack(ref_toks))
    else:
        check_16bit(eng, ref, runs[True], act, f"config 1 {act}")
        check_greedy_near_ties(toks, ref_toks, eng, ref)


# ---------------------------------------------------------------------------------------------------------------
# the configuration bench.py times: full shape, int8 weights with one scale per output row, bf16 activations, prompts
# prefilled in groups of 2 rows, long enough for the TMA-fed conv's multi-block path, lengths not multiples of 64;
# more than 8 rows, so decode runs the decode GEMM and greedy tokens come from the LM head's argmax epilogue


@pytest.mark.slow
def test_bench_configuration_parity(cuda):
    from duo import Model, qwen35_0p8b
    from duo.weights import random_weights
    cfg = qwen35_0p8b(group=0, act_dtype="bf16")
    W = random_weights(cfg, seed=5)
    Wd = to_cpu(W.dequantized())
    ocfg = Cfg()
    rows, T1, T2, steps, vec_layer = 12, 601, 37, 8, 12
    gen = torch.Generator().manual_seed(7)
    ids = torch.randint(0, ocfg.vocab, (rows, T1 + T2), generator=gen)
    # steering vectors on the first half of the rows, N(0, 1) * 0.5 * the median residual norm after layer 12 of a
    # calibration prompt (token 0 skipped), as bench.py sets them
    cal = OracleModel(ocfg, Wd, rows=1, max_len=64)
    resid = cal.forward(torch.randint(0, ocfg.vocab, (64,), generator=gen), 0, 1, 64, capture_resid=True)
    p50 = float(resid[vec_layer][1:].norm(dim=-1).median())
    vecs = [torch.randn(ocfg.hidden, generator=gen) * 0.5 * p50 if r < rows // 2 else None for r in range(rows)]

    m = Model(cfg, W).alloc(rows=rows, max_len=T1 + T2 + steps + 1, max_t=T1, max_tokens=2 * T1)
    m.set_vectors(vecs)
    opts = {"vec": vec_layer}
    for a, b in ((0, T1), (T1, T1 + T2)):
        for g0 in range(0, rows, 2):  # row groups of 2, as the bench's max_tokens gives
            m.forward(ids[g0:g0 + 2, a:b].reshape(-1), g0, 2, b - a, opts)
    eng = [m.logits_all().cpu()]
    gen_toks = m.generate(steps, vec=vec_layer).cpu().long()  # [rows, steps]: first = argmax of the prefill state
    eng.append(m.logits_all().cpu())
    assert m.row_len(0) == T1 + T2 + steps

    runs = {}
    for emulate in (False, True):
        om = make_oracle(ocfg, Wd, "bf16", 0, rows, T1 + T2 + steps + 1, emulate)
        om.set_vectors(vecs)
        for a, b in ((0, T1), (T1, T1 + T2)):
            for g0 in range(0, rows, 2):
                om.forward(ids[g0:g0 + 2, a:b].reshape(-1), g0, 2, b - a, vec=vec_layer)
        lg = [om.logits()]
        for s in range(steps):
            om.forward(gen_toks[:, s].tolist(), 0, rows, 1, vec=vec_layer)  # teacher-forced on the engine's tokens
            lg.append(om.logits())
        runs[emulate] = lg
    ref, emu = runs[False], runs[True]
    check_16bit(eng, [ref[0], ref[-1]], [emu[0], emu[-1]], "bf16", "bench configuration")
    # the engine's greedy tokens against the oracle's logits at every step (near-ties within the measured error)
    err = max(float((a.double() - b.double()).abs().max()) for a, b in zip(eng, [ref[0], ref[-1]]))
    for s in range(steps):
        ref_tok = ref[s].argmax(-1)
        for r in torch.nonzero(gen_toks[:, s] != ref_tok).flatten().tolist():
            top2 = ref[s][r].topk(2).values
            assert float(top2[0] - top2[1]) <= 2 * err, ("divergence away from a near-tie", s, r)
    from duo import ops
    assert ops.fault_status() == 0


# ---------------------------------------------------------------------------------------------------------------
# capture hooks (model.js:7-12, 445-461), stopAfter (427), tokenExtremes (kernels.js:288-306)


@pytest.mark.parametrize("act", ["f32", "bf16"])
def test_capture_hooks(tiny, act):
    """resid (every layer), resid "attn" and the down_proj-input capture of two layers, over a prefill chunked by maxT
    (capT0 advances per chunk, model.js:486-491), against the oracle's values at the same points."""
    from duo import Model
    types, packs = tiny
    W, Wd = packs[128]
    c = TINY
    ids, push, _, _ = tiny_workload()
    T = ids.shape[1]
    m = Model(duo_cfg_from_tiny(types, act), W).alloc(rows=3, max_len=64, max_t=7, max_tokens=21)
    nl = c["layers"]
    resid = torch.full((nl, T, c["hidden"]), float("nan"), device="cuda")
    attn = torch.full((nl, T, c["hidden"]), float("nan"), device="cuda")
    cap_layers = [1, nl - 1]
    capt = torch.full((2, T, c["inter"]), float("nan"), device="cuda")
    m.prefill(1, ids[1].tolist(), {"pushes": push, "resid": True, "residBuf": resid, "capT": T})
    m.reset(1)
    m.prefill(1, ids[1].tolist(), {"pushes": push, "resid": "attn", "residBuf": attn, "capture": capt,
                                   "capLayers": cap_layers, "capT": T})
    om = make_oracle(oracle_cfg(types), Wd, act, 128, 3, 64, True)
    got = {}
    for i in range(0, T, 7):  # the engine's 7-token chunks
        part = {}
        chunk = ids[1][i:i + 7]
        om.forward(chunk, 1, 1, len(chunk), pushes=push, capture=part)
        for k, v in part.items():
            got.setdefault(k, []).append(torch.stack(v))
    ref = {k: torch.cat(v, 1) for k, v in got.items()}  # [layers, T, width]
    tol = 1e-4 if act == "f32" else TOL16
    assert rel_max(resid.cpu(), ref["resid"]) < tol
    assert rel_max(attn.cpu(), ref["resid_attn"]) < tol
    assert rel_max(capt.cpu(), ref["act"][cap_layers]) < tol
    # the hooks were per call: a later forward writes nothing
    resid.fill_(0)
    m.step([1, 2, 3])
    assert float(resid.abs().max()) == 0.0


def test_capture_overflow_and_stop_after(tiny):
    from duo import DuoError, Model
    types, packs = tiny
    W, Wd = packs[128]
    c = TINY
    ids, _, _, _ = tiny_workload()
    m = Model(duo_cfg_from_tiny(types, "f32"), W).alloc(rows=3, max_len=64, max_t=64, max_tokens=64)
    small = torch.empty(c["layers"], 4, c["hidden"], device="cuda")
    n0 = m.row_len(0)
    with pytest.raises(DuoError, match="capture holds"):
        m.forward(ids[0][:5].tolist(), 0, 1, 5, {"resid": True, "residBuf": small, "capT": 4})
    assert m.row_len(0) == n0  # refused before anything ran
    # stopAfter: the row's last hidden state is the residual after that layer
    k = 2
    m.forward(ids[0].tolist(), 0, 1, ids.shape[1], {"stopAfter": k})
    om = OracleModel(oracle_cfg(types), Wd, rows=3, max_len=64)
    om.forward(ids[0], 0, 1, ids.shape[1], stop_after=k)
    assert rel_max(m.logits_row(0).cpu(), om.logits([0])[0]) < 1e-4


def test_token_extremes(cuda):
    from duo import lib as L
    g = torch.Generator().manual_seed(4)
    nl, T, I, t0 = 3, 37, 1000, 1
    cap = torch.randn(nl, T, I, generator=g)
    cap[0, 5, 7] = cap[0, 9, 7] = 50.0  # a tie: the first token wins
    out = torch.empty(nl, I, 4, device="cuda")
    L.call("duo_token_extremes", L.ptr(cap.cuda()), nl, T, I, t0, L.ptr(out), L.stream_ptr())
    sub = cap[:, t0:]
    mx, amx = sub.max(1)
    mn, amn = sub.min(1)
    o = out.cpu()
    assert torch.equal(o[..., 0], mx) and torch.equal(o[..., 2], mn)
    assert torch.equal(o[..., 1].long(), amx + t0) and torch.equal(o[..., 3].long(), amn + t0)
    assert int(o[0, 7, 1]) == 5


# ---------------------------------------------------------------------------------------------------------------
# the batched push probe (analysis.js:480-537) on the engine against the oracle


def test_push_test_matches_oracle(tiny):
    from duo import Model, probe
    from oracle import probe as oprobe
    types, packs = tiny
    W, Wd = packs[128]
    c = TINY
    cands = [(0, 5), (2, c["inter"] - 1), (2, 17), (c["layers"] - 1, 3)]
    gen = torch.Generator().manual_seed(9)
    contexts = [torch.randint(0, c["vocab"], (16,), generator=gen).tolist() for _ in range(2)]
    targets = torch.randint(0, c["vocab"], (24,), generator=gen).tolist()
    tw = (torch.rand(24, generator=gen) + 0.1).tolist()
    units = [1.5, 0.7, 2.0, 1.1]
    rows = 3 * len(cands) * len(contexts)
    m = Model(duo_cfg_from_tiny(types, "f32"), W).alloc(rows=rows, max_len=32, max_t=16, max_tokens=rows * 16)
    res = probe.push_test(m, cands, contexts, targets, tw, dose=0.8, units=units, keep_d=True)
    ids, pushes, base = probe.build_batch(cands, contexts, units, 0.8)
    om = OracleModel(oracle_cfg(types), Wd, rows=rows, max_len=32)
    om.forward(ids, 0, rows, 16, pushes=pushes)
    lg = om.logits()
    assert rel_max(res["logits"].cpu(), lg) < 1e-4
    rs, rd = oprobe.push_stats(lg.numpy(), np.asarray(base), np.asarray(targets), np.log(np.asarray(tw)))
    st = res["stats"].double().cpu().numpy()
    for col in range(6):
        err = np.abs(st[:, col] - rs[:, col])
        assert (err <= 1e-4 * (1 + np.abs(rs[:, col]))).all(), (col, err.max())
    assert rel_max(res["d"].cpu(), torch.from_numpy(rd)) < 1e-3
    # the strength-0 rows carry no push: all three rows of a triple see the same context
    assert float(np.abs(st[1::3, 3]).max()) == 0.0
    assert len(res["summary"]) == 2 * len(cands)


def test_host_ids_may_be_reused_when_forward_returns(tiny):
    """duo_engine_forward copies the caller's ids before returning: forwards queued back to back from one reused host
    array (the GPU still busy with the earlier ones) give the same rows as device-resident ids."""
    import numpy as np
    from duo import Model
    types, packs = tiny
    W, _ = packs[128]
    rows, T = 24, 40
    ids = torch.randint(0, TINY["vocab"], (rows, T), generator=torch.Generator().manual_seed(21))
    a = Model(duo_cfg_from_tiny(types, "bf16"), W).alloc(rows=rows, max_len=T + 1, max_t=T, max_tokens=2 * T)
    b = Model(duo_cfg_from_tiny(types, "bf16"), W).alloc(rows=rows, max_len=T + 1, max_t=T, max_tokens=2 * T)
    buf = np.empty(2 * T, dtype=np.int32)
    for g0 in range(0, rows, 2):
        buf[:] = ids[g0:g0 + 2].reshape(-1).numpy()  # the same host array, rewritten for every call
        a.forward(buf, g0, 2, T)
    for g0 in range(0, rows, 2):
        b.forward(ids[g0:g0 + 2].reshape(-1).to(torch.int32).cuda(), g0, 2, T)
    assert torch.equal(a.logits_all().cpu(), b.logits_all().cpu())
