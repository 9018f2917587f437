"""The batched push probe: each candidate neuron pushed at +dose / 0 / -dose in a few short contexts, all in one forward.

Mirrors the reference's Explorer (engine/analysis.js):
  * dose unit (analysis.js:52-110): an add-mode dose of 1 moves a neuron by (median residual norm leaving its layer)
    / |its down_proj column|; resid_p50() measures the medians with the `resid` capture of one calibration prompt
    (token 0 skipped), col_norms() the column norms from the int8 weights;
  * probe (analysis.js:480-537): every candidate's pushed rows are compared with the unpushed row of the same
    context -- probability mass on the target ids (dp), weighted target log-odds (gain), KL and the per-vocabulary
    log-probability delta.  The reference runs three rows per forward (its engine holds four); here a forward runs
    every (candidate, context) triple at once, one push record per (layer, neuron) with a value per row, and the
    statistics come from duo_push_stats on the device.
Rows are ordered (candidate, context, strength) with strengths (+dose, 0, -dose); row 3i + 1 is the base of rows 3i and
3i + 2.  A rank of a multi-GPU run takes whole triples, so every pushed row has its base on the same GPU.
"""
import math

import torch

from . import ops
from .lib import DUO_STATS_COLS


def resid_p50(model, ids):
    """Median over tokens 1 .. T-1 of the residual norm after every layer, for one calibration prompt (row 0 of the
    model, reset before and after; analysis.js:52-77)."""
    cfg = model.cfg
    T = len(ids)
    buf = torch.empty(cfg.num_hidden_layers, T, cfg.hidden_size, dtype=torch.float32, device="cuda")
    model.reset(0)
    model.forward(ids, 0, 1, T, {"resid": True, "residBuf": buf, "capT": T, "capT0": 0})
    torch.cuda.synchronize()
    model.reset(0)
    norms = buf[:, 1:].double().norm(dim=-1).sort(dim=-1).values  # [L, T-1]
    return norms[:, norms.shape[1] >> 1].float().cpu()


def col_norms(weights, layer, neurons):
    """|W_down[layer][:, n]| for each neuron n, from the int8 weights (dequantised f32(q) * scale; analysis.js:80-91)."""
    d = weights.layers[layer]["down"]
    w = ops.q8_dequantize(d.q, d.s, torch.float32)  # [hidden, inter]
    return w[:, torch.as_tensor(neurons, device=w.device)].double().norm(dim=0).float().cpu()


def triple_rows(n_cands, n_ctx, units=None):
    """(candidate, context, strength index) of every row, strengths (+, 0, -) innermost; units = the (candidate,
    context) pairs as candidate-major indices k * n_ctx + c (default all)."""
    units = range(n_cands * n_ctx) if units is None else units
    return [(u // n_ctx, u % n_ctx, s) for u in units for s in range(3)]


def build_batch(cands, contexts, units, dose=0.8, pairs=None):
    """Rows of one probe batch.  cands: [(layer, neuron)]; contexts: [list of T ids] (one length); units: dose unit
    of each candidate; pairs: the (candidate, context) indices k * n_ctx + c to run (default all, candidate-major).
    Returns (ids [rows * T] token-major, pushes {layer: [{n, mode, vals}]}, base [rows])."""
    T = len(contexts[0])
    if any(len(c) != T for c in contexts):
        raise ValueError("probe contexts must share one length (one forward)")
    rows = triple_rows(len(cands), len(contexts), pairs)
    ids = [t for (_, c, _) in rows for t in contexts[c]]
    strength = (dose, 0.0, -dose)
    recs = {}  # (layer, n) -> per-row values
    for r, (k, c, s) in enumerate(rows):
        key = (int(cands[k][0]), int(cands[k][1]))
        vals = recs.setdefault(key, [0.0] * len(rows))
        vals[r] = strength[s] * float(units[k])
    pushes = {}
    for (layer, n), vals in recs.items():
        pushes.setdefault(layer, []).append({"n": n, "mode": "add", "vals": vals})
    base = [3 * (r // 3) + 1 if r % 3 != 1 else -1 for r in range(len(rows))]
    return ids, pushes, base


def push_test(model, cands, contexts, targets, target_w=None, dose=0.8, units=None, calib=None, keep_d=False,
              row_base=0, pairs=None, summarize=True):
    """One batched push test on the engine (rows row_base .. of `model`).  units: dose units per candidate (computed
    from `calib` ids with resid_p50 / col_norms when None).  Returns a dict with the per-row statistics [rows, 6]
    (lse, mass, tlse, kl, dp, gain as duo_push_stats), the logits [rows, vocab], d [rows, vocab] when keep_d, and
    per-candidate means over contexts for the + and - rows (dp, gain, kl: analysis.js:515-523)."""
    if units is None:
        p50 = resid_p50(model, calib)
        units = [float(p50[l]) / max(float(col_norms(model.weights, l, [n])[0]), 1e-30) for l, n in cands]
    ids, pushes, base = build_batch(cands, contexts, units, dose, pairs)
    rows = len(base)
    T = len(contexts[0])
    if row_base == 0 and rows == model.rows:
        model.reset_all()
    else:
        for r in range(row_base, row_base + rows):
            model.reset(r)
    model.forward(ids, row_base, rows, T, {"pushes": _shift(pushes, row_base, model.rows)})
    logits = model.logits(row_base, rows)
    tid = torch.as_tensor(targets, dtype=torch.int32, device="cuda")
    logw = None
    if target_w is not None:
        logw = torch.as_tensor([math.log(w) for w in target_w], dtype=torch.float32, device="cuda")
    base_t = torch.as_tensor(base, dtype=torch.int32, device="cuda")
    d = torch.zeros_like(logits) if keep_d else None
    stats, d = ops.push_stats(logits, base_t, tid, logw, d=d)
    n_ctx = len(contexts)
    summary = []
    st = stats.double().cpu() if summarize else None
    for k in (range(len(cands)) if summarize and pairs is None else ()):
        for s, sign in ((0, 1), (2, -1)):
            rr = [3 * (k * n_ctx + c) + s for c in range(n_ctx)]
            summary.append({"layer": int(cands[k][0]), "n": int(cands[k][1]), "sign": sign, "unit": float(units[k]),
                            "dp": float(st[rr, 4].mean()), "gain": float(st[rr, 5].mean()),
                            "kl": float(st[rr, 3].mean())})
    assert stats.shape[1] == DUO_STATS_COLS
    return {"stats": stats, "logits": logits, "d": d, "base": base, "units": units, "summary": summary}


def _shift(pushes, row_base, total_rows):
    """Per-row push values indexed by absolute engine row (the engine's push tables are [records, rows])."""
    if row_base == 0:
        return pushes
    out = {}
    for layer, recs in pushes.items():
        out[layer] = []
        for rec in recs:
            vals = [0.0] * row_base + list(rec["vals"])
            vals += [0.0] * (total_rows - len(vals))
            out[layer].append({**rec, "vals": vals})
    return out
