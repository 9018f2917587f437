"""Statistics of the reference's push probe, restated on the CPU in float64 (test infrastructure only).

Follows engine/analysis.js:480-537 (`probe`): every steered row's next-token log-probabilities lp (logSoftmax,
analysis.js:693-702) are compared with those of the unsteered row of the same context, b:
  mass = sum_j exp(lp[t_j])                                  (analysis.js:515)
  dp   = mass(lp) - mass(b)                                  (analysis.js:518)
  gain = lse(lp[t] + log w) - lse(b[t] + log w)              (analysis.js:517, 519; lse 665)
  kl   = sum over p_i > 1e-12 of p_i (lp_i - b_i)            (analysis.js:520, kl 704-708)
  d   += lp - b                                              (analysis.js:522-523)
The PyTorch form of the same test is tools/find_steering.py:86-103 (KL without the cutoff there).
"""
import numpy as np


def log_softmax(x):
    x = np.asarray(x, dtype=np.float64)
    m = x.max(-1, keepdims=True)
    return x - (m + np.log(np.exp(x - m).sum(-1, keepdims=True)))


def lse(x):
    x = np.asarray(x, dtype=np.float64)
    m = x.max(-1, keepdims=True)
    return (m + np.log(np.exp(x - m).sum(-1, keepdims=True)))[..., 0]


def push_stats(logits, base, targets, target_logw=None):
    """logits [n, V]; base [n] (index of each row's unsteered row, -1 for none); targets [nt] ids; target_logw [nt].

    Returns (stats [n, 6] = lse, mass, tlse, kl, dp, gain as in duo_push_stats, d [n, V] = lp - lb or 0)."""
    x = np.asarray(logits, dtype=np.float64)
    n, v = x.shape
    lsev = lse(x)
    lp = x - lsev[:, None]
    t = np.asarray(targets, dtype=np.int64)
    w = np.zeros(len(t)) if target_logw is None else np.asarray(target_logw, dtype=np.float64)
    ok = (t >= 0) & (t < v)
    lpt = np.where(ok[None, :], lp[:, np.clip(t, 0, v - 1)], -np.inf)
    mass = np.exp(lpt).sum(-1)
    tl = lpt + w[None, :]
    tlse = np.array([lse(r[np.isfinite(r)]) if np.isfinite(r).any() else -np.inf for r in tl])
    out = np.zeros((n, 6))
    out[:, 0], out[:, 1], out[:, 2] = lsev, mass, tlse
    d = np.zeros((n, v))
    for r in range(n):
        b = int(base[r])
        if b < 0:
            continue
        p = np.exp(lp[r])
        keep = p > 1e-12
        out[r, 3] = float((p[keep] * (lp[r][keep] - lp[b][keep])).sum())
        out[r, 4] = mass[r] - mass[b]
        out[r, 5] = tlse[r] - tlse[b]
        d[r] = lp[r] - lp[b]
    return out, d
