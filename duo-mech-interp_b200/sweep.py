"""Op-level sweeps of the mixer kernels (BASELINE configs 2 and 3, and the projection GEMM) with CUDA-event timing.

    python duo-mech-interp_b200/sweep.py gemm [--m M --n N --k K] [--acc]
    python duo-mech-interp_b200/sweep.py gemm-decode [--m M] [--colscale] [--intw]
                                           # the projection shapes at m rows (256), optionally with per-row weight
                                           # scales in the epilogue and int8-valued weights as the engine runs them
    python duo-mech-interp_b200/sweep.py gemv [--m M --n N --k K]             # int8 GEMV, m <= 8
    python duo-mech-interp_b200/sweep.py gdn-decode [--b B --steps S]      # config 2b
    python duo-mech-interp_b200/sweep.py gdn-prefill [--b B --t T]         # config 2a
    python duo-mech-interp_b200/sweep.py attn-prefill [--b B --t T]        # config 3a
    python duo-mech-interp_b200/sweep.py attn-decode [--b B --len L]       # config 3b
    python duo-mech-interp_b200/sweep.py all                               # every config, one JSON line each

Each case prints one JSON line: the algorithmic work per launch, the mean launch time (CUDA events around replays of
a CUDA graph of the launches, after warm-up, so host launch cost is excluded; inputs larger than L2 or rotated through
several copies), achieved GB/s or TFLOP/s and the fraction of the measured peak of this pool (MEASURED_PEAKS.json).
"""
import argparse
import json
import math
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

from duo import ops  # noqa: E402


def peaks():
    try:
        return json.load(open(os.path.join(os.path.dirname(HERE), "MEASURED_PEAKS.json"))), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def timed(fn, iters=10, warmup=3, graph=True):
    """Mean device time (ms) of one fn() call: after `warmup` eager calls, `iters` calls are captured into a CUDA
    graph and the graph is replayed, so the host's per-call launch cost (Python, ctypes) is not what is measured.
    graph=False times an eager loop instead."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if not graph:
        a.record()
        for _ in range(iters):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / iters
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize()
    reps = 3
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / (reps * iters)


def report(case, shape, ms, flops=None, bytes_=None, extra=None):
    pk, src = peaks()
    line = {"case": case, "shape": shape, "ms": ms}
    if flops is not None:
        line["tflops"] = flops / ms / 1e9
        line["frac_bf16_peak"] = line["tflops"] / pk["bf16_tflops"]
    if bytes_ is not None:
        line["gbs"] = bytes_ / ms / 1e6
        line["frac_hbm_peak"] = line["gbs"] / pk["hbm_gbs"]
    line["peak_source"] = src
    line.update(extra or {})
    print(json.dumps(line), flush=True)
    return line


def gemm(m, n, k, iters=10, compare=True, accumulate=False):
    """bf16 C = A B^T, or (accumulate) the residual-add epilogue X += A B^T into an f32 X; cuBLAS beside it
    (for the residual add: an f32-output matmul plus the add)."""
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    b = (torch.randn(n, k, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    c = torch.zeros(m, n, device="cuda", dtype=torch.float32 if accumulate else torch.bfloat16)
    ms = timed(lambda: ops.gemm_bf16(a, b, out=c, accumulate=accumulate), iters)
    extra = {"epilogue": "add_f32" if accumulate else "store_bf16"}
    if compare:
        if accumulate:
            ms_ref = timed(lambda: c.add_(torch.matmul(a, b.T).float()), iters)
        else:
            ms_ref = timed(lambda: torch.matmul(a, b.T, out=c), iters)
        extra.update({"cublas_ms": ms_ref, "cublas_tflops": 2.0 * m * n * k / ms_ref / 1e9})
    return report("gemm_bf16", [m, n, k], ms, flops=2.0 * m * n * k, extra=extra)


def gemm_decode(m=256, iters=8, colscale=False, intw=False):
    """The forward's projection shapes at m rows (Qwen3.5-0.8B: DeltaNet in-projection, attention q|gate|k|v,
    MLP gate|up + SwiGLU, and the residual-add projections); at decode sizes (m <= 256) each launch reads its own
    weight copy so that the weights stream from HBM as they do in a decode step; cuBLAS beside each."""
    if m > 256:
        iters = 3
    g = torch.Generator(device="cuda").manual_seed(0)
    a16 = {kk: torch.randn(m, kk, device="cuda", generator=g).to(torch.bfloat16) for kk in (1024, 2048, 3584)}
    for n, k, epi in [(8224, 1024, "store"), (5120, 1024, "store"), (7168, 1024, "swiglu"), (1024, 2048, "add"),
                      (1024, 3584, "add")]:
        if intw:  # int8-valued weights, as the engine's packs hold them (the row scale goes to col_scale)
            ws = [torch.randint(-127, 128, (n, k), device="cuda", generator=g).to(torch.bfloat16) for _ in range(iters)]
        else:
            ws = [(torch.randn(n, k, device="cuda", generator=g) * 0.05).to(torch.bfloat16) for _ in range(iters)]
        cs = (torch.rand(n, device="cuda", generator=g) * 1e-3 + 1e-4) if colscale else None
        a = a16[k]
        if epi == "add":
            c = torch.zeros(m, n, device="cuda", dtype=torch.float32)
            it = iter(range(1 << 30))
            run = lambda: ops.gemm_bf16(a, ws[next(it) % iters], col_scale=cs, out=c, accumulate=True)
            it2 = iter(range(1 << 30))
            ref = lambda: c.add_(torch.matmul(a, ws[next(it2) % iters].T).float())
        elif epi == "swiglu":
            c = torch.empty(m, n // 2, device="cuda", dtype=torch.bfloat16)
            it = iter(range(1 << 30))
            run = lambda: ops.gemm_swiglu(a, ws[next(it) % iters], col_scale=cs)
            it2 = iter(range(1 << 30))
            ref = lambda: torch.matmul(a, ws[next(it2) % iters].T)
        else:
            c = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
            it = iter(range(1 << 30))
            run = lambda: ops.gemm_bf16(a, ws[next(it) % iters], col_scale=cs, out=c)
            it2 = iter(range(1 << 30))
            ref = lambda: torch.matmul(a, ws[next(it2) % iters].T, out=c)
        ms = timed(run, iters)
        ms_ref = timed(ref, iters)
        wbytes = n * k * 2
        report("gemm_decode", [m, n, k], ms, flops=2.0 * m * n * k, bytes_=wbytes + m * k * 2,
               extra={"epilogue": epi, "cublas_ms": ms_ref, "weights": "%d copies" % iters,
                      "col_scale": colscale, "int_weights": intw})
        del ws


def gemv(m, n, k, group=128):
    """The int8 GEMV of decode (m <= 8 rows): y = x . dequant(W)^T with int8 W [n, k] and one f32 scale per 128-group,
    bf16 x and y.  Weight copies are rotated so that every launch streams W from HBM."""
    copies = max(1, math.ceil(4 * 126e6 / (n * k)))
    g = torch.Generator(device="cuda").manual_seed(0)
    qs = [torch.randint(-127, 128, (n, k), device="cuda", generator=g, dtype=torch.int8) for _ in range(copies)]
    ss = [torch.rand(n, k // group, device="cuda", generator=g) * 0.01 for _ in range(copies)]
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    y = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    it = {"i": 0}

    def one():
        i = it["i"] % copies
        it["i"] += 1
        ops.q8_gemv(x, qs[i], ss[i], y=y)

    ms = timed(one, iters=max(8, copies), warmup=copies)
    bytes_ = n * k + n * (k // group) * 4 + m * k * 2 + m * n * 2
    return report("q8_gemv", {"m": m, "n": n, "k": k, "group": group, "weight_copies": copies}, ms, bytes_=bytes_)


def gdn_inputs(b, t, h=16, dtype=torch.bfloat16, copies=1, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda *s: torch.randn(*s, device="cuda", generator=g)
    q = torch.nn.functional.normalize(mk(b, t, h, 128), dim=-1).to(dtype)
    k = torch.nn.functional.normalize(mk(b, t, h, 128), dim=-1).to(dtype)
    v = mk(b, t, h, 128).to(dtype)
    beta = torch.sigmoid(mk(b, t, h))
    gg = -torch.nn.functional.softplus(mk(b, t, h))
    states = [torch.zeros(b, h, 128, 128, device="cuda") for _ in range(copies)]
    return q, k, v, gg, beta, states


def gdn_decode(b, steps=256, h=16):
    """Config 2b: `steps` single-token recurrent steps carrying the state.  The state is rotated through enough
    copies that every launch reads it from HBM (the 1 MiB-per-row state would otherwise sit in L2)."""
    copies = max(1, math.ceil(4 * 126e6 / (b * h * 128 * 128 * 4)))
    q, k, v, gg, beta, states = gdn_inputs(b, steps, h, copies=copies)
    qs = [x[:, i:i + 1].contiguous() for i in range(steps) for x in (q,)]
    ks = [k[:, i:i + 1].contiguous() for i in range(steps)]
    vs = [v[:, i:i + 1].contiguous() for i in range(steps)]
    gs = [gg[:, i:i + 1].contiguous() for i in range(steps)]
    bs = [beta[:, i:i + 1].contiguous() for i in range(steps)]
    it = {"i": 0}

    def one():
        i = it["i"]
        it["i"] += 1
        s = i % steps
        ops.gdn_recurrent(qs[s], ks[s], vs[s], gs[s], bs[s], states[i % copies], l2norm_qk=False)

    ms = timed(one, iters=steps, warmup=8)
    bytes_ = b * h * (2 * 128 * 128 * 4 + 4 * 128 * 2 + 8)
    return report("gdn_decode_step", {"b": b, "h": h, "steps": steps, "state_copies": copies}, ms, bytes_=bytes_)


def gdn_prefill(b, t, h=16, fn="gdn_chunk"):
    """Config 2a: the chunked scan over b rows x t tokens x 16 heads (bf16 q/k/v, f32 g/beta/state)."""
    q, k, v, gg, beta, states = gdn_inputs(b, t, h)
    f = getattr(ops, fn)
    ms = timed(lambda: f(q, k, v, gg, beta, states[0], l2norm_qk=False), iters=5)
    c = 64
    flops = b * h * (t / c) * (5 * 2 * c * c * 128 + 3 * 2 * c * 128 * 128 + c ** 3 / 3)
    bytes_ = b * t * h * ((3 * 128 + 128) * 2 + 8)
    return report(fn, {"b": b, "t": t, "h": h}, ms, flops=flops, bytes_=bytes_)


def attn_inputs(b, t, max_len, nh=8, nkv=2, hd=256, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda *s: torch.randn(*s, device="cuda", generator=g).to(torch.bfloat16)
    return mk(b, t, nh, hd), mk(b, max_len, nkv, hd), mk(b, max_len, nkv, hd), mk(b, t, nh, hd)


def attn_prefill(b, t):
    """Config 3a: causal GQA prefill (8 q / 2 kv heads, hd 256) with the sigmoid gate over a fresh cache."""
    q, kc, vc, gate = attn_inputs(b, t, t)
    start = torch.zeros(b, dtype=torch.int32, device="cuda")
    ms = timed(lambda: ops.attention(q, kc, vc, start, gate=gate), iters=3)
    flops = 2.0 * b * 8 * 256 * t * t  # causal QK^T + PV
    return report("attn_prefill", {"b": b, "t": t}, ms, flops=flops)


def attn_decode(b, length):
    """Config 3b: one new token per row against a `length`-token bf16 KV cache (B=32 x 8192 = 537 MB)."""
    q, kc, vc, gate = attn_inputs(b, 1, length + 1)
    start = torch.full((b,), length, dtype=torch.int32, device="cuda")
    ms = timed(lambda: ops.attention(q, kc, vc, start, gate=gate), iters=20)
    bytes_ = b * (length + 1) * 2 * 256 * 2 * 2 + 2 * q.numel() * 2
    return report("attn_decode", {"b": b, "cache": length}, ms, bytes_=bytes_)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["gemm", "gemm-decode", "gemv", "gdn-decode", "gdn-prefill", "attn-prefill", "attn-decode", "all"])
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=7168)
    ap.add_argument("--k", type=int, default=1024)
    ap.add_argument("--b", type=int, default=None)
    ap.add_argument("--t", type=int, default=4096)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--len", type=int, default=8192)
    ap.add_argument("--fn", default="gdn_chunk")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--acc", action="store_true", help="gemm: residual-add epilogue into f32")
    ap.add_argument("--colscale", action="store_true", help="gemm-decode: per-row weight scale in the epilogue")
    ap.add_argument("--intw", action="store_true", help="gemm-decode: int8-valued weights (the engine's packs)")
    a = ap.parse_args()
    if a.case == "gemm":
        gemm(a.m, a.n, a.k, a.iters, accumulate=a.acc)
    elif a.case == "gemm-decode":
        gemm_decode(a.m if a.m != 8192 else 256, colscale=a.colscale, intw=a.intw)
    elif a.case == "gemv":
        gemv(a.m if a.m <= 8 else 1, a.n, a.k)
    elif a.case == "gdn-decode":
        gdn_decode(a.b or 1, a.steps)
    elif a.case == "gdn-prefill":
        gdn_prefill(a.b or 1, a.t, fn=a.fn)
    elif a.case == "attn-prefill":
        attn_prefill(a.b or 4, a.t)
    elif a.case == "attn-decode":
        attn_decode(a.b or 32, a.len)
    else:
        for m, n, k in [(65536, 8224, 1024), (65536, 7168, 1024), (65536, 1024, 3584), (256, 8224, 1024),
                        (256, 7168, 1024), (256, 248320, 1024), (8192, 8192, 8192)]:
            gemm(m, n, k)
        for m, n, k in [(1, 8224, 1024), (3, 8224, 1024), (8, 7168, 1024), (1, 248320, 1024), (3, 248320, 1024)]:
            gemv(m, n, k)
        for b in (1, 8):
            gdn_decode(b, a.steps)
        for b in (1, 8):
            for t in (512, 4096, 16384):
                gdn_prefill(b, t, fn=a.fn)
        for t in (1024, 4096, 16384):
            attn_prefill(4, t)
        attn_decode(32, 8192)


if __name__ == "__main__":
    main()
