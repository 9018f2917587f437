"""bench.py -- throughput of the Qwen3.5-0.8B-shaped engine on 1..8 B200s, one process per GPU.

Workloads (random-init weights of the 0.8B architecture with transformers' init distributions, int8 weights with one
scale per output row, bf16 activations; synthetic seeded token ids -- no checkpoint or dataset offline):
  config5 (default)  throughput serving: one batch of 256 prompts of 2048 random ids, then 512 greedy decode steps;
                     rows 0..127 carry a random layer-12 residual steering vector N(0,1) * 0.5 * median residual
                     norm.  Metric: prefill + decode tokens per second.
  config4            batched steering push test: 36 candidate neurons (layer, index) x 2 contexts of 16 random ids x
                     strengths {+0.8, 0, -0.8} dose units = 216 rows in one forward, then per row the next-token
                     log-softmax statistics against the strength-0 row of its (candidate, context): mass on 64 random
                     target ids, log-odds gain, KL (duo_push_stats).  Metric: prompt tokens per second.
The batch is fixed and split across the ranks (strong scaling) into contiguous blocks of whole units -- prompt rows
for config5, (candidate, context) triples for config4 -- with no exchange in the forward; one NCCL all_gather per step
collects the generated tokens (config5) or the statistics and logits (config4).  A step is one pass of the whole
batch: reset, prefill, decode / statistics, gather.

    python bench.py [--gpus N --steps K --warmup W] [--workload config4]    # our engine (one JSON line on rank 0)
    python bench.py --workload ops                                          # op cases of configs 2 / 3 and the
                                                                            # projections, one line ("ops" list)
    python bench.py --impl reference [--steps K --warmup W]                  # the reference's CPU PyTorch path
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "duo-mech-interp_b200"))

METRIC5 = "prefill+decode tok/s, Qwen3.5-0.8B shape (256 x 2048 prompt + 512 greedy decode)"
METRIC4 = "push-test prompt tok/s, Qwen3.5-0.8B shape (216 rows x 16 ids + next-token KL / mass statistics)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["duo", "reference"], default="duo")
    ap.add_argument("--workload", choices=["config5", "config4", "ops"], default="config5")
    ap.add_argument("--no-ops", action="store_true", help="config5: skip the op cases appended to the line")
    ap.add_argument("--op", default=None, help="ops: run only the cases whose name starts with this")
    ap.add_argument("--rows", type=int, default=256, help="config5: rows of the whole batch (split across GPUs)")
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--decode", type=int, default=512)
    ap.add_argument("--max-tokens", type=int, default=131072, help="tokens per prefill forward call")
    ap.add_argument("--vec-layer", type=int, default=12)
    ap.add_argument("--cands", type=int, default=36, help="config4: candidate neurons")
    ap.add_argument("--contexts", type=int, default=2, help="config4: contexts per candidate")
    ap.add_argument("--ctx-len", type=int, default=16)
    ap.add_argument("--targets", type=int, default=64)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    return ap.parse_args()


def cpu_desc():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown CPU"


# ---------------------------------------------------------------------------------------------------------------
# the reference's CPU path (transformers Qwen3_5ForCausalLM, fp32), timed on a bounded sample of each workload

# config5 sample: 4 prompts x 512 ids + 128 greedy steps -- the workload's 4 : 1 prompt : generated token mix
CPU_SAMPLE5 = (4, 512, 128)
# config4 sample: 4 candidates x 2 contexts x 3 strengths = 24 rows x 16 ids, statistics on the host
CPU_SAMPLE4 = (4, 2, 16)


class CpuReference:
    """The reference's PyTorch model built once on the host cores (all of them), with the push / vector hooks of
    tests/engine_ref.py and tools/find_steering.py."""

    def __init__(self, seed):
        import torch
        sys.path.insert(0, ROOT)
        from oracle import hf
        from oracle.model import Cfg
        torch.set_num_threads(os.cpu_count() or 1)
        self.torch, self.hf, self.cfg = torch, hf, Cfg()
        self.model = hf.build_model_fast(self.cfg, seed=seed)
        self.hooks = hf.Hooks(self.model)
        self.cores = torch.get_num_threads()
        self.seed = seed

    def sample5(self):
        """tok/s of prefill + greedy decode on CPU_SAMPLE5 (prompt and generated tokens counted, as the GPU metric)."""
        rows, prompt, decode = CPU_SAMPLE5
        ids = self.torch.randint(0, self.cfg.vocab, (rows, prompt), generator=self.torch.Generator().manual_seed(1))
        t0 = time.perf_counter()
        self.hf.prefill_and_greedy(self.model, ids, decode)
        dt = time.perf_counter() - t0
        return rows * (prompt + decode) / dt, dt

    def sample4(self):
        """tok/s of the push test on CPU_SAMPLE4: one forward of every row with per-row pushes, then log-softmax,
        target mass, gain and KL against the strength-0 row on the host (analysis.js:480-537)."""
        torch = self.torch
        n_c, n_ctx, T = CPU_SAMPLE4
        g = torch.Generator().manual_seed(2)
        cands = [(int(torch.randint(0, 24, (1,), generator=g)), int(torch.randint(0, 3584, (1,), generator=g)))
                 for _ in range(n_c)]
        ctx = torch.randint(0, self.cfg.vocab, (n_ctx, T), generator=g)
        tid = torch.randint(0, self.cfg.vocab, (64,), generator=g)
        rows = [(k, c, s) for k in range(n_c) for c in range(n_ctx) for s in (0.8, 0.0, -0.8)]
        ids = torch.stack([ctx[c] for (_, c, _) in rows])
        push = {}
        for r, (k, _, s) in enumerate(rows):
            layer, n = cands[k]
            vals = torch.zeros(len(rows))
            vals[r] = s * 40.0
            push.setdefault(layer, []).append((n, "add", vals))
        t0 = time.perf_counter()
        with torch.inference_mode():
            self.hooks.push = push
            lp = torch.log_softmax(self.model(input_ids=ids).logits[:, -1].double(), -1)
            self.hooks.push = {}
            for r in range(0, len(rows), 3):
                for s in (r, r + 2):
                    p = lp[s].exp()
                    keep = p > 1e-12
                    _ = float((p[keep] * (lp[s][keep] - lp[r + 1][keep])).sum())
                    _ = float(lp[s][tid].exp().sum() - lp[r + 1][tid].exp().sum())
        dt = time.perf_counter() - t0
        return len(rows) * T / dt, dt


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import torch
    import transformers
    ref = CpuReference(a.seed)
    sample = ref.sample4 if a.workload == "config4" else ref.sample5
    for _ in range(a.warmup):
        sample()
    vals, secs = [], []
    for _ in range(max(1, a.steps)):
        v, dt = sample()
        vals.append(v)
        secs.append(dt)
    v = statistics.median(vals)
    if a.workload == "config4":
        n_c, n_ctx, T = CPU_SAMPLE4
        what = f"{n_c} candidates x {n_ctx} contexts x 3 strengths = {3 * n_c * n_ctx} rows x {T} ids + statistics"
        metric, cfg = METRIC4, {"workload": "config4 slice on the host CPU (the reference's PyTorch path)",
                                "rows": 3 * n_c * n_ctx, "ctx_len": T}
    else:
        rows, prompt, decode = CPU_SAMPLE5
        what = f"{rows} prompts x {prompt} ids + {decode} greedy steps (the workload's 4:1 prompt:generated mix)"
        metric, cfg = METRIC5, {"workload": "config5 slice on the host CPU (the reference's PyTorch path)",
                                "rows": rows, "prompt": prompt, "decode": decode}
    sample_desc = (f"{what}, fp32, transformers {transformers.__version__} / torch {torch.__version__}, "
                   f"{cpu_desc()}")
    line = {"metric": metric, "value": v, "unit": "tok/s", "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": 1000 * statistics.median(secs), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random ids, random-init weights)",
            "impl": "reference", "config": cfg,
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": ref.cores, "kind": "reference",
                             "sample": sample_desc},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------------------------------------------
# clocks during the timed region


class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                       "--format=csv,noheader,nounits", "-lms", "200"], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        out, _ = self.p.communicate(timeout=10)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        loaded = [s for s in sm if s > 0.5 * max(mx or [1])] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------------------------------------------
# measurement helpers


def measured_traffic(kernel, rows, prompt):
    """DRAM bytes (read + write) per launch of a (phase:class) kernel from the committed ncu summary
    profiles/traffic.json, when it was measured on this rank's rows and prompt length; None otherwise."""
    try:
        t = json.load(open(os.path.join(ROOT, "profiles", "traffic.json")))
    except (OSError, ValueError):
        return None
    e = t.get("kernels", {}).get(kernel)
    if not e or e.get("rows") != rows or e.get("prompt", prompt) != prompt:
        return None
    return e["bytes_per_launch"]


def peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def algorithmic_work(cfg, rows, prompt, decode):
    """Algorithmic FLOPs / bytes of each (phase, kernel class) of one step on one rank (rows = rows of this rank):
    the per-unit figure of each class (per token, per row-layer, per chunk-head, per cached key) times the units of
    the step, as the comments below state; param_bytes counts one byte per int8 weight, i.e. the parameter count."""
    from duo.weights import param_bytes
    H, V = cfg.hidden_size, cfg.vocab_size
    n_lin = sum(1 for l in range(cfg.num_hidden_layers) if not cfg.is_full(l))
    n_full = cfg.num_hidden_layers - n_lin
    layer_params = param_bytes(cfg) - V * H
    hv, dk, dv = cfg.linear_num_value_heads, cfg.linear_key_head_dim, cfg.linear_value_head_dim
    nh, nkv, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    w = {}
    # prefill GEMMs: 2 * tokens * layer parameters (tensor); config4's logits add 2 * rows * V * H (decode = 0)
    w[("prefill", "gemm")] = ("tensor", 2.0 * rows * prompt * layer_params + (2.0 * rows * V * H if decode == 0 else 0))
    # decode GEMMs: every step runs the layer projections and the LM head for every row (tensor)
    w[("decode", "gemm")] = ("tensor", 2.0 * rows * decode * (layer_params + V * H))
    # decode DeltaNet step: read + write the f32 state, read q/k/v/z, write o (HBM)
    per_row_layer = hv * (2 * dk * dv * 4) + (2 * cfg.key_dim + 2 * cfg.value_dim) * 2 + cfg.value_dim * 2
    w[("decode", "gdn_scan")] = ("hbm", float(rows * decode * n_lin * per_row_layer))
    # decode attention: every step reads the K and V cache of every row up to its length (HBM)
    kv_tok = nkv * hd * 2 * 2  # K and V, bf16
    keys = sum(prompt + s + 1 for s in range(decode))
    w[("decode", "attn")] = ("hbm", float(rows * n_full * keys * kv_tok))
    # prefill attention: causal QK^T + PV = 2 * 2 * nh * hd * T^2 / 2 per row-layer (tensor)
    w[("prefill", "attn")] = ("tensor", 2.0 * rows * n_full * nh * hd * prompt * prompt)
    # prefill DeltaNet scan: chunked-form FLOPs, 11.62 M per (64-token chunk, head)
    c = 64
    per_chunk = 5 * 2 * c * c * dk + 3 * 2 * c * dk * dv + c ** 3 / 3
    w[("prefill", "gdn_scan")] = ("tensor", float(rows * n_lin * hv * (prompt / c) * per_chunk))
    return w


def roofline_of(m, phase_prof, work, run_dominant, pk, pk_src, traffic):
    """The dominant (phase, class) of the profiled warm-up step, timed per launch with CUDA events over one more
    step of the workload (run_dominant(kind) runs it with that class profiled)."""
    dominant = max(((ph, k) for ph in phase_prof for k in phase_prof[ph] if (ph, k) in work),
                   key=lambda pk_: phase_prof[pk_[0]][pk_[1]][0])
    dprof = run_dominant(dominant)
    dom_ms, dom_n = dprof.get(dominant[1], (float("nan"), 1))
    bound, units = work[dominant]
    per_launch = units / max(dom_n, 1)
    avg_s = dom_ms / max(dom_n, 1) / 1000
    if bound == "tensor":
        achieved, unit = per_launch / avg_s / 1e12, "TFLOP/s"
        peak = pk.get("bf16_tflops_sustained" if dominant[0] == "prefill" else "bf16_tflops")
    else:
        achieved, unit = per_launch / avg_s / 1e9, "GB/s"
        peak = pk.get("hbm_gbs")
    return {"kernel": f"{dominant[0]}:{dominant[1]}", "bound": bound, "achieved": achieved, "peak": peak,
            "unit": unit, "frac": achieved / peak if peak else None, "traffic": traffic(f"{dominant[0]}:{dominant[1]}"),
            "peak_source": pk_src, "launches": dom_n, "avg_launch_ms": dom_ms / max(dom_n, 1)}


def max_over_ranks(ms, world):
    import torch
    import torch.distributed as dist
    t = torch.tensor([ms], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())



# ---------------------------------------------------------------------------------------------------------------
# op cases: config 2 (chunked DeltaNet prefill, recurrent decode step), config 3 (gated attention prefill and decode),
# the int8 GEMV of the M <= 8 decode path and the forward's projection GEMMs beside cuBLAS.  Each is timed with CUDA
# events around replays of a CUDA graph of its launches (host launch cost excluded), after warm-up, on inputs larger
# than L2 or rotated through enough copies that every launch reads them from HBM; one dict per case with the
# algorithmic work per launch, the achieved rate and its fraction of the measured peak.


def op_timed(fn, iters=10, warmup=3):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / (reps * iters)


def op_report(case, shape, ms, flops=None, bytes_=None, target=None, extra=None):
    pk, src = peaks()
    r = {"case": case, "shape": shape, "ms": round(ms, 5)}
    if flops is not None:
        r.update(bound="tensor", achieved=flops / ms / 1e9, unit="TFLOP/s", peak=pk["bf16_tflops"])
    else:
        r.update(bound="hbm", achieved=bytes_ / ms / 1e6, unit="GB/s", peak=pk["hbm_gbs"])
    r["frac"] = r["achieved"] / r["peak"]
    r["peak_source"] = src
    if target is not None:
        r["north_star_target"] = target
    r.update(extra or {})
    return r


def op_gdn_inputs(b, t, h=16, copies=1, seed=0):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda *s: torch.randn(*s, device="cuda", generator=g)
    q = torch.nn.functional.normalize(mk(b, t, h, 128), dim=-1).to(torch.bfloat16)
    k = torch.nn.functional.normalize(mk(b, t, h, 128), dim=-1).to(torch.bfloat16)
    v = mk(b, t, h, 128).to(torch.bfloat16)
    beta = torch.sigmoid(mk(b, t, h))
    gg = -torch.nn.functional.softplus(mk(b, t, h))
    return q, k, v, gg, beta, [torch.zeros(b, h, 128, 128, device="cuda") for _ in range(copies)]


def op_gdn_prefill(b, t, h=16):
    """config 2a: the chunked scan over b rows x t tokens x 16 heads; 11.62 MFLOP per (64-token chunk, head)."""
    from duo import ops
    q, k, v, gg, beta, st = op_gdn_inputs(b, t, h)
    ms = op_timed(lambda: ops.gdn_chunk(q, k, v, gg, beta, st[0], l2norm_qk=False), iters=5)
    c = 64
    flops = b * h * (t / c) * (5 * 2 * c * c * 128 + 3 * 2 * c * 128 * 128 + c ** 3 / 3)
    return op_report("gdn_chunk_prefill", {"b": b, "t": t, "h": h}, ms, flops=flops, target=">= 0.50 at T >= 4096")


def op_gdn_decode(b, steps=64, h=16):
    """config 2b: single-token steps carrying the f32 state (2 x 64 KiB per row-head + q/k/v/o), the state rotated
    through enough copies to stream from HBM."""
    import math
    from duo import ops
    copies = max(1, math.ceil(4 * 126e6 / (b * h * 128 * 128 * 4)))
    q, k, v, gg, beta, states = op_gdn_inputs(b, steps, h, copies=copies)
    sl = [tuple(x[:, i:i + 1].contiguous() for x in (q, k, v, gg, beta)) for i in range(steps)]
    it = {"i": 0}

    def one():
        i = it["i"]
        it["i"] += 1
        qq, kk, vv, g1, b1 = sl[i % steps]
        ops.gdn_recurrent(qq, kk, vv, g1, b1, states[i % copies], l2norm_qk=False)

    ms = op_timed(one, iters=steps, warmup=8)
    return op_report("gdn_decode_step", {"b": b, "h": h, "state_copies": copies}, ms,
                     bytes_=b * h * (2 * 128 * 128 * 4 + 4 * 128 * 2 + 8), target=">= 0.70")


def op_attn_prefill(b, t):
    """config 3a: causal GQA prefill (8 q / 2 kv heads, hd 256) with the sigmoid gate; 2 b nh hd t^2 FLOP."""
    import torch
    from duo import ops
    g = torch.Generator(device="cuda").manual_seed(0)
    mk = lambda *s: torch.randn(*s, device="cuda", generator=g).to(torch.bfloat16)
    q, gate, kc, vc = mk(b, t, 8, 256), mk(b, t, 8, 256), mk(b, t, 2, 256), mk(b, t, 2, 256)
    start = torch.zeros(b, dtype=torch.int32, device="cuda")
    ms = op_timed(lambda: ops.attention(q, kc, vc, start, gate=gate), iters=3)
    return op_report("attn_prefill", {"b": b, "t": t}, ms, flops=2.0 * b * 8 * 256 * t * t,
                     target=">= 0.50 at T >= 4096")


def op_attn_decode(b, length):
    """config 3b: one new token per row against a `length`-token bf16 KV cache (B = 32 x 8192: 537 MB)."""
    import torch
    from duo import ops
    g = torch.Generator(device="cuda").manual_seed(0)
    mk = lambda *s: torch.randn(*s, device="cuda", generator=g).to(torch.bfloat16)
    q, gate, kc, vc = mk(b, 1, 8, 256), mk(b, 1, 8, 256), mk(b, length + 1, 2, 256), mk(b, length + 1, 2, 256)
    start = torch.full((b,), length, dtype=torch.int32, device="cuda")
    ms = op_timed(lambda: ops.attention(q, kc, vc, start, gate=gate), iters=20)
    return op_report("attn_decode", {"b": b, "cache": length}, ms,
                     bytes_=b * (length + 1) * 2 * 256 * 2 * 2 + 2 * q.numel() * 2)


def op_gemv(m, n, k, group=128):
    """The int8 GEMV of decode (m <= 8 rows): y = x . dequant(W)^T, int8 W [n, k] with an f32 scale per 128-group,
    bf16 x and y; the weights rotated through copies so that every launch streams them from HBM."""
    import math
    import torch
    from duo import ops
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

    ms = op_timed(one, iters=max(8, copies), warmup=copies)
    return op_report("q8_gemv", {"m": m, "n": n, "k": k, "group": group, "weight_copies": copies}, ms,
                     bytes_=n * k + n * (k // group) * 4 + m * k * 2 + m * n * 2, target=">= 0.70")


def op_gemm_decode(m=256, iters=8):
    """The forward's projection shapes at m decode rows as the engine runs them: the int8 weights (one scale per row)
    streamed and converted on chip (`ms`, bytes = the int8 weights + the activations), the same GEMM on the 16-bit
    pack of those weights (`pack_ms`), and cuBLAS on the 16-bit weights (bf16, no scale, no SwiGLU; for the residual
    add an f32 matmul plus the add; `cublas_ms`); each launch reads its own weight copy from HBM."""
    import torch
    from duo import ops
    g = torch.Generator(device="cuda").manual_seed(0)
    out = []
    for n, k, epi in [(8224, 1024, "store"), (5120, 1024, "store"), (7168, 1024, "swiglu"), (1024, 2048, "add"),
                      (1024, 3584, "add")]:
        a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
        qs = [torch.randint(-127, 128, (n, k), device="cuda", generator=g, dtype=torch.int8) for _ in range(iters)]
        ws = [q.to(torch.bfloat16) for q in qs]
        cs = torch.rand(n, device="cuda", generator=g) * 1e-3 + 1e-4
        s = cs[:, None].contiguous()
        it, it2, it3 = iter(range(1 << 30)), iter(range(1 << 30)), iter(range(1 << 30))
        if epi == "add":
            c = torch.zeros(m, n, device="cuda", dtype=torch.float32)
            run = lambda: ops.q8_gemm(a, qs[next(it3) % iters], s, y=c, accumulate=True)
            pack = lambda: ops.gemm_bf16(a, ws[next(it) % iters], col_scale=cs, out=c, accumulate=True)
            ref = lambda: c.add_(torch.matmul(a, ws[next(it2) % iters].T).float())
        elif epi == "swiglu":
            o = torch.empty(m, n // 2, device="cuda", dtype=torch.bfloat16)
            run = lambda: ops.q8_gemm(a, qs[next(it3) % iters], s, y=o, swiglu=True)
            pack = lambda: ops.gemm_swiglu(a, ws[next(it) % iters], col_scale=cs)
            ref = lambda: torch.matmul(a, ws[next(it2) % iters].T)
        else:
            c = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
            run = lambda: ops.q8_gemm(a, qs[next(it3) % iters], s, y=c)
            pack = lambda: ops.gemm_bf16(a, ws[next(it) % iters], col_scale=cs, out=c)
            ref = lambda: torch.matmul(a, ws[next(it2) % iters].T, out=c)
        ms_pack, ms, ms_ref = op_timed(pack, iters), op_timed(run, iters), op_timed(ref, iters)  # pack launches first
        out.append(op_report("gemm_decode", [m, n, k], ms, bytes_=n * k + m * k * 2,
                             extra={"epilogue": epi, "weights": "int8", "pack_ms": round(ms_pack, 5),
                                    "cublas_ms": round(ms_ref, 5)}))
        del ws, qs
    return out


def op_cases(full, only=None):
    """Every op case (full) or the compact set that the default run appends to its line; `only` keeps the cases
    whose name starts with it (gdn_chunk_prefill, gdn_decode_step, attn_prefill, attn_decode, q8_gemv, gemm_decode)."""
    todo = [("gdn_chunk_prefill", op_gdn_prefill, (8, 4096)), ("gdn_decode_step", op_gdn_decode, (8,)),
            ("attn_prefill", op_attn_prefill, (4, 4096)), ("attn_decode", op_attn_decode, (32, 8192)),
            ("q8_gemv", op_gemv, (1, 248320, 1024))]
    if full:
        todo += [("gdn_chunk_prefill", op_gdn_prefill, (b, t)) for b in (1, 8) for t in (512, 16384)]
        todo += [("gdn_chunk_prefill", op_gdn_prefill, (1, 4096)), ("gdn_decode_step", op_gdn_decode, (1,)),
                 ("attn_prefill", op_attn_prefill, (4, 1024)), ("attn_prefill", op_attn_prefill, (4, 16384))]
        todo += [("q8_gemv", op_gemv, s) for s in [(1, 8224, 1024), (3, 8224, 1024), (8, 7168, 1024),
                                                    (3, 248320, 1024)]]
        todo += [("gemm_decode", op_gemm_decode, (256,))]
    cases = []
    for name, fn, args in todo:
        if only and not name.startswith(only):
            continue
        r = fn(*args)
        cases += r if isinstance(r, list) else [r]
    return cases


def bench_ops(a):
    import torch
    cases = op_cases(full=True, only=a.op)
    return {"metric": "mixer op roofline fractions (configs 2 and 3, int8 GEMV, decode projections)",
            "value": min(c["frac"] for c in cases), "unit": "fraction of measured peak (min over the cases run)", "n_gpus": 1, "steps": 1, "warmup": 3, "higher_is_better": True, "scaling": "none",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) inputs as configs 2 and 3 state)",
            "config": {"workload": "op cases of configs 2 and 3, the int8 GEMV and the decode projection GEMMs"},
            "ops": cases, "gpu": torch.cuda.get_device_name()}


# ---------------------------------------------------------------------------------------------------------------
# config5: serving


def bench_config5(a, world, rank, local, stream, cfg, W):
    import torch
    import torch.distributed as dist
    import duo
    from duo import lib as L
    from duo import serve
    r0, r1 = serve.shard(rank, world, a.rows)
    rows = r1 - r0
    if a.rows % world:
        raise SystemExit("config5: the batch's rows must split evenly across the GPUs (one all_gather)")
    group_rows = max(1, min(rows, a.max_tokens // a.prompt))
    m = duo.Model(cfg, W, stream=stream)
    m.alloc(rows=rows, max_len=a.prompt + a.decode + 1, max_t=a.prompt, max_tokens=group_rows * a.prompt)
    batch_ids = serve.batch_prompts(a.rows, a.prompt, cfg.vocab_size, a.seed)
    ids_host = batch_ids[r0:r1].contiguous().pin_memory()
    ids_dev = ids_host.to("cuda")

    # dose unit of the steering vector: median residual norm after layer 12 over the batch's first prompt (token 0
    # skipped), measured with the engine's residual capture (analysis.js:52-77 does the same with `resid`); every
    # rank measures the same prompt, so every rank gets the same scale
    with torch.cuda.stream(stream):
        cap = m.capture_resid(a.vec_layer)
        m.reset_all()
        m.forward(batch_ids[0].to("cuda"), 0, 1, a.prompt)
        stream.synchronize()
        p50 = float(cap[1:a.prompt].norm(dim=-1).median())
        m.capture_resid(None)
    vecs = serve.batch_vectors(a.rows, cfg.hidden_size, 0.5 * p50, a.seed)[r0:r1]  # batch rows 0..127 carry one
    m.set_vectors(list(vecs))
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def prefill(host_io=False):
        for g0 in range(0, rows, group_rows):
            n = min(group_rows, rows - g0)
            src = ids_host[g0:g0 + n].reshape(-1).numpy() if host_io else ids_dev[g0:g0 + n].reshape(-1)
            m.forward(src, g0, n, a.prompt)

    def serve_step(host_io=False):
        """One step: fresh state, prefill every row group, decode, gather."""
        m.reset_all()
        e0, e1, e2 = ev(), ev(), ev()
        e0.record(stream)
        prefill(host_io)
        e1.record(stream)
        toks = m.generate(a.decode, vec=a.vec_layer)
        with torch.cuda.stream(stream):
            allt = serve.gather_rows(toks, world)  # [batch rows, decode]
        e2.record(stream)
        out = allt.to("cpu", non_blocking=False) if host_io else None
        return e0, e1, e2, out

    # warm-up (the first one with every kernel class profiled, per phase, to find the dominant kernel)
    phase_prof = {}
    for i in range(a.warmup):
        if i == 0:
            m.profile()
            m.reset_all()
            prefill()
            phase_prof["prefill"] = m.profile_read()
            m.generate(a.decode, vec=a.vec_layer)
            phase_prof["decode"] = m.profile_read()
            m.profile([])
            with torch.cuda.stream(stream):
                serve.gather_rows(torch.zeros(rows, a.decode, dtype=torch.int32, device="cuda"), world)
        else:
            serve_step()
    torch.cuda.synchronize()

    clocks = Clocks(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = L.lib().duo_launch_count()
    clocks.start()
    t_start, t_end = ev(), ev()
    t_start.record(stream)
    step_events = [serve_step()[:3] for _ in range(a.steps)]
    t_end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    launches = L.lib().duo_launch_count() - launches0
    total_ms = max_over_ranks(t_start.elapsed_time(t_end), world)
    pre_ms = statistics.mean(s[0].elapsed_time(s[1]) for s in step_events)
    dec_ms = statistics.mean(s[1].elapsed_time(s[2]) for s in step_events)
    value = a.rows * (a.prompt + a.decode) * a.steps / (total_ms / 1000)

    def run_dominant(dominant):
        if dominant[0] == "prefill":
            m.profile([dominant[1]])
            m.reset_all()
            prefill()
        else:
            m.profile([])
            m.reset_all()
            prefill()
            m.profile([dominant[1]])
            m.generate(a.decode, vec=a.vec_layer)
        d = m.profile_read()
        m.profile([])
        return d

    pk, pk_src = peaks()
    work = algorithmic_work(cfg, rows, a.prompt, a.decode)
    roof = roofline_of(m, phase_prof, work, run_dominant, pk, pk_src,
                       lambda k: measured_traffic(k, rows, a.prompt))
    if world > 1:
        dist.barrier()  # every rank ran the same profiled step

    e2e = None
    if not a.no_e2e:
        k2 = max(1, min(2, a.steps))
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        w0, w1 = ev(), ev()
        w0.record(stream)
        for _ in range(k2):
            serve_step(host_io=True)
        w1.record(stream)
        torch.cuda.synchronize()
        e_ms = max_over_ranks(w0.elapsed_time(w1), world)
        # per step: this rank's ids in (rows x prompt int32); out: the whole batch's gathered tokens
        e2e = {"value": a.rows * (a.prompt + a.decode) * k2 / (e_ms / 1000), "unit": "tok/s",
               "h2d_bytes_per_step": rows * a.prompt * 4, "d2h_bytes_per_step": a.rows * a.decode * 4, "steps": k2}
    line = {
        "metric": METRIC5, "value": value, "unit": "tok/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": total_ms / a.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded random ids, random-init weights)",
        "config": {"workload": "config5: one batch of 256 prompts x 2048 random ids + 512 greedy decode steps, int8 "
                               "weights (per-row absmax), bf16 activations, layer-12 vector on batch rows 0..127",
                   "rows_total": a.rows, "rows_per_gpu": rows, "prompt": a.prompt, "decode": a.decode,
                   "parallelism": f"dp{world} (the batch's rows split {rows} per GPU, no exchange in the forward; "
                                  "tokens gathered once per step)",
                   "prefill_tok_s": a.rows * a.prompt / (pre_ms / 1000),
                   "decode_tok_s": a.rows * a.decode / (dec_ms / 1000),
                   "l2": "inputs larger than L2 (state, KV cache and weights far exceed 126 MB)",
                   "prefill_rows_per_call": group_rows},
        "roofline": roof,
        "breakdown_ms": {ph: {k: round(v[0], 3) for k, v in d.items()} for ph, d in phase_prof.items()},
        "e2e": e2e, "gpu_launches": int(launches), "clocks": clk,
    }
    del m
    return line


# ---------------------------------------------------------------------------------------------------------------
# config4: batched push test


def bench_config4(a, world, rank, local, stream, cfg, W):
    import torch
    import torch.distributed as dist
    import duo
    from duo import lib as L
    from duo import ops, probe, serve
    n_units = a.cands * a.contexts
    if n_units % world:
        raise SystemExit("config4: the (candidate, context) triples must split evenly across the GPUs")
    u0, u1 = serve.triple_block(rank, world, a.cands, a.contexts)
    rows = 3 * (u1 - u0)
    cands, contexts, targets, tw = serve.probe_batch(a.cands, a.contexts, a.ctx_len, a.targets,
                                                     cfg.num_hidden_layers, cfg.intermediate_size, cfg.vocab_size,
                                                     a.seed)
    m = duo.Model(cfg, W, stream=stream)
    m.alloc(rows=rows, max_len=max(64, a.ctx_len) + 1, max_t=64, max_tokens=max(rows * a.ctx_len, 64))
    # dose units (analysis.js:52-110): median residual norm per layer over a seeded 64-id calibration prompt, over the
    # down_proj column norms of the candidates; identical on every rank
    calib = torch.randint(0, cfg.vocab_size, (64,), generator=torch.Generator().manual_seed(a.seed + 5)).tolist()
    with torch.cuda.stream(stream):
        p50 = probe.resid_p50(m, calib)
    units = [float(p50[l]) / max(float(probe.col_norms(W, l, [n])[0]), 1e-30) for l, n in cands]
    pairs = list(range(u0, u1))
    ids, pushes, base = probe.build_batch(cands, contexts, units, 0.8, pairs)
    ids_dev = torch.tensor(ids, dtype=torch.int32, device="cuda")
    base_t = torch.tensor(base, dtype=torch.int32, device="cuda")
    tid = torch.tensor(targets, dtype=torch.int32, device="cuda")
    logw = torch.tensor([math.log(w) for w in tw], dtype=torch.float32, device="cuda")
    logits = torch.empty(rows, cfg.vocab_size, dtype=torch.float32, device="cuda")
    stats = torch.empty(rows, L.DUO_STATS_COLS, dtype=torch.float32, device="cuda")
    m._set_pushes(pushes)  # the push tables stay in force for every step
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def step():
        m.reset_all()
        m._forward(ids_dev, 0, rows, a.ctx_len, {})  # the push tables set above stay in force
        L.call("duo_engine_logits", m._h, 0, rows, L.ptr(logits), L.stream_ptr(stream))
        L.call("duo_push_stats", L.ptr(logits), rows, cfg.vocab_size, L.ptr(base_t), L.ptr(tid), L.ptr(logw),
               len(targets), L.ptr(stats), None, L.stream_ptr(stream))
        with torch.cuda.stream(stream):
            all_stats = serve.gather_rows(stats, world)
            all_logits = serve.gather_rows(logits, world)
        return all_stats, all_logits

    phase_prof = {}
    for i in range(a.warmup):
        if i == 0:
            m.profile()
            step()
            phase_prof["prefill"] = m.profile_read()
            m.profile([])
        else:
            step()
    torch.cuda.synchronize()

    clocks = Clocks(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = L.lib().duo_launch_count()
    clocks.start()
    t_start, t_end = ev(), ev()
    t_start.record(stream)
    for _ in range(a.steps):
        step()
    t_end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    launches = L.lib().duo_launch_count() - launches0
    total_ms = max_over_ranks(t_start.elapsed_time(t_end), world)
    batch_rows = 3 * n_units
    value = batch_rows * a.ctx_len * a.steps / (total_ms / 1000)

    def run_dominant(dominant):
        m.profile([dominant[1]])
        step()
        d = m.profile_read()
        m.profile([])
        return d

    pk, pk_src = peaks()
    work = algorithmic_work(cfg, rows, a.ctx_len, 0)
    roof = roofline_of(m, phase_prof, work, run_dominant, pk, pk_src, lambda k: None)
    if world > 1:
        dist.barrier()

    e2e = None
    if not a.no_e2e:  # through the public API: probe.push_test from host ids, statistics read back to the host
        k2 = max(1, min(3, a.steps))
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        w0, w1 = ev(), ev()
        w0.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(k2):
                res = probe.push_test(m, cands, contexts, targets, tw, dose=0.8, units=units, pairs=pairs,
                                      summarize=False)
                serve.gather_rows(res["stats"], world).cpu()
        w1.record(stream)
        torch.cuda.synchronize()
        e_ms = max_over_ranks(w0.elapsed_time(w1), world)
        e2e = {"value": batch_rows * a.ctx_len * k2 / (e_ms / 1000), "unit": "tok/s",
               "h2d_bytes_per_step": rows * a.ctx_len * 4, "d2h_bytes_per_step": batch_rows * L.DUO_STATS_COLS * 4,
               "steps": k2}
    st = stats.double().cpu()
    line = {
        "metric": METRIC4, "value": value, "unit": "tok/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": total_ms / a.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded random ids, random-init weights)",
        "config": {"workload": f"config4: {a.cands} candidates x {a.contexts} contexts of {a.ctx_len} random ids x "
                               "strengths (+0.8, 0, -0.8) = one forward of "
                               f"{batch_rows} rows, next-token statistics vs the strength-0 row, {a.targets} "
                               "targets, int8 weights (per-row absmax), bf16 activations",
                   "rows_total": batch_rows, "rows_per_gpu": rows, "rows_per_s": batch_rows * a.steps / (total_ms / 1000),
                   "parallelism": f"dp{world} (whole (candidate, context) triples per GPU; statistics and logits "
                                  "gathered once per step)",
                   "kl_mean_rank0": float(st[[i for i in range(rows) if i % 3 != 1], 3].mean()),
                   "l2": "logits (216 x 248320 f32 = 214 MB) and weights exceed L2"},
        "roofline": roof,
        "breakdown_ms": {ph: {k: round(v[0], 3) for k, v in d.items()} for ph, d in phase_prof.items()},
        "e2e": e2e, "gpu_launches": int(launches), "clocks": clk,
    }
    del m
    return line


# ---------------------------------------------------------------------------------------------------------------


def main():
    a = parse()
    if a.impl == "reference":
        return run_reference(a)
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    import duo
    from duo.weights import random_weights
    cfg = duo.qwen35_0p8b(group=0, act_dtype="bf16")
    W = random_weights(cfg, seed=a.seed)
    stream = torch.cuda.Stream()
    if a.workload == "ops":
        if rank == 0:
            print(json.dumps(bench_ops(a)), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return 0
    line = (bench_config4 if a.workload == "config4" else bench_config5)(a, world, rank, local, stream, cfg, W)
    if a.workload == "config5" and rank == 0 and world == 1 and not a.no_ops:
        del W
        torch.cuda.empty_cache()
        line["ops"] = op_cases(full=False)  # config 2 / 3 / int8 GEMV cases, timed after the step (not in `value`)

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        ref = CpuReference(a.seed)
        (ref.sample4 if a.workload == "config4" else ref.sample5)()  # warm the allocator and kernels
        v, dt = (ref.sample4 if a.workload == "config4" else ref.sample5)()
        desc = (f"{CPU_SAMPLE4[0]} candidates x {CPU_SAMPLE4[1]} contexts x 3 strengths x {CPU_SAMPLE4[2]} ids"
                if a.workload == "config4" else
                f"{CPU_SAMPLE5[0]} prompts x {CPU_SAMPLE5[1]} ids + {CPU_SAMPLE5[2]} greedy steps (4:1 mix)")
        cpu = {"value": v, "unit": "tok/s", "cores": ref.cores, "kind": "reference",
               "sample": f"{desc}, transformers fp32 on {cpu_desc()} ({dt:.1f} s)"}
    if rank == 0:
        line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
