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
    ap.add_argument("--workload", choices=["config5", "config4"], default="config5")
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
    line = (bench_config4 if a.workload == "config4" else bench_config5)(a, world, rank, local, stream, cfg, W)

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
