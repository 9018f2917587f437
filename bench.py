"""bench.py -- prefill + decode tok/s of the Qwen3.5-0.8B-shaped engine on 1..8 B200s.

Workload ("throughput serving"): 256 independent prompts of 2048 random token ids, then 512 greedy
decode steps; int8 weights with one scale per output row, bf16 activations; rows 0..127 carry a random layer-12
residual steering vector N(0,1) * 0.5 * median residual norm.  Random-init weights of the 0.8B architecture
(transformers' init distributions), synthetic seeded ids.  Rows are independent, so the batch is sharded by rows
across the ranks with no exchange in the forward (weak scaling: each rank serves its own 256-row batch, seeded by
rank); the generated tokens of all ranks are gathered with one NCCL all_gather at the end of each step.  One step =
one full serve of every rank's batch (reset, prefill, 512 decode steps, gather).

    python bench.py [--gpus N --steps K --warmup W]          # our engine (one JSON line on rank 0)
    python bench.py --impl reference [--steps K --warmup W]   # the reference's CPU PyTorch path, bounded sample
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "duo-mech-interp_b200"))

METRIC = "prefill+decode tok/s, Qwen3.5-0.8B shape (256 x 2048 prompt + 512 greedy decode)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["duo", "reference"], default="duo")
    ap.add_argument("--rows", type=int, default=256)
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--decode", type=int, default=512)
    ap.add_argument("--max-tokens", type=int, default=131072, help="tokens per prefill forward call")
    ap.add_argument("--vec-layer", type=int, default=12)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    return ap.parse_args()


# ---------------------------------------------------------------------------------------------------------------
# the reference's CPU path (transformers Qwen3_5ForCausalLM, fp32), timed on a bounded sample


# the bounded CPU sample: 8 prompts x 1024 ids + 16 greedy steps (about 15 s of work on 16 host cores)
CPU_SAMPLE = (8, 1024, 16)


def cpu_reference_sample(rows=2, prompt=256, decode=8, seed=0):
    """tok/s of the reference's PyTorch forward on the host cores for `rows` prompts of `prompt` ids plus `decode`
    greedy steps (the same per-token work as the GPU workload, on a slice of it)."""
    import torch
    sys.path.insert(0, ROOT)
    from oracle import hf
    from oracle.model import Cfg
    torch.set_num_threads(os.cpu_count() or 1)
    model = hf.build_model_fast(Cfg(), seed=seed)
    ids = torch.randint(0, 248320, (rows, prompt), generator=torch.Generator().manual_seed(seed))
    hf.prefill_and_greedy(model, ids[:, :16], 1)  # warm the allocator / kernels
    t0 = time.perf_counter()
    hf.prefill_and_greedy(model, ids, decode)
    dt = time.perf_counter() - t0
    return rows * (prompt + decode) / dt, dt, torch.get_num_threads()


def cpu_desc():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown CPU"


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    rows, prompt, decode = CPU_SAMPLE
    for _ in range(a.warmup):
        pass  # each sample builds its own cache; the model build below is the warm-up
    vals = []
    secs = []
    for _ in range(max(1, a.steps)):
        v, dt, cores = cpu_reference_sample(rows, prompt, decode, a.seed)
        vals.append(v)
        secs.append(dt)
    v = statistics.median(vals)
    import torch
    import transformers
    sample = (f"{rows} prompts x {prompt} ids + {decode} greedy steps of the 0.8B shape, fp32, "
              f"transformers {transformers.__version__} / torch {torch.__version__}, {cpu_desc()}")
    line = {"metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": 1000 * statistics.median(secs), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random ids, random-init weights)",
            "impl": "reference",
            "config": {"workload": "config5 slice on the host CPU (the reference's PyTorch path)", "rows": rows,
                       "prompt": prompt, "decode": decode},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "reference", "sample": sample},
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
# our engine


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
    # prefill GEMMs: 2 * tokens * layer parameters (tensor)
    w[("prefill", "gemm")] = ("tensor", 2.0 * rows * prompt * layer_params)
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
    from duo import lib as L
    from duo import serve as rowshard
    from duo.weights import random_weights

    cfg = duo.qwen35_0p8b(group=0, act_dtype="bf16")
    rows = a.rows  # per rank (weak scaling)
    group_rows = max(1, min(rows, a.max_tokens // a.prompt))
    W = random_weights(cfg, seed=a.seed)
    stream = torch.cuda.Stream()
    m = duo.Model(cfg, W, stream=stream)
    m.alloc(rows=rows, max_len=a.prompt + a.decode + 1, max_t=a.prompt, max_tokens=group_rows * a.prompt)
    ids_host = rowshard.rank_prompts(rank, rows, a.prompt, cfg.vocab_size, a.seed).pin_memory()
    ids_dev = ids_host.to("cuda")

    # dose unit of the steering vector: median residual norm after layer 12 over a calibration prompt (token 0
    # skipped), measured with the engine's residual capture (analysis.js:52-77 does the same with `resid`)
    with torch.cuda.stream(stream):
        cap = m.capture_resid(a.vec_layer)
        m.reset_all()
        m.forward(ids_dev[0], 0, 1, a.prompt)
        stream.synchronize()
        p50 = float(cap[1:a.prompt].norm(dim=-1).median())
        m.capture_resid(None)
    vecs = rowshard.rank_vectors(rank, rows, cfg.hidden_size, 0.5 * p50, a.seed)  # rows 0..127 carry the vector
    m.set_vectors(list(vecs))

    tokens = torch.empty(rows, a.decode, dtype=torch.int32, device="cuda")
    gathered = None
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def serve(host_io=False):
        """One step: fresh state, prefill every row group, decode, gather."""
        m.reset_all()
        e0, e1, e2 = ev(), ev(), ev()
        e0.record(stream)
        for g0 in range(0, rows, group_rows):
            n = min(group_rows, rows - g0)
            src = ids_host if host_io else ids_dev
            m.forward(src[g0:g0 + n].reshape(-1) if not host_io else src[g0:g0 + n].reshape(-1).numpy(), g0, n,
                      a.prompt)
        e1.record(stream)
        toks = m.generate(a.decode, vec=a.vec_layer)
        with torch.cuda.stream(stream):
            allt = rowshard.gather_rows(toks, world)  # [world, rows, decode]
        e2.record(stream)
        out = None
        if host_io:
            out = allt.to("cpu", non_blocking=False)
        return e0, e1, e2, out

    pk, pk_src = peaks()
    # warm-up (the first one with every kernel class profiled, per phase, to find the dominant kernel)
    phase_prof = {}
    for i in range(a.warmup):
        if i == 0:
            m.profile()
            m.reset_all()
            for g0 in range(0, rows, group_rows):
                n = min(group_rows, rows - g0)
                m.forward(ids_dev[g0:g0 + n].reshape(-1), g0, n, a.prompt)
            phase_prof["prefill"] = m.profile_read()
            m.generate(a.decode, vec=a.vec_layer)
            phase_prof["decode"] = m.profile_read()
            m.profile([])
        else:
            serve()
    torch.cuda.synchronize()
    work = algorithmic_work(cfg, rows, a.prompt, a.decode)
    # the class with the most device time among those with a defined algorithmic work
    dominant = max(((ph, k) for ph in phase_prof for k in phase_prof[ph] if (ph, k) in work),
                   key=lambda pk_: phase_prof[pk_[0]][pk_[1]][0])

    # timed region: K steps between barrier + synchronize; the dominant class is timed per launch with events
    clocks = Clocks(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = L.lib().duo_launch_count()
    clocks.start()
    t_start, t_end = ev(), ev()
    t_start.record(stream)
    step_events = []
    for _ in range(a.steps):
        e0, e1, e2, _ = serve()
        step_events.append((e0, e1, e2))
    t_end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    launches = L.lib().duo_launch_count() - launches0
    total_ms = t_start.elapsed_time(t_end)
    pre_ms = statistics.mean(s[0].elapsed_time(s[1]) for s in step_events)
    dec_ms = statistics.mean(s[1].elapsed_time(s[2]) for s in step_events)
    t = torch.tensor([total_ms], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    tokens_total = world * rows * (a.prompt + a.decode) * a.steps
    value = tokens_total / (total_ms / 1000)

    # live per-launch timing of the dominant kernel class (one more step, profiled for that class only)
    m.profile([dominant[1]])
    m.reset_all()
    if dominant[0] == "prefill":
        for g0 in range(0, rows, group_rows):
            n = min(group_rows, rows - g0)
            m.forward(ids_dev[g0:g0 + n].reshape(-1), g0, n, a.prompt)
        dprof = m.profile_read()
    else:
        m.profile([])
        for g0 in range(0, rows, group_rows):
            n = min(group_rows, rows - g0)
            m.forward(ids_dev[g0:g0 + n].reshape(-1), g0, n, a.prompt)
        m.profile([dominant[1]])
        m.generate(a.decode, vec=a.vec_layer)
        dprof = m.profile_read()
    m.profile([])
    dom_ms, dom_n = dprof.get(dominant[1], (float("nan"), 1))
    bound, units = work.get(dominant, ("hbm", float("nan")))
    per_launch = units / max(dom_n, 1)
    avg_s = dom_ms / max(dom_n, 1) / 1000
    if bound == "tensor":
        achieved = per_launch / avg_s / 1e12
        peak = pk.get("bf16_tflops_sustained" if dominant[0] == "prefill" else "bf16_tflops")
        unit = "TFLOP/s"
    else:
        achieved = per_launch / avg_s / 1e9
        peak = pk.get("hbm_gbs")
        unit = "GB/s"

    traffic = measured_traffic(f"{dominant[0]}:{dominant[1]}", rows, a.prompt)

    # end to end through the public API with host buffers (ids from pinned host memory, tokens back to the host)
    e2e = None
    if not a.no_e2e:
        k2 = max(1, min(2, a.steps))
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        w0, w1 = ev(), ev()
        w0.record(stream)
        for _ in range(k2):
            serve(host_io=True)
        w1.record(stream)
        torch.cuda.synchronize()
        e_ms = w0.elapsed_time(w1)
        te = torch.tensor([e_ms], device="cuda")
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        # per rank and step: its ids in (rows x prompt int32); out: every rank's gathered tokens (world x rows x decode)
        e2e = {"value": world * rows * (a.prompt + a.decode) * k2 / (float(te.item()) / 1000), "unit": "tok/s",
               "h2d_bytes_per_step": rows * a.prompt * 4, "d2h_bytes_per_step": world * rows * a.decode * 4,
               "steps": k2}

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        v, dt, cores = cpu_reference_sample(*CPU_SAMPLE, a.seed)
        cpu = {"value": v, "unit": "tok/s", "cores": cores, "kind": "reference",
               "sample": f"{CPU_SAMPLE[0]} prompts x {CPU_SAMPLE[1]} ids + {CPU_SAMPLE[2]} greedy steps, transformers fp32 "
                         f"on {cpu_desc()} ({dt:.1f} s)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": total_ms / a.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random ids, random-init weights)",
            "config": {"workload": "config5: 256 prompts x 2048 random ids + 512 greedy decode steps per GPU, int8 "
                                   "weights (per-row absmax), bf16 activations, layer-12 vector on rows 0..127",
                       "rows_per_gpu": rows, "rows_total": world * rows, "prompt": a.prompt, "decode": a.decode,
                       "parallelism": f"dp{world} (rows sharded, no exchange; tokens gathered once per step)",
                       "prefill_tok_s": world * rows * a.prompt / (pre_ms / 1000),
                       "decode_tok_s": world * rows * a.decode / (dec_ms / 1000),
                       "l2": "inputs larger than L2 (state, KV cache and weights far exceed 126 MB)",
                       "prefill_rows_per_call": group_rows},
            "roofline": {"kernel": f"{dominant[0]}:{dominant[1]}", "bound": bound, "achieved": achieved,
                         "peak": peak, "unit": unit, "frac": achieved / peak if peak else None, "traffic": traffic,
                         "peak_source": pk_src, "launches": dom_n, "avg_launch_ms": dom_ms / max(dom_n, 1)},
            "breakdown_ms": {ph: {k: round(v[0], 3) for k, v in d.items()} for ph, d in phase_prof.items()},
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": int(launches), "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    del m
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
