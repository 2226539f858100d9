#!/usr/bin/env python3
"""Batch-1 greedy decode of the Granite-3B-A800M-shaped MoE model on B200.

Workload (default, --workload c3): 32 layers, hidden 1536, 24 q / 8 kv heads (d 64), 40 experts top-8 (I 512),
vocab 49155, random-init bf16 weights (synthetic generator, seed 2, std 0.02), KV cache pre-filled to 2048 positions
by feeding 2048 uniform random ids (seed 2) through the model itself in multi-position steps of 32, then greedy
decode.  One bench step = one
decoded token.  --workload c4: the same architecture with every linear weight Q8_0 (int8 ~U[-127,127] and one fp16
scale ~U(1e-4, 4e-3) per 32 values; embedding bf16), seeds 4, context 512.

Under torchrun (WORLD_SIZE set) the default workload is c5 at every world size: 64 sequences in total (strong
scaling), experts partitioned over the ranks; a plain `python bench.py` runs c3.

  value  device-resident throughput: K graph-replayed decode steps, the token fed back on the device, timed with
         CUDA events on the library's stream (max over ranks; every rank decodes its own replica: batch-1 decode
         does not shard, so N GPUs run N independent replicas = weak scaling)
  e2e    the same decode through the public C-ABI step call a user makes (lastro_model_step): the token goes
         host->device and the next token device->host every step, inside the timed region
  roofline  the dominant kernel of the step (by its share of the step's critical path in the replayed graph):
         algorithmic bytes per launch / its in-graph duration (first CTA start to last CTA exit, every CTA stamping
         %globaltimer in a graph captured like the product's, lastro_model_trace).  --fused runs the step as one
         persistent kernel instead of the per-layer chain; its roofline is then the whole step's bytes / its duration
  cpu_baseline  the CPU oracle (a C restatement of the reference's CPU path, rust/moe-rt/src/{cpu,model}.rs)
         decoding the same model at the same context on this host's cores

--impl reference times that CPU path as the reference arm (the reference itself is Rust + cuTile and cannot be
built here: no cargo, no network).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "lastro-rust_b200"))

from lastro_b200 import configs as CFG  # noqa: E402

KERNELS = ("qkv_rope", "attention", "oproj", "router", "gate_up", "down", "head", "fused_step", "moe")
WORKLOADS = {"c3": CFG.C3_3B, "c4": CFG.C4_3B_Q8, "c5": CFG.C5_BATCH}


def metric_name(c, context):
    q8 = c["model"].get("weight_dtype") == "q8_0"
    return f"decode tok/s (bs1) Granite-3B-A800M shape{' Q8_0' if q8 else ''}, ctx {context}"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", choices=("lastro", "reference"), default="lastro")
    ap.add_argument("--workload", choices=tuple(WORKLOADS), default=None,
                    help="c3: bf16 weights, ctx 2048 (the headline; the default of a plain `python bench.py`); c4: "
                         "Q8_0 weights, ctx 512; c5: 64 sequences x ctx 1024, Zipf expert load, experts partitioned "
                         "over the torchrun ranks (the default under torchrun, at every world size including 1)")
    ap.add_argument("--context", type=int, default=None, help="context length (default: the workload's)")
    ap.add_argument("--kv", choices=("bf16", "f32"), default="bf16")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="bounded CPU-baseline sample")
    ap.add_argument("--profile-only", action="store_true", help="small run for ncu: synthetic KV + 3 decode steps")
    ap.add_argument("--synthetic-kv", action="store_true", help="fill the context with synthetic K/V instead of "
                    "decoding the prompt through the model")
    ap.add_argument("--layers", type=int, default=0, help="with --profile-only: a 3B-shaped model with this many "
                    "layers (small ncu captures; the kernels are those of the full model)")
    ap.add_argument("--placement", choices=("balanced", "interleaved", "contiguous"), default="balanced",
                    help="c5 on N > 1 GPUs: experts over ranks, balanced over the pair counts of the first step "
                    "(greedy, E/N per rank), e mod N, or contiguous blocks")
    ap.add_argument("--gemm", type=int, default=2, choices=(0, 1, 2), help="c5 GEMMs: 2 tcgen05 warp-specialised "
                    "(TMA weight tiles), 1 tcgen05 with all-thread cp.async stages, 0 mma.sync")
    ap.add_argument("--fused", action="store_true", help="the fused step kernel (one persistent launch per step) instead "
                    "of the per-layer kernel chain")
    a = ap.parse_args()
    if a.workload is None:
        # under torchrun the driver measures scaling: the expert-parallel batched decode (strong scaling, 64 sequences
        # in total at every N); a single process measures the batch-1 headline
        a.workload = "c5" if under_torchrun() else "c3"
    if a.context is None:
        a.context = WORKLOADS[a.workload]["context"]
    return a


def under_torchrun():
    return "WORLD_SIZE" in os.environ or "TORCHELASTIC_RUN_ID" in os.environ


def workload_config(a):
    """The `config` object, identical in both arms for the same workload (the run's own measurements go elsewhere)."""
    c = WORKLOADS[a.workload]
    return {"workload": c["name"], "batch": c.get("batch", 1), "context": a.context, "kv_cache": f"paged {a.kv}",
            "weights": c["model"].get("weight_dtype", "bf16")}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def kernel_bytes(cfg, context):
    """Algorithmic HBM bytes of one launch of each kernel (bf16 or Q8_0 linear weights, bf16 KV and embedding), at
    the given mean context."""
    H, I, E, k, V = cfg["hidden"], cfg["inter"], cfg["experts"], cfg["k"], cfg["vocab"]
    qd, kvd = cfg["heads"] * cfg["head_dim"], cfg["kv_heads"] * cfg["head_dim"]
    wb = CFG.weight_bytes(cfg)
    kb = dict(qkv_rope=(qd + 2 * kvd) * H * wb + 2 * kvd * 2, attention=2 * kvd * 2 * context,
              oproj=H * qd * wb + H * E * 4, router=0, gate_up=k * 2 * I * H * wb, down=k * H * I * wb,
              head=V * H * 2)
    kb["moe"] = kb["gate_up"] + kb["down"]  # the one-launch MoE block streams both
    # the fused step kernel moves every layer's bytes and the head's in one launch
    kb["fused_step"] = cfg["layers"] * sum(kb[n] for n in ("qkv_rope", "attention", "oproj", "gate_up", "down")) + kb["head"]
    return kb


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.flush()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], 0.0, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
                for n, v in zip(names, r[5:9]):
                    if "Active" in v and "Not" not in v:
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_decode_rate(cfg, context, seed, seconds, steps=None, warmup=1):
    """The oracle (reference CPU path restated) decoding at `context`: returns (tok/s, threads, tokens, sample)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    threads = os.cpu_count() or 1
    t0 = time.time()
    om = O.Model(cfg, synthetic_seed=seed, std=CFG.WEIGHT_STD, norm_std=0.0, threads=threads)
    pool = O.Pool(threads)
    n_max = (steps or 256) + warmup + 2
    s = O.Session(om, pool, context + n_max)
    s.fill_kv(context, seed, 0.5)
    setup = time.time() - t0
    tok = CFG.synthetic_tokens(1, seed, cfg["vocab"])[0]
    for _ in range(warmup):
        lg, _, _ = s.step(tok)
        tok = O.argmax_last(lg)
    n, t1 = 0, time.time()
    while True:
        lg, _, _ = s.step(tok)
        tok = O.argmax_last(lg)
        n += 1
        el = time.time() - t1
        if (steps is not None and n >= steps) or (steps is None and (el >= seconds or n >= 256)):
            break
    s.close()
    om.close()
    pool.close()
    sample = (f"{n} greedy decode steps of the full {cfg['layers']}-layer model at context {context}-{context + n}"
              f" (K/V rows synthetic), weights from the same generator; setup {setup:.1f} s untimed")
    return n / el, threads, n, sample


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    c = WORKLOADS[a.workload]
    cfg = c["model"]
    if a.workload == "c5":
        rate, threads, n, sample = cpu_batched_rate(cfg, a.context, c, steps=min(a.steps, 2))
    else:
        rate, threads, n, sample = cpu_decode_rate(cfg, a.context, c["weight_seed"], 0, steps=a.steps,
                                                   warmup=min(a.warmup, 2))
    line = {
        "impl": "reference", "metric": metric_name(c, a.context) if a.workload != "c5" else BATCH_METRIC, "value": rate,
        "unit": "tok/s", "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1000.0 / rate,
        "higher_is_better": True, "scaling": "strong" if a.workload == "c5" else "weak", "vs_baseline": None,
        "dtype": cfg.get("weight_dtype", "bf16"), "data": "synthetic",
        "config": workload_config(a),
        "cpu_baseline": {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": rate, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference (Rust + cuTile, rust/moe-rt) cannot be built here; its CPU path is timed through the "
                "C restatement in oracle/ with all host threads",
    }
    print(json.dumps(line), flush=True)
    return 0


BATCH_METRIC = "decode tok/s (bs64) Granite-3B-A800M shape, ctx 1024, Zipf(0.8) expert load"


def cpu_batched_rate(cfg, context, c, steps=2, seqs=4):
    """The oracle decoding `seqs` of the batch's sequences (each its own session: a CPU path has no batching, its
    tokens/s is the per-token rate) at `context` with the Zipf router bias: (tok/s, threads, tokens, sample)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    threads = os.cpu_count() or 1
    om = O.Model(cfg, synthetic_seed=c["weight_seed"], std=CFG.WEIGHT_STD, norm_std=0.0, threads=threads)
    om.set_router_bias(CFG.zipf_router_bias(cfg))
    pool = O.Pool(threads)
    ss = [O.Session(om, pool, context + steps + 2) for _ in range(seqs)]
    for q, s in enumerate(ss):
        s.fill_kv(context, c["prompt_seed"] + q, 0.5)
    toks = CFG.synthetic_tokens(seqs, c["prompt_seed"], cfg["vocab"])
    n, t0 = 0, time.time()
    for _ in range(steps):
        for q, s in enumerate(ss):
            lg, _, _ = s.step(toks[q])
            toks[q] = O.argmax_last(lg)
            n += 1
    el = time.time() - t0
    for s in ss:
        s.close()
    om.close()
    pool.close()
    sample = (f"{n} tokens: {seqs} sequences x {steps} greedy steps of the full model at context {context} (K/V rows "
              "synthetic), one CPU session per sequence")
    return n / el, threads, n, sample


def run_batched(a):
    """C5: 64 sequences (64/N per rank) with 1024-token contexts decode together; every layer's MoE pairs go to the
    rank that owns their expert (experts 40/N per rank, placed by --placement) through the peer-memory exchange."""
    import torch
    import torch.distributed as dist

    import lastro_b200 as LB
    from lastro_b200 import ep as EP

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    c = CFG.C5_BATCH
    cfg = c["model"]
    K, W = a.steps, a.warmup
    if a.profile_only:  # small run for ncu: a 3B-shaped model with --layers layers, synthetic contexts, 2 steps
        cfg = dict(cfg, layers=a.layers or 2)
        K, W = 2, 1
        a.synthetic_kv = True
    total = c["batch"]
    mine = list(CFG.shard(total, rank, world))
    n = len(mine)
    stream = torch.cuda.Stream()
    ctx = LB.Context(local, stream.cuda_stream)
    model = LB.GpuModel(ctx, cfg, 8, kv_dtype=a.kv)
    model.fill_synthetic(c["weight_seed"], CFG.WEIGHT_STD, 0.0)
    max_len = a.context + W + 2 * K + 16
    batch = LB.GpuBatch(model, n, max_len, rank, world)
    if world > 1:
        handles = [None] * world
        dist.all_gather_object(handles, batch.exchange_handle())
        batch.connect(handles)
    else:
        batch.connect()
    batch.set_router_bias(CFG.zipf_router_bias(cfg))
    batch.set_options(gemm=a.gemm)
    seqs = list(range(n))
    t0 = time.time()
    if a.synthetic_kv:
        for q in seqs:
            batch.fill_kv_synthetic(q, a.context, c["prompt_seed"] + mine[q], 0.5)
        toks = [int(t) for t in CFG.synthetic_tokens(n, c["prompt_seed"] + 7 * rank, cfg["vocab"])]
    else:
        prompts = [CFG.synthetic_tokens(a.context, c["prompt_seed"] + g, cfg["vocab"]) for g in mine]
        for t in range(a.context):  # teacher-forced prefill of the contexts, one batched step per position
            nxt, _, _ = batch.step(seqs, [p[t] for p in prompts])
        toks = [int(x) for x in nxt]
    prefill_s = time.time() - t0
    if a.profile_only:
        batch.decode(seqs, toks, K, want_ids=False)
        ctx.synchronize()
        batch.close()
        model.close()
        ctx.close()
        if world > 1:
            dist.destroy_process_group()
        print(json.dumps({"profile_only": True, "layers": cfg["layers"], "rank": rank}))
        return 0
    # expert load of one step: share of the token-expert pairs each rank's experts receive (all ranks' tokens)
    nxt, _, routes = batch.step(seqs, toks, want_routes=True)
    toks = [int(x) for x in nxt]
    counts = np.bincount(routes.ravel(), minlength=cfg["experts"]).astype(np.int64)
    if world > 1:
        tc = torch.tensor(counts, device="cuda")
        dist.all_reduce(tc)
        counts = tc.cpu().numpy()
    if a.placement == "balanced":
        owner = EP.balanced_placement(counts, world)
    elif a.placement == "interleaved":
        owner = EP.interleaved_placement(cfg["experts"], world)
    else:
        owner = EP.contiguous_placement(cfg["experts"], world)
    if world > 1:
        batch.set_expert_placement(owner)  # the same on every rank (counts were all-reduced)
    batch.decode(seqs, toks, W, want_ids=False)
    toks = [int(x) for x in batch.decode(seqs, toks, 1)[-1]]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx0 = batch.position(0)
    ev0.record(stream)
    ids = batch.decode(seqs, toks, K)
    ev1.record(stream)
    stream.synchronize()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    toks = [int(x) for x in ids[-1]]
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    value = total * K / (ms / 1000.0)
    # end to end through the public step call: token ids host -> device, next ids device -> host, every step
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    e0.record(stream)
    for _ in range(K):
        nxt, _, _ = batch.step(seqs, toks)
        toks = [int(x) for x in nxt]
    e1.record(stream)
    stream.synchronize()
    e2e_ms = max(e0.elapsed_time(e1), (time.perf_counter() - w0) * 1000.0)
    if world > 1:
        t = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    prof = batch.profile(seqs, toks, 2)
    # in the replayed graph (the step's own regime): each kind's share of the step's critical path, every rank
    tr = batch.trace(seqs, toks, 3)
    exposed = {k: round(v, 4) for k, v in tr["exposed"].items() if v > 0}
    if world > 1:  # the slowest rank's figures
        t = torch.tensor([tr["step_ms"]], device="cuda")
        gathered = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(gathered, t)
        slow = int(torch.stack(gathered).argmax().item())
        ex = torch.tensor([tr["exposed"][k] for k in batch.KERNELS], device="cuda")
        dist.broadcast(ex, src=slow)
        exposed = {k: round(float(v), 4) for k, v in zip(batch.KERNELS, ex.tolist()) if v > 0}
    mean_ctx = ctx0 + (K + 1) / 2.0
    H, I, L, E, kk = cfg["hidden"], cfg["inter"], cfg["layers"], cfg["experts"], cfg["k"]
    qd, kvd = cfg["heads"] * cfg["head_dim"], cfg["kv_heads"] * cfg["head_dim"]
    touched = int((counts > 0).sum())
    expert_b = L * touched * 3 * I * H * 2
    kv_b = L * total * 2 * kvd * 2 * mean_ctx
    dense_b = L * ((qd + 2 * kvd) * H + H * qd + E * H) * 2 + cfg["vocab"] * H * 2
    step_bytes = expert_b + kv_b + world * dense_b  # every rank streams the replicated dense weights
    step_s = ms / 1000.0 / K
    hbm, peak_kind = peaks()
    achieved = step_bytes / world / step_s / 1e9  # per GPU
    share = [float(counts[EP.owned(owner, r)].sum() / counts.sum()) for r in range(world)]
    line = {
        "metric": BATCH_METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": workload_config(a),
        "run": {"seqs_per_rank": n, "context_start": ctx0, "mean_context": mean_ctx,
                "parallelism": f"ep{world}: experts {E // world}/rank ({a.placement} placement), attention "
                "data-parallel over sequences" if world > 1 else "single GPU",
                "weights": "bf16; batched GEMMs on tensor cores (" + ("mma.sync", "tcgen05, cp.async stages",
                           "tcgen05 warp-specialised, TMA weight tiles")[a.gemm] + ", accumulators f32, bf16 operands, "
                           "activations split hi + lo)",
                "expert_load_share_by_rank": [round(x, 4) for x in share], "experts_touched": touched,
                "router_bias": "Zipf(0.8), beta 0.8", "prefill": "synthetic KV" if a.synthetic_kv else
                "teacher-forced batched steps", "prefill_s": round(prefill_s, 2),
                "l2": f"inputs larger than L2: every step streams ~{step_bytes / 1e9:.1f} GB (L2 126 MB)"},
        "roofline": {"bound": "hbm", "kernel": "batched step (all kernels)", "achieved": achieved, "peak": hbm,
                     "unit": "GB/s", "frac": achieved / hbm, "peak_kind": peak_kind, "traffic": None,
                     "bytes_per_step": step_bytes, "bytes_note": "touched experts + KV of all sequences + the dense "
                     "weights every rank streams; per GPU"},
        "kernels_ms_per_step": {k: round(v, 4) for k, v in prof.items()},
        "in_graph_exposed_ms_per_step": exposed,
        "e2e": {"value": total * K / (e2e_ms / 1000.0), "unit": "tok/s", "h2d_bytes_per_step": 8 * n,
                "d2h_bytes_per_step": 4 * n},
        "gpu_launches": K * (L * 8 + 3),  # norm; 8 kernels per layer; lm_head, argmax
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        rate, threads, nt, sample = cpu_batched_rate(cfg, a.context, c)
        line["cpu_baseline"] = {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample}
    batch.close()
    model.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def main():
    a = parse()
    if a.impl == "reference":
        return run_reference(a)
    if a.workload == "c5":
        return run_batched(a)

    import torch
    import torch.distributed as dist

    import lastro_b200 as LB

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    c = WORKLOADS[a.workload]
    cfg = c["model"]
    q8 = cfg.get("weight_dtype") == "q8_0"
    if a.layers:
        assert a.profile_only, "--layers is for profiling captures only"
        cfg = dict(cfg, layers=a.layers)
    K, W = a.steps, a.warmup
    if a.profile_only:
        K, W = 2, 1
    stream = torch.cuda.Stream()
    ctx = LB.Context(local, stream.cuda_stream)
    max_len = a.context + 2 * (K + W) + 64
    model = LB.GpuModel(ctx, cfg, max_len, kv_dtype=a.kv)
    model.set_options(fused=a.fused)
    model.fill_synthetic(c["weight_seed"], CFG.WEIGHT_STD, 0.0)
    t0 = time.time()
    if a.synthetic_kv or a.profile_only:
        model.fill_kv_synthetic(a.context, c["prompt_seed"], 0.5)
    else:
        prompt = CFG.synthetic_tokens(a.context, c["prompt_seed"], cfg["vocab"])
        if q8:  # the multi-position step runs bf16 weights: Q8_0 prompts go through the decode step
            model.generate(prompt, 1)
        else:  # multi-position steps of 32 positions (lastro_model_step_positions), untimed
            model.prefill(prompt, 32)
    prefill_s = time.time() - t0
    if a.profile_only:
        model.decode(K)
        ctx.synchronize()
        print(json.dumps({"profile_only": True, "prefill_s": prefill_s}))
        return 0

    # ---- device-resident decode ------------------------------------------------------------------------------
    model.decode(W)
    ctx.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx0 = model.pos
    ev0.record(stream)
    model.decode(K)
    ev1.record(stream)
    stream.synchronize()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    mean_ctx = ctx0 + (K + 1) / 2.0
    value = world * K / (ms / 1000.0)

    # ---- end to end through the C-ABI step call (host token in, host token out) -----------------------------
    tok = int(CFG.synthetic_tokens(1, 99, cfg["vocab"])[0])
    for _ in range(W):
        _, tok, _, _ = model.step(tok, want_logits=False, want_routes=False)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    e0.record(stream)
    for _ in range(K):
        _, tok, _, _ = model.step(tok, want_logits=False, want_routes=False)
    e1.record(stream)
    stream.synchronize()
    wall_ms = (time.perf_counter() - w0) * 1000.0
    e2e_ms = max(e0.elapsed_time(e1), wall_ms)
    if world > 1:
        t = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = {"value": world * K / (e2e_ms / 1000.0), "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4}

    # ---- per-kernel device time -------------------------------------------------------------------------------
    # in the replayed graph (the step's own regime): every CTA stamps the global timer; exposed = each kind's share of
    # the step's critical path, span = first CTA start to last CTA exit of each launch
    L = cfg["layers"]
    launches = {k: (1 if k in ("head", "fused_step") else L) for k in KERNELS}
    fused = model.fused
    tr = None if fused else model.trace(4)
    # direct launches with an event between kernels (no PDL overlap): the serialised per-kernel figure
    prof = model.profile(4)
    prof_ctx = model.pos - 2
    kb = kernel_bytes(cfg, prof_ctx)
    hbm, peak_kind = peaks()
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if fused:
        dominant = "fused_step"
        per_launch_ms = prof[dominant]
        regime = "direct launch, CUDA events"
    else:
        dominant = max(("qkv_rope", "attention", "oproj", "gate_up", "down", "head", "moe"),
                       key=lambda k: tr["exposed"][k])
        per_launch_ms = tr["span"][dominant] / launches[dominant]
        regime = "in graph: first CTA start to last CTA exit, %globaltimer, mean over launches and 4 steps"
    achieved = kb[dominant] / (per_launch_ms / 1000.0) / 1e9
    if os.path.exists(tp):  # per workload: c3 bf16, c4 Q8_0 (half the weight bytes)
        traffic = json.load(open(tp)).get(a.workload, {}).get(dominant)
    # the router GEMV runs inside the oproj kernel; the MoE block's streamed bytes are the experts'
    moe_bytes = kb["gate_up"] + kb["down"]
    moe_ms = (sum(tr["exposed"][k] for k in ("gate_up", "down", "moe")) if tr else
              (prof["gate_up"] + prof["down"] + prof["moe"])) / L
    B = CFG.bytes_per_token(cfg, mean_ctx)
    step_s = ms / 1000.0 / K
    line = {
        "metric": metric_name(c, a.context), "value": value, "unit": "tok/s",
        "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms / K, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "q8_0" if q8 else "bf16", "data": "synthetic",
        "config": workload_config(a),
        "run": {"context_start": ctx0, "mean_context": mean_ctx,
                "weights": ("Q8_0 linears (int8 + fp16 scale per 32, dequantised in registers), bf16 embedding"
                            if q8 else "bf16") + ", activations/accumulators f32",
                "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                "step_kernel": "fused: one persistent cooperative launch per step" if fused else
                f"chain: {4 if model.moe else 5} kernels per layer + head, PDL, CUDA graph",
                "l2": f"inputs larger than L2: every step streams ~{B['full'] / 1e9:.1f} GB of weights and KV "
                      "(L2 126 MB)",
                "prefill": "synthetic KV" if a.synthetic_kv else ("the prompt through the decode step" if q8 else
                                                                  "the prompt in multi-position steps of 32"),
                "prefill_s": round(prefill_s, 2)},
        "roofline": {"bound": "hbm", "kernel": dominant, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "peak_kind": peak_kind, "traffic": traffic,
                     "bytes_per_launch": kb[dominant], "ms_per_launch": per_launch_ms, "timing": regime},
        "step_roofline": {"literal_bytes": B["literal"], "full_bytes": B["full"],
                          "literal_frac": B["literal"] / step_s / 1e9 / hbm,
                          "full_frac": B["full"] / step_s / 1e9 / hbm,
                          "literal_frac_vs_8tbs": B["literal"] / step_s / 1e9 / 8000.0},
        "moe_block": None if fused else {"gbs": moe_bytes / (moe_ms / 1000.0) / 1e9,
                                         "frac": moe_bytes / (moe_ms / 1000.0) / 1e9 / hbm, "us_per_layer": moe_ms * 1000.0,
                                         "timing": "the MoE block's exposed time in the graph"},
        "kernels_ms_per_step": {k: round(v, 4) for k, v in prof.items()},
        "in_graph_ms_per_step": None if fused else {
            "exposed": {k: round(v, 4) for k, v in tr["exposed"].items() if k not in ("router", "fused_step")},
            "span": {k: round(v, 4) for k, v in tr["span"].items() if k not in ("router", "fused_step")},
            "handoff": {k: round(v, 4) for k, v in tr["wait"].items() if k not in ("router", "fused_step")},
            "step": round(tr["step_ms"], 4)},
        "e2e": e2e,
        "gpu_launches": K * (1 if fused else (4 if model.moe else 5) * L + 1),
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        rate, threads, n, sample = cpu_decode_rate(cfg, a.context, c["weight_seed"], a.cpu_seconds)
        line["cpu_baseline"] = {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample}
    model.close()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
