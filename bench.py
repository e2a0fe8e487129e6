"""Benchmark of the routed-MoE hot path on B200 (one JSON line on rank 0).

Headline workload: a Qwen3.8-Max-shaped MoE layer decoding one token per
GPU -- hidden 8192, 512 MXFP4 experts (SwiGLU 8192->2048->8192), softmax top-10, gated shared
expert, all experts resident in HBM. Metric: microseconds per token for the whole layer (lower
is better). Each timed step is one full layer forward (router, top-k, dispatch, expert GEMVs,
combine) on a fresh token already resident in HBM; L2 is flushed between steps.

Also reported on the same line: prefill tokens/s (config 2, 2048 tokens), the dominant kernel's
roofline (algorithmic bytes / CUDA-event duration vs the measured HBM copy peak), the end-to-end
number through the host-buffer C entry point (rmoe_moe_forward_host, copies included), and the
reference path restated in C (AVX-512 tier, oracle/) timed on this host's cores.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl rmoe|reference]

With N > 1 (torchrun, one process per GPU) every rank runs its own replica of the layer on its
own tokens (weak scaling): value = max-over-ranks time / all tokens processed. The line's "ep"
object is config 3 at the same N: a 4-layer stack, 4096 tokens per step, experts sharded 512 / N
per GPU with NCCL all-to-all dispatch and combine (strong scaling: total work fixed).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from rabbit_b200 import synth  # noqa: E402

DECODE_CFG = "c1_qwen_decode"
PREFILL_CFG = "c2_qwen_prefill"
L2_FLUSH_BYTES = 256 << 20


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d.get("bf16_tflops"), "measured"
    return 6650.0, 1590.0, "fallback"


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = f"/tmp/rmoe_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.fh,
                stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------ CPU path
def cpu_decode_setup(cfg, n_tokens=4, seed=0):
    """Tokens + the experts they route to, on the host, for the C restatement."""
    from oracle import oracle as orc

    x = synth.activations(cfg, tokens=n_tokens, token_offset=10_000)
    router = synth.router_weights(cfg, seed)
    logits = orc.matmul(x, router, n_tokens, cfg.hidden, cfg.n_experts)
    logits = (logits + synth.logit_bias(cfg, seed)[None, :]).astype(np.float32)
    need = set()
    for t in range(n_tokens):
        need.update(i for i, _ in orc.qwen_route(logits[t], cfg.topk))
    experts = {e: synth.expert(cfg, e, seed) for e in sorted(need)}
    shared = synth.expert(cfg, cfg.n_experts, seed)
    return x, router, experts, shared


def cpu_decode_time(cfg, budget_s=12.0, min_tokens=3, threads=None, setup=None):
    """Seconds per token of the reference path restated in C (AVX-512 tier, all row-parallel
    threads), decoding the setup's tokens round-robin until the time budget is spent."""
    from oracle import oracle as orc

    if threads:
        orc.set_threads(threads)
    x, router, experts, shared = setup or cpu_decode_setup(cfg)
    sg, lb = synth.shared_gate(cfg), synth.logit_bias(cfg)
    # warm once (page faults, thread pool)
    orc.moe_forward_qwen(x[:1], router, experts, cfg.n_experts, cfg.topk, cfg.inter, shared=shared,
                         shared_gate=sg, logit_bias=lb, shared_inter=cfg.shared_inter, tier="avx512")
    n, t0 = 0, time.perf_counter()
    while True:
        t = n % x.shape[0]
        orc.moe_forward_qwen(x[t:t + 1], router, experts, cfg.n_experts, cfg.topk, cfg.inter,
                             shared=shared, shared_gate=sg, logit_bias=lb,
                             shared_inter=cfg.shared_inter, tier="avx512")
        n += 1
        el = time.perf_counter() - t0
        if n >= min_tokens and el >= budget_s:
            break
    return el / n, n, orc.get_threads()


def cpu_decode_warm_cold(cfg, setup, reps=3):
    """Seconds per decode token with warm caches (the same token again) and cold ones (a buffer
    larger than L3 written before each call), as benches/kernels.rs:355-408 times its kernels."""
    from oracle import oracle as orc

    x, router, experts, shared = setup
    sg, lb = synth.shared_gate(cfg), synth.logit_bias(cfg)

    def one():
        orc.moe_forward_qwen(x[:1], router, experts, cfg.n_experts, cfg.topk, cfg.inter, shared=shared,
                             shared_gate=sg, logit_bias=lb, shared_inter=cfg.shared_inter, tier="avx512")

    one()
    t0 = time.perf_counter()
    for _ in range(reps):
        one()
    warm = (time.perf_counter() - t0) / reps
    evict = np.zeros(512 << 20, np.uint8)
    cold = 0.0
    for r in range(reps):
        evict[::64] = r + 1
        t0 = time.perf_counter()
        one()
        cold += time.perf_counter() - t0
    return warm, cold / reps


def physical_cores():
    try:
        import psutil

        return psutil.cpu_count(logical=False) or os.cpu_count()
    except ImportError:
        return os.cpu_count()


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def decode_config(world):
    """The headline workload's config object: the same dict on both arms of the bench."""
    cfg = synth.CONFIGS[DECODE_CFG]
    return {"workload": DECODE_CFG, "tokens_per_step_per_gpu": 1, "hidden": cfg.hidden,
            "n_experts": cfg.n_experts, "topk": cfg.topk, "inter": cfg.inter,
            "shared_inter": cfg.shared_inter, "weights": "mxfp4 (E2M1 + E8M0/32)",
            "parallelism": f"replicas x{world}" if world > 1 else "single gpu",
            "l2": "flushed between timed steps (256 MiB write, then a 256 MiB read that drains the write-backs)"}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    cfg = synth.CONFIGS[DECODE_CFG]
    threads = physical_cores()
    from oracle import oracle as orc

    orc.build()
    orc.set_threads(threads)
    setup = cpu_decode_setup(cfg)
    # warmup steps, then K timed steps; each step is one token through the whole layer
    sec, n, used = cpu_decode_time(cfg, budget_s=0.0, min_tokens=max(1, args.warmup), setup=setup)
    sec, n, used = cpu_decode_time(cfg, budget_s=0.0, min_tokens=max(1, args.steps), setup=setup)
    us = sec * 1e6
    line = {
        "impl": "reference", "metric": "moe_layer_decode_us_per_token", "value": us,
        "unit": "us/token", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sec * 1e3, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": decode_config(world),
        "cpu": cpu_model(),
        "cpu_baseline": {"value": us, "unit": "us/token", "cores": used, "kind": "port",
                         "sample": f"{n} decode tokens round-robin over 4 seeded tokens; C "
                                   "restatement of rabbit's AVX-512 MXFP4 tier + f32 router, "
                                   "OpenMP over output rows"},
        "e2e": {"value": us, "unit": "us/token", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------ GPU path
def ncu_traffic(key):
    """DRAM bytes per launch of a kernel from the committed ncu capture (profiles/), or None."""
    try:
        with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "profiles", "ncu_traffic.json")) as f:
            return json.load(f).get(key)
    except (OSError, ValueError):
        return None


def expert_touch_bytes(cfg, ids_np, with_shared=True):
    """Algorithmic bytes of one forward: distinct touched experts (+ shared) + router + x + out."""
    distinct = len(np.unique(ids_np[ids_np >= 0]))
    eb = cfg.expert_bytes()
    T = ids_np.shape[0]
    total = (distinct + (1 if with_shared else 0)) * eb
    total += cfg.n_experts * cfg.hidden * 2 + T * cfg.hidden * 2 + T * cfg.hidden * 4
    gu = (distinct + (1 if with_shared else 0)) * (2 * cfg.inter * (cfg.hidden // 2 + cfg.hidden // 32))
    return total, gu, distinct


EP_CFG = "c3_qwen_ep"
EP_PARITY_TOKENS = 16


def run_ep(args, ctx, dev, rank, world, flush):
    """Config 3: a stack of 4 MoE layers, 4096 tokens per step over the whole job, experts sharded
    512 / N per GPU (expert e on rank e // (512 / N)), tokens split 4096 / N per GPU, NCCL
    all-to-all dispatch and combine (rabbit_b200.ep). Layer l + 1 reads layer l's output (bf16).
    Returns the sub-object of the JSON line (value = tokens/s over the job, max-over-ranks time)."""
    import torch
    import torch.distributed as dist

    from rabbit_b200.ep import ExpertParallelMoe
    from rabbit_b200.synth import build_layer, x_device

    cfg = synth.CONFIGS[EP_CFG]
    t_local = cfg.tokens // world
    t_build = time.perf_counter()
    layers = [build_layer(ctx, cfg, max_tokens=cfg.tokens, layer=l, ep_rank=rank, ep_size=world)
              for l in range(cfg.n_layers)]
    build_s = time.perf_counter() - t_build
    eps = [ExpertParallelMoe(L) for L in layers]
    x0 = x_device(cfg, synth.activations(cfg, tokens=t_local, token_offset=rank * t_local))
    stream = torch.cuda.current_stream()

    def step(keep=None):
        x, ids_l = x0, []
        for ep in eps:
            out, ids, _ = ep.forward(x)
            ids_l.append(ids)
            if keep is not None:
                keep.append((x[:EP_PARITY_TOKENS].clone(), out[:EP_PARITY_TOKENS].clone(),
                             ids[:EP_PARITY_TOKENS].clone()))
            x = out.to(torch.bfloat16)
        return x, ids_l

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ev = []
    xbytes = []
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for _ in range(args.ep_steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        _, ids_l = step()
        b.record(stream)
        ev.append((a, b))
        xbytes.append(sum(ep.last_exchange_bytes for ep in eps))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = sum(a.elapsed_time(b) for a, b in ev) / args.ep_steps
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    # algorithmic bytes on this rank: its distinct touched experts per layer (+ shared, router, x, out)
    per = cfg.n_experts // world
    lo, hi = rank * per, (rank + 1) * per
    rbytes = 0.0
    for ids in ids_l:
        if world > 1:
            g = torch.empty((world,) + tuple(ids.shape), dtype=ids.dtype, device=dev)
            dist.all_gather_into_tensor(g, ids.contiguous())
            ids = g.reshape(-1, cfg.topk)
        a = ids.cpu().numpy()
        distinct = len(np.unique(a[(a >= lo) & (a < hi)]))
        rbytes += (distinct + 1) * cfg.expert_bytes() + cfg.n_experts * cfg.hidden * 2 + \
            t_local * cfg.hidden * (2 + 4)
    # parity at this N: rank 0's first tokens, layer by layer, against one GPU holding all the
    # layer's experts (moe_forward on the same layer input): routing ids bit-exact, output rel-L2
    keep = []
    step(keep)
    torch.cuda.synchronize()
    for L in layers:
        L.close()
    layers = []
    torch.cuda.empty_cache()
    parity = None
    if rank == 0:
        rels, ids_equal = [], True
        for l, (xin, got, got_ids) in enumerate(keep):
            full = build_layer(ctx, cfg, max_tokens=EP_PARITY_TOKENS, layer=l)
            want, want_ids, _ = full.moe_forward(xin, return_routing=True)
            torch.cuda.synchronize()
            full.close()
            ids_equal &= bool(torch.equal(got_ids, want_ids))
            rels.append(float((got - want).norm() / want.norm()))
        parity = {"reference": "one GPU holding all 512 experts of each layer (moe_forward on the same layer input)",
                  "tokens": EP_PARITY_TOKENS, "layers": cfg.n_layers, "ids_bit_exact": ids_equal,
                  "max_rel_l2": max(rels), "tolerance": 1e-2,
                  "ok": ids_equal and max(rels) < 1e-2}
    if world > 1:
        dist.barrier()
    rb_t = torch.tensor([rbytes, float(np.mean(xbytes))], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(rb_t, op=dist.ReduceOp.MAX)
    max_bytes, max_x = (float(v) for v in rb_t.tolist())
    hbm_peak, _, peak_kind = peaks()
    res = {"metric": "moe_ep_stack_tokens_per_s", "value": cfg.tokens / (ms / 1e3), "unit": "tokens/s",
           "ms_per_step": ms, "steps": args.ep_steps, "warmup": args.warmup,
           "config": {"workload": EP_CFG, "layers": cfg.n_layers, "tokens_per_step": cfg.tokens,
                      "tokens_per_gpu": t_local, "experts_per_gpu": per,
                      "parallelism": f"ep{world}" if world > 1 else "single gpu (all experts local)",
                      "l2": "inputs larger than L2 (GBs of expert weights per step) and flushed between steps"},
           "max_rank_algorithmic_bytes": max_bytes,
           "achieved_gbs_per_gpu": max_bytes / (ms / 1e3) / 1e9,
           "hbm_frac_per_gpu": max_bytes / (ms / 1e3) / 1e9 / hbm_peak, "peak_kind": peak_kind,
           "remote_bytes_per_gpu_per_step": max_x, "build_s": build_s, "parity": parity}
    return res


LATENT_CFG = "c5_k3_latent"
C4_CFG = "c4_glm_int4"


def run_latent(args, ctx, dev, rank, world, flush):
    """Row a14: Kimi K3's latent MoE at the real checkpoint's shapes, decoding one token per step
    (route 896 experts at 7168, down-project to 3584, 16 MXFP4 experts with SituAndMul, RMSNorm,
    up-project), inputs resident, L2 flushed between steps. Each rank runs its own replica."""
    import torch
    import torch.distributed as dist

    from rabbit_b200.synth import build_layer, x_device

    cfg = synth.CONFIGS[LATENT_CFG]
    L = build_layer(ctx, cfg, max_tokens=1)
    n_steps = args.warmup + args.latent_steps
    xs = synth.activations(cfg, tokens=n_steps, token_offset=rank * n_steps)
    xd = x_device(cfg, xs)
    out = torch.empty((1, cfg.full_hidden), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()
    for i in range(args.warmup):
        flush.zero_()
        L.latent_moe(xd[i:i + 1], out=out)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.latent_steps)]
    for j in range(args.latent_steps):
        flush.zero_()
        ev[j][0].record(stream)
        L.latent_moe(xd[args.warmup + j:args.warmup + j + 1], out=out)
        ev[j][1].record(stream)
    torch.cuda.synchronize()
    us = sum(a.elapsed_time(b) for a, b in ev) * 1e3 / args.latent_steps
    t = torch.tensor([us], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    us = float(t.item())
    # algorithmic bytes of one token: its k distinct experts, the router, both projections, x, out
    h, rh, i = cfg.hidden, cfg.full_hidden, cfg.inter
    expert = 3 * h * i // 2 + 3 * h * i // 32
    nbytes = cfg.topk * expert + cfg.n_experts * rh * 2 + 2 * rh * h * 2 + rh * 2 + rh * 4
    hbm_peak, _, peak_kind = peaks()
    res = {"metric": "k3_latent_moe_decode_us_per_token", "value": us, "unit": "us/token",
           "steps": args.latent_steps, "warmup": args.warmup,
           "config": {"workload": LATENT_CFG, "router_hidden": rh, "expert_hidden": h, "inter": i,
                      "n_experts": cfg.n_experts, "topk": cfg.topk, "activation": "situ (beta 4, linear 25)",
                      "latent_norm": True, "projections": "bf16", "experts": "mxfp4",
                      "l2": "flushed between steps"},
           "algorithmic_bytes": nbytes, "achieved_gbs": nbytes / (us * 1e-6) / 1e9,
           "hbm_frac": nbytes / (us * 1e-6) / 1e9 / hbm_peak, "peak_kind": peak_kind}
    L.close()
    return res


def run_c4(args, ctx, dev, rank, world, flush):
    """Config 4: the GLM-style grouped-int4 layer, 512 tokens per step (sigmoid grouped router,
    256 experts top-8, symmetric int4 with a bf16 scale per 32, always-on shared expert), inputs
    resident, L2 flushed between steps. Each rank runs its own replica."""
    import torch
    import torch.distributed as dist

    from rabbit_b200.synth import build_layer, x_device

    cfg = synth.CONFIGS[C4_CFG]
    L = build_layer(ctx, cfg, max_tokens=cfg.tokens, scale_dtype="bf16")
    xd = x_device(cfg, synth.activations(cfg, tokens=cfg.tokens, token_offset=rank * cfg.tokens))
    out = torch.empty((cfg.tokens, cfg.hidden), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        flush.zero_()
        L.moe_forward(xd, out=out)
    torch.cuda.synchronize()
    L.set_profiling(True)
    L.profile()
    ev = []
    for _ in range(args.c4_steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        L.moe_forward(xd, out=out)
        b.record(stream)
        ev.append((a, b))
    torch.cuda.synchronize()
    prof = L.profile()
    L.set_profiling(False)
    ms = sum(a.elapsed_time(b) for a, b in ev) / args.c4_steps
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    ids = L.route(xd)[0].cpu().numpy()
    L.check()
    L.close()
    distinct = len(np.unique(ids))
    eb = cfg.expert_bytes(scale_bytes=2)  # bf16 scales: 21,233,664 B per expert
    nbytes = (distinct + 1) * eb + cfg.n_experts * cfg.hidden * 2 + cfg.tokens * cfg.hidden * (2 + 4)
    hbm_peak, _, peak_kind = peaks()
    return {"metric": "glm_int4_layer_us_per_step", "value": ms * 1e3, "unit": "us/step",
            "tokens_per_s": cfg.tokens * world / (ms / 1e3), "ms_per_step": ms, "steps": args.c4_steps,
            "config": {"workload": C4_CFG, "tokens_per_step_per_gpu": cfg.tokens, "hidden": cfg.hidden,
                       "n_experts": cfg.n_experts, "topk": cfg.topk, "inter": cfg.inter,
                       "weights": "int4 (offset-binary nibbles) + bf16 scale per 32",
                       "router": "sigmoid + correction bias, 8 groups top-4, scale 2.5",
                       "l2": "flushed between steps"},
            "distinct_experts": distinct, "expert_bytes": eb, "algorithmic_bytes": nbytes,
            "achieved_gbs": nbytes / (ms / 1e3) / 1e9, "hbm_frac": nbytes / (ms / 1e3) / 1e9 / hbm_peak,
            "peak_kind": peak_kind,
            "stages_ms": {k: prof[k] / max(1, prof["calls"]) for k in prof if k != "calls"}}


def cpu_c4_time(threads, n_tokens=8):
    """Seconds per step of config 4 on the host: the reference's GLM path restated in C (exact f32
    router chains, sigmoid grouped top-k, scalar matmul_i4_grouped as in src/kernels.rs:276-296,
    OpenMP over output rows like its rayon), over a bounded batch of n_tokens tokens."""
    from oracle import oracle as orc

    cfg = synth.CONFIGS[C4_CFG]
    orc.set_threads(threads)
    x = synth.activations(cfg, tokens=n_tokens, token_offset=20_000)
    router, bias = synth.router_weights(cfg), synth.correction_bias(cfg)
    ids, _ = orc.glm_route(x, router, bias, n_tokens, cfg.hidden, cfg.n_experts, cfg.topk, cfg.n_group,
                           cfg.topk_group, cfg.norm_topk, cfg.routed_scale)
    experts = {int(e): synth.expert(cfg, int(e)) for e in np.unique(ids)}
    shared = synth.expert(cfg, cfg.n_experts)
    t0 = time.perf_counter()
    orc.moe_glm(x, router, bias, experts, cfg.n_experts, cfg.topk, cfg.inter, cfg.n_group, cfg.topk_group,
                cfg.norm_topk, cfg.routed_scale, shared=shared, shared_inter=cfg.shared_inter,
                fmt=cfg.fmt_id, gs=cfg.group_size)
    return time.perf_counter() - t0


def run_gpu(args):
    import torch
    import torch.distributed as dist

    import rabbit_b200 as rb

    from rabbit_b200.synth import build_layer, x_device

    rank, world, local = dist_env()
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ctx = rb.Context(local)
    cfg = synth.CONFIGS[PREFILL_CFG]  # same weights as config 1; sized for the prefill run
    dcfg = synth.CONFIGS[DECODE_CFG]
    if args.small_experts:
        # profiling-size variant: identical shapes and kernels, fewer resident experts
        import dataclasses

        cfg = dataclasses.replace(cfg, n_experts=args.small_experts)
        dcfg = dataclasses.replace(dcfg, n_experts=args.small_experts)
    layer = build_layer(ctx, cfg, max_tokens=cfg.tokens)
    flush_buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    drain_buf = torch.zeros(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    class _Flush:
        # L2 flush between steps: write a buffer larger than L2, then read another one so the
        # dirty lines are written back before the next step starts (otherwise their write-back
        # shares HBM bandwidth with the step being timed)
        def zero_(self):
            flush_buf.zero_()
            drain_buf.sum()

    flush = _Flush()
    n_steps = args.warmup + args.steps
    xs = synth.activations(dcfg, tokens=n_steps, token_offset=rank * n_steps)
    xd = x_device(dcfg, xs)
    out = torch.empty((1, cfg.hidden), dtype=torch.float32, device=dev)
    ids_all = torch.empty((n_steps, cfg.topk), dtype=torch.int32, device=dev)
    w_all = torch.empty((n_steps, cfg.topk), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()

    def step(i):
        layer.moe_forward(xd[i:i + 1], out=out)

    # the clock sampler starts (and settles) before the warm-up steps, so the GPU is busy right
    # up to the first timed step
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    for i in range(args.warmup):
        flush.zero_()
        step(i)
    torch.cuda.synchronize()
    launches0 = layer.stats()["kernel_launches"]
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for j in range(args.steps):
        flush.zero_()
        ev[j][0].record(stream)
        step(args.warmup + j)
        ev[j][1].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    step_ms = [a.elapsed_time(b) for a, b in ev]
    total_ms = sum(step_ms)
    launches = (layer.stats()["kernel_launches"] - launches0) // args.steps
    # stage breakdown (and the roofline kernel's duration) from a separate pass over the same
    # tokens with per-stage events on the launching stream; the timed steps above carry none
    layer.set_profiling(True)
    layer.profile()
    for j in range(args.steps):
        flush.zero_()
        step(args.warmup + j)
    torch.cuda.synchronize()
    prof = layer.profile()
    layer.set_profiling(False)
    t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    us_per_token = total_ms * 1e3 / (args.steps * world)

    # routing of the timed tokens -> algorithmic bytes (every step touches k distinct + shared)
    layer.route(xd[args.warmup:])  # warm path check; ids below from one extra forward each
    ids_np = layer.route(xd[args.warmup:])[0].cpu().numpy()
    per_step = [expert_touch_bytes(dcfg, ids_np[j:j + 1]) for j in range(args.steps)]
    layer_bytes = float(np.mean([p[0] for p in per_step]))
    gu_bytes = float(np.mean([p[1] for p in per_step]))
    expert_bytes = float(np.mean([(p[2] + 1) * dcfg.expert_bytes() for p in per_step]))
    hbm_peak, _, peak_kind = peaks()
    gu_ms = prof["gate_up"] / max(1, prof["calls"])
    dn_ms = prof["down"] / max(1, prof["calls"])
    # one token: gate/up and down of its experts run as one fused kernel (its time is the
    # gate_up stage) unless RMOE_DISABLE_FUSED=1 selects the two-kernel path
    fused = os.environ.get("RMOE_DISABLE_FUSED", "0") != "1"
    if fused:
        rf_name = "moe_decode_fused_kernel (tcgen05 kind::mxf4: gate/up + SwiGLU + down of the token's 11 experts)"
        rf_bytes, rf_ms, rf_key = expert_bytes, gu_ms, "moe_decode_fused_kernel_bytes"
    else:
        rf_name = "moe_tc_kernel<gate_up> (tcgen05 kind::mxf4, SwiGLU epilogue)"
        rf_bytes, rf_ms, rf_key = gu_bytes, gu_ms, "moe_tc_kernel_gate_up_decode_bytes"
    stages_us = {k: prof[k] * 1e3 / max(1, prof["calls"]) for k in prof if k != "calls"}

    # end to end through the host-buffer entry point (pinned host in/out, copies inside)
    x_host = torch.from_numpy(synth.f32_to_bf16_bits(xs).view(np.int16)).pin_memory().view(torch.bfloat16)
    out_host = torch.empty((1, cfg.hidden), dtype=torch.float32).pin_memory()
    for i in range(min(3, n_steps)):
        layer.moe_forward_host(x_host[i:i + 1], out=out_host)
    e2e = []
    for j in range(args.steps):
        flush.zero_()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        layer.moe_forward_host(x_host[args.warmup + j:args.warmup + j + 1], out=out_host)
        e2e.append(time.perf_counter() - t0)
    e2e_t = torch.tensor([sum(e2e)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_us = float(e2e_t.item()) * 1e6 / (args.steps * world)

    # prefill (config 2): 2048 tokens per step
    pre = None
    if not args.no_prefill:
        xp = x_device(cfg, synth.activations(cfg, tokens=cfg.tokens, token_offset=100_000 + rank * cfg.tokens))
        outp = torch.empty((cfg.tokens, cfg.hidden), dtype=torch.float32, device=dev)
        for _ in range(2):
            flush.zero_()
            layer.moe_forward(xp, out=outp)
        torch.cuda.synchronize()
        layer.set_profiling(True)
        layer.profile()
        pev = []
        for _ in range(args.prefill_steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            layer.moe_forward(xp, out=outp)
            b.record(stream)
            pev.append((a, b))
        torch.cuda.synchronize()
        pprof = layer.profile()
        layer.set_profiling(False)
        pms = sum(a.elapsed_time(b) for a, b in pev) / args.prefill_steps
        pt = torch.tensor([pms], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(pt, op=dist.ReduceOp.MAX)
        pms = float(pt.item())
        pids = layer.route(xp)[0].cpu().numpy()
        pbytes, pgu, pdistinct = expert_touch_bytes(cfg, pids)
        flops = 2.0 * (cfg.tokens * cfg.topk + cfg.tokens) * 3 * cfg.hidden * cfg.inter + \
            2.0 * cfg.tokens * cfg.n_experts * cfg.hidden
        pre = {"metric": "moe_layer_prefill_tokens_per_s",
               "value": cfg.tokens * world / (pms / 1e3), "unit": "tokens/s",
               "ms_per_step": pms, "tokens_per_step_per_gpu": cfg.tokens,
               "distinct_experts": pdistinct, "algorithmic_bytes": pbytes,
               "achieved_gbs": pbytes / (pms / 1e3) / 1e9, "hbm_frac": pbytes / (pms / 1e3) / 1e9 / hbm_peak,
               "tflops": flops / (pms / 1e3) / 1e12,
               "stages_ms": {k: pprof[k] / max(1, pprof["calls"]) for k in pprof if k != "calls"}}

    line = {
        "metric": "moe_layer_decode_us_per_token", "value": us_per_token, "unit": "us/token",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "step_us_spread": {"min": round(min(step_ms) * 1e3, 2), "median": round(float(np.median(step_ms)) * 1e3, 2),
                           "max": round(max(step_ms) * 1e3, 2), "argmax": int(np.argmax(step_ms))},
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
        "dtype": "mxfp4 weights x 4-term e2m1 activations (tcgen05 kind::mxf4), f32 accumulate", "data": "synthetic",
        "config": decode_config(world),
        "roofline": {"bound": "hbm", "kernel": rf_name,
                     "achieved": rf_bytes / (rf_ms / 1e3) / 1e9 if rf_ms > 0 else None,
                     "peak": hbm_peak, "unit": "GB/s", "peak_kind": peak_kind,
                     "frac": (rf_bytes / (rf_ms / 1e3) / 1e9 / hbm_peak) if rf_ms > 0 else None,
                     "traffic": ncu_traffic(rf_key),
                     "traffic_source": "profiles/moe_tc_kernel_decode_small.md (ncu, per launch)",
                     "kernel_us": rf_ms * 1e3, "kernel_bytes": rf_bytes,
                     "kernel_timing": "CUDA events around the kernel on its stream, profiling pass over the timed tokens",
                     "layer_algorithmic_bytes": layer_bytes,
                     "layer_achieved_gbs": layer_bytes / (ms_per_step / 1e3) / 1e9,
                     "layer_frac": layer_bytes / (ms_per_step / 1e3) / 1e9 / hbm_peak},
        "stages_us": stages_us,
        "e2e": {"value": e2e_us, "unit": "us/token", "h2d_bytes_per_step": cfg.hidden * 2,
                "d2h_bytes_per_step": cfg.hidden * 4,
                "api": "rmoe_moe_forward_host (pinned host x/out, copies + sync inside)"},
        "gpu_launches": int(launches),
        "router_fallbacks": layer.stats()["router_fallbacks"],
        "router_order_resolved": layer.stats()["router_order_resolved"],
        "device_error_flags": layer.stats()["device_error_flags"],
        "clocks": clk,
        "prefill": pre,
    }
    if not args.no_ep:
        layer.close()
        layer = None
        torch.cuda.empty_cache()
        line["ep"] = run_ep(args, ctx, dev, rank, world, flush)
    if not args.no_c4:
        if layer is not None:
            layer.close()
            layer = None
        torch.cuda.empty_cache()
        line["c4"] = run_c4(args, ctx, dev, rank, world, flush)
    if not args.no_latent:
        if layer is not None:
            layer.close()
            layer = None
        torch.cuda.empty_cache()
        line["latent"] = run_latent(args, ctx, dev, rank, world, flush)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        setup = cpu_decode_setup(dcfg)
        sec, n, used = cpu_decode_time(dcfg, budget_s=args.cpu_budget, threads=physical_cores(), setup=setup)
        warm, cold = cpu_decode_warm_cold(dcfg, setup)
        line["cpu_baseline"] = {
            "value": sec * 1e6, "unit": "us/token", "cores": used, "kind": "port",
            "cpu": cpu_model(),
            "warm_us": warm * 1e6, "cold_us": cold * 1e6,
            "sample": f"{n} decode tokens round-robin over 4 seeded tokens (~{args.cpu_budget:.0f} s); "
                      "C restatement of rabbit's AVX-512 MXFP4 tier + f32 router, OpenMP over rows. "
                      "warm: one token repeated; cold: a 512 MiB write before each call evicts the caches"}
        if not args.no_c4:
            c4_s = cpu_c4_time(physical_cores())
            line["cpu_baseline"]["c4"] = {
                "value": c4_s * 1e6 / 8, "unit": "us/token", "tokens_per_s": 8 / c4_s, "cores": used,
                "kind": "port", "sample": "8 tokens of config 4 through the restated GLM layer (scalar int4)"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if layer is not None:
        layer.close()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


def run_profile_case(args):
    """A profiling workload, not a bench line: build one layer and run --forwards forwards of one
    case, the last one inside a cudaProfilerStart/Stop range when --profile-last is given (so that
    `ncu --profile-from-start off` captures exactly that call). --small-experts shrinks the
    resident experts (same shapes and kernels) so that a multi-metric capture stays small.
    Cases: prefill (c2, 2048 tokens), decode (c1, one token), latent (K3 latent MoE, one token),
    int4 (c4, 512 tokens)."""
    import dataclasses

    import torch

    import rabbit_b200 as rb
    from rabbit_b200.synth import build_layer, x_device

    name = {"prefill": PREFILL_CFG, "decode": DECODE_CFG, "latent": LATENT_CFG, "int4": C4_CFG}[args.profile_case]
    cfg = synth.CONFIGS[name]
    if args.small_experts:
        cfg = dataclasses.replace(cfg, n_experts=args.small_experts)
    ctx = rb.Context(0)
    layer = build_layer(ctx, cfg, max_tokens=cfg.tokens, scale_dtype="bf16" if cfg.fmt != "mxfp4" else "f32")
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    for i in range(args.forwards):
        x = x_device(cfg, synth.activations(cfg, tokens=cfg.tokens, token_offset=100_000 + i * cfg.tokens))
        flush.zero_()
        torch.cuda.synchronize()
        last = i == args.forwards - 1
        if last and args.profile_last:
            torch.cuda.cudart().cudaProfilerStart()
        if args.profile_case == "latent":
            layer.latent_moe(x)
        else:
            layer.moe_forward(x)
        torch.cuda.synchronize()
        if last and args.profile_last:
            torch.cuda.cudart().cudaProfilerStop()
    layer.check()
    errs = layer.stats()["device_error_flags"]
    layer.close()
    ctx.close()
    print(f"{args.profile_case}: {args.forwards} forwards of {cfg.name} ({cfg.n_experts} experts), "
          f"device error flags {errs}")
    return 0 if errs == 0 else 1


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="rmoe", choices=["rmoe", "reference"])
    ap.add_argument("--prefill-steps", type=int, default=3)
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ep", action="store_true", help="skip the expert-parallel stack (config 3)")
    ap.add_argument("--ep-steps", type=int, default=5)
    ap.add_argument("--no-latent", action="store_true", help="skip the K3 latent MoE decode (row a14)")
    ap.add_argument("--latent-steps", type=int, default=10)
    ap.add_argument("--no-c4", action="store_true", help="skip the GLM int4 layer (config 4)")
    ap.add_argument("--c4-steps", type=int, default=5)
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--small-experts", type=int, default=0,
                    help="profiling only: resident experts (same shapes); not a bench config")
    ap.add_argument("--profile-case", choices=["prefill", "decode", "latent", "int4"], default=None,
                    help="profiling workload only (no bench line): see run_profile_case")
    ap.add_argument("--forwards", type=int, default=3, help="--profile-case: forwards to run")
    ap.add_argument("--profile-last", action="store_true",
                    help="--profile-case: last forward inside cudaProfilerStart/Stop")
    args = ap.parse_args()
    if args.profile_case:
        raise SystemExit(run_profile_case(args))
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
