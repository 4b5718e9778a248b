#!/usr/bin/env python
"""Mixtral-block forward+backward throughput on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl reference]

One step is one pass of the block lens over one batch: zero the parameter
adjoint, forward (get), backward (put) and, with N > 1 GPUs, the exchange of
the expert-parallel block (or the data-parallel reduction of the parameter
adjoint over NCCL).  The stack workload runs the staged plan of four blocks
(one step = the global batch through every block); the MLP workload runs the
kernel.rs program (forward, MSE head, backward) from a CUDA graph.  Inputs are
seeded synthetic tensors of the workload's shapes (no dataset exists for this
path): matrices ~ N(0, 0.02^2), RMSNorm weights 1, x and dy ~ N(0, 1).

Prints one JSON line (rank 0).  `value` is whole-job tokens/s with inputs
resident in HBM; `e2e` is the same metric through the public C-ABI call with
the step's inputs copied from pinned host memory and its whole result (y, dx
and the fp32 parameter adjoint) read back every step; `roofline` is the expert gate/up grouped GEMM against the
measured bf16 peak; `cpu_baseline` is the CPU oracle (a port of the crate's
single-threaded CPU lens) on a bounded sample of the same workload.

`--impl reference` times that CPU lens instead, on all host cores (one
independent sample per worker process), and prints the same metric.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "dependent-optics_b200"))
sys.path.insert(0, str(ROOT / "tests"))

METRIC = "Mixtral-block fwd+bwd tokens/s at 1/2/4/8 B200; % of bf16 tensor peak"

WORKLOADS = {
    # Mixtral-8x7B-shaped block, bf16 weights / fp32 accumulate, balanced routing
    "mixtral8x7b_block": dict(cfg=dict(vocab=32000, dim=4096, layers=1, heads=32, kv_heads=8,
                                       head_dim=128, intermediate=14336, experts=8, top_k=2,
                                       rms_eps=1e-5, rope_theta=1e6, sliding_window=4096),
                              batch=8, seq=4096, precision="bf16", skew=False, cpu_seq=16),
    # same, with a Zipf(s=1.2) per-expert logit bias scaled to 2.0
    "mixtral8x7b_block_skewed": dict(cfg=dict(vocab=32000, dim=4096, layers=1, heads=32,
                                              kv_heads=8, head_dim=128, intermediate=14336,
                                              experts=8, top_k=2, rms_eps=1e-5, rope_theta=1e6,
                                              sliding_window=4096),
                                     batch=8, seq=4096, precision="bf16", skew=True,
                                     cpu_seq=16),
    # dense block (one expert, top-1, full causal attention)
    "dense_block": dict(cfg=dict(vocab=32000, dim=2048, layers=1, heads=16, kv_heads=16,
                                 head_dim=128, intermediate=5632, experts=1, top_k=1,
                                 rms_eps=1e-5, rope_theta=1e4, sliding_window=2048),
                        batch=8, seq=2048, precision="bf16", skew=False, cpu_seq=128),
    # Mixtral-8x7B widths at batch 1, seq 1024: the small case for profiler captures
    "mixtral8x7b_block_profile": dict(cfg=dict(vocab=32000, dim=4096, layers=1, heads=32,
                                               kv_heads=8, head_dim=128, intermediate=14336,
                                               experts=8, top_k=2, rms_eps=1e-5, rope_theta=1e6,
                                               sliding_window=4096),
                                      batch=1, seq=1024, precision="bf16", skew=False,
                                      cpu_seq=16),
    # the Mixtral-8x7B router stage's shape (d_model 4096, 8 experts, top-2,
    # 32768 tokens) with a small expert hidden size: the profiling case of the
    # router kernel (a few GB on the device, inputs larger than L2)
    "router_profile": dict(cfg=dict(vocab=32000, dim=4096, layers=1, heads=32, kv_heads=8,
                                    head_dim=128, intermediate=128, experts=8, top_k=2,
                                    rms_eps=1e-5, rope_theta=1e6, sliding_window=4096),
                           batch=8, seq=4096, precision="bf16", skew=False, cpu_seq=16),
    # the tensor-core GEMM alone on one expert's gate projection at batch 2,
    # seq 4096 routed rows (16384 x 14336, contraction 4096): the kernel-level
    # profiling case, timed beside cuBLAS on the same shape
    # the Mixtral-8x7B block's attention alone (32 / 8 heads, head_dim 128,
    # causal, window 4096) through dop_gqa_forward / dop_gqa_backward
    "mixtral8x7b_attention": dict(attention=(8, 4096, 32, 8, 128, 4096), precision="bf16",
                                  skew=False),
    "mixtral8x7b_attention_profile": dict(attention=(2, 4096, 32, 8, 128, 4096),
                                          precision="bf16", skew=False),
    "gemm_bf16_expert": dict(gemm=(16384, 14336, 4096, 0), precision="bf16", skew=False),
    # the expert-input cotangent's shape: 16384 rows, N 4096, contraction
    # 28672, B read transposed (the crate's [D, I] gate/up weights)
    "gemm_bf16_dx": dict(gemm=(16384, 4096, 28672, 1), precision="bf16", skew=False),
    # staged 4-block stack of Mixtral-8x7B-shaped blocks: global batch 32 at seq
    # 4096 in 8 micro-batches, pipeline-staged over the GPUs (dop.cluster)
    "mixtral8x7b_stack4": dict(cfg=dict(vocab=32000, dim=4096, layers=4, heads=32, kv_heads=8,
                                        head_dim=128, intermediate=14336, experts=8, top_k=2,
                                        rms_eps=1e-5, rope_theta=1e6, sliding_window=4096),
                               batch=32, seq=4096, micro_batches=8, precision="bf16",
                               skew=False, stack=True, cpu_seq=16),
    # small Mixtral block, fp32
    "small_mixtral_block_f32": dict(cfg=dict(vocab=32000, dim=512, layers=1, heads=8, kv_heads=2,
                                             head_dim=64, intermediate=1408, experts=8, top_k=2,
                                             rms_eps=1e-5, rope_theta=1e6, sliding_window=128),
                                    batch=4, seq=512, precision="f32", skew=False, cpu_seq=512),
    # the crate's CPU-run case: kernel.rs MLP program, batch 64, 128 -> 256 -> 128,
    # ReLU hidden, MSE against targets
    "mlp_f32": dict(program="mlp", batch=64, dims=[128, 256, 128], precision="f32", skew=False),
}
DEFAULT_WORKLOAD = "mixtral8x7b_block"
# The CPU sample of a block workload is one sequence of `cpu_seq` tokens at
# the workload's full widths (batch 1), sized so one oracle fwd+bwd takes
# seconds on a many-core host; it includes the attention over its positions.
# DRAM bytes (read 7.43e9 + write 5.80e9) of one expert gate/up launch of
# the Mixtral-8x7B block at batch 8, seq 4096: one launch (-s 4 -c 1) of
# dram__bytes_read/write.sum, which ncu collects in one pass (checked on the
# batch 1, seq 1024 case first); a bench run cannot read DRAM counters.  The
# traffic does not scale with the routed rows (the weights are re-read once
# per band of row tiles), so it is quoted for that workload only.
GATE_UP_TRAFFIC = 7.43e9 + 5.80e9


def flops_per_step(cfg, batch, seq):
    """Algorithmic FLOPs of one block fwd+bwd: 3 x forward, selected experts
    only, visible attention pairs only, no recomputation counted."""
    D, H, KV, hd = cfg["dim"], cfg["heads"], cfg["kv_heads"], cfg["head_dim"]
    E, k, I, W = cfg["experts"], cfg["top_k"], cfg["intermediate"], cfg["sliding_window"]
    T = batch * seq
    vis = sum(min(s + 1, W) for s in range(seq)) * batch
    fwd = (2 * T * (D * H * hd + 2 * D * KV * hd + H * hd * D) + 4 * hd * H * vis
           + 2 * T * k * 3 * D * I + (2 * T * D * E if E > 1 else 0))
    return 3 * fwd


def zipf_bias(E, seed=0, s=1.2, scale=2.0):
    """b_e = scale * r_e^-s with expert ranks r from a seeded permutation."""
    import torch
    g = torch.Generator().manual_seed(seed)
    ranks = torch.randperm(E, generator=g) + 1
    return (scale * ranks.double() ** -s).float()


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d["bf16_tflops_sustained"], "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.proc = index, None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc:
            self.proc.terminate()
            try:
                self.out = self.proc.communicate(timeout=5)[0]
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out = self.proc.communicate()[0]

    def summary(self):
        rows = [r.split(",") for r in self.out.strip().splitlines() if r.count(",") >= 7]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" == r[4 + i].strip()})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


def make_params(cfg_d, precision, seed, device):
    import torch
    from dop.mixtral import MixtralConfig, layer_layout
    cfg = MixtralConfig(**cfg_d)
    ll = layer_layout(cfg)
    g = torch.Generator(device=device).manual_seed(seed)
    dt = torch.bfloat16 if precision == "bf16" else torch.float32
    P = torch.empty(ll.total, dtype=dt, device=device)
    chunk = 1 << 28
    for a in range(0, ll.total, chunk):  # N(0, 0.02^2) in chunks (bounded fp32 temporary)
        b = min(ll.total, a + chunk)
        P[a:b] = (torch.randn(b - a, generator=g, device=device) * 0.02).to(dt)
    P[ll.attn_norm: ll.attn_norm + cfg.dim] = 1.0
    P[ll.ffn_norm: ll.ffn_norm + cfg.dim] = 1.0
    return cfg, ll, P


class _Cfg:
    """A MixtralConfig-shaped record for the oracle (no library load)."""
    def __init__(self, d):
        self.__dict__.update(d)


def cpu_oracle_sample(cfg_d, seq, seed, repeats=1, threads=0):
    """(seconds of each fwd+bwd, threads used) of the CPU oracle on
    (batch 1, seq) at full widths, on `threads` host threads (0 = all)."""
    import numpy as np
    import torch
    import oracle_ffi as orc
    cfg = _Cfg(cfg_d)
    ll = orc.layer_offsets(cfg)
    used = orc.set_threads(threads)
    g = torch.Generator().manual_seed(seed)
    # 16 Mi seeded N(0, 0.02^2) values tiled over the layer: drawing 1.45e9
    # normals on the host would take longer than the sample itself
    base = (torch.randn(1 << 24, generator=g) * 0.02).numpy()
    lp = np.resize(base, ll["total"])
    lp[ll["attn_norm"]: ll["attn_norm"] + cfg.dim] = 1.0
    lp[ll["ffn_norm"]: ll["ffn_norm"] + cfg.dim] = 1.0
    x = torch.randn(seq * cfg.dim, generator=g).numpy()
    dy = torch.randn(seq * cfg.dim, generator=g).numpy()
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        r = orc.block_forward(cfg, lp, x, 1, seq)
        orc.block_backward(cfg, lp, r, dy)
        times.append(time.perf_counter() - t0)
        del r
    return times, used


def use_expert_parallel(a, wl, world) -> bool:
    """Expert parallel when the experts split over the ranks (the contract's
    partitioning of the Mixtral block), else data parallel.  Skewed routing
    runs expert-parallel too: the block's per-step plan splits a hot
    expert's rows over several ranks."""
    from dop import parallel
    return (world > 1 and a.parallel != "dp"
            and parallel.ep_mode(world, wl["cfg"]["experts"], wl["precision"] == "bf16"))


def arm_config(a, wl, world) -> dict:
    """The `config` both arms print for a workload at `world` GPUs."""
    if wl.get("program"):
        return {"workload": a.workload, "batch_per_gpu": wl["batch"], "dims": wl["dims"],
                "loss": "mse", "parallelism": "single" if world == 1 else
                f"{world} independent replicas",
                "graph": "one CUDA graph per step (forward, MSE head, backward)",
                "l2": "inputs smaller than L2 (the workload is 2 x 32 KiB)"}
    if wl.get("stack"):
        pp = math.gcd(wl["cfg"]["layers"], world)
        return {"workload": a.workload, "global_batch": wl["batch"], "seq": wl["seq"],
                "micro_batches": wl["micro_batches"], **wl["cfg"],
                "parallelism": f"pp{pp}" + (f"xdp{world // pp}" if world // pp > 1 else ""),
                "schedule": "one-forward-one-backward per stage (dop.cluster plan)",
                "l2": "inputs larger than L2 (each micro-batch is 4 B x 16384 x 4096)"}
    E = wl["cfg"]["experts"]
    return {"workload": a.workload, "batch_per_gpu": wl["batch"], "seq": wl["seq"],
            "global_batch": wl["batch"] * world, **wl["cfg"],
            "parallelism": ("single" if world == 1 else
                            f"ep{world} ({E // world} experts per rank, exchange over NVLink "
                            "peer reads, shared adjoint all-reduced)"
                            if use_expert_parallel(a, wl, world) else
                            f"dp{world}, expert adjoints reduced during the attention backward"),
            "l2": "inputs larger than L2 (x, dy are 4 B x T x D each)"}


def run_reference(a):
    """The CPU lens (the oracle, a port of the crate's CPU lens) on every
    host thread: each step is one fwd+bwd of a (batch 1, cpu_seq) sample at
    the workload's full widths; tokens/s = sample tokens / its time.  Only
    rank 0 works (the other ranks of a torchrun launch exit at once)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    wl = WORKLOADS[a.workload]
    world = int(os.environ.get("WORLD_SIZE", str(a.gpus)))
    cores = os.cpu_count() or 1
    if wl.get("program"):
        run_reference_program(a, wl, cores, world)
        return
    if wl.get("gemm") or wl.get("attention"):
        print(json.dumps({"impl": "reference", "unavailable": "a kernel-level profiling workload "
                          "with no counterpart in the crate's CPU lens"}), flush=True)
        return
    steps = max(1, a.steps)
    seq = wl["cpu_seq"]
    times, used = cpu_oracle_sample(wl["cfg"], seq, seed=0, repeats=a.warmup + steps)
    layers = wl["cfg"]["layers"]
    # a stack of identical blocks costs `layers` block passes per token: one
    # block is timed and the time scaled by the layer count
    per_step = [layers * t for t in times[a.warmup:]]
    t = sum(per_step) / steps
    v = seq / t
    sample = (f"batch 1, seq {seq} at the full widths of {a.workload}, one fwd+bwd per step "
              f"on {used} host threads"
              + (f", one block timed x {layers} blocks" if layers > 1 else ""))
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": a.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": arm_config(a, wl, world),
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": used, "kind": "port",
                         "sample": sample},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def mlp_inputs(wl, seed=0):
    """x, targets ~ N(0,1); W ~ N(0, 1/fan_in); b = 0 (host fp32 tensors)."""
    import torch
    from dop import kernel as K
    prog = K.Program.mlp(wl["batch"], wl["dims"])
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(prog.input_len, generator=g)
    t = torch.randn(prog.output_len, generator=g)
    params = torch.zeros(prog.param_len)
    for st in prog.stages:
        n = st.din * st.dout
        params[st.param_at: st.param_at + n] = torch.randn(n, generator=g) / st.din ** 0.5
    return prog, x, t, params


def mlp_flops(wl):
    """fwd+bwd = 3 x the forward's 2 * batch * din * dout per layer."""
    d = wl["dims"]
    return 3 * sum(2 * wl["batch"] * a * b for a, b in zip(d[:-1], d[1:]))


def cpu_program_sample(wl, seconds=1.0):
    """(steps, seconds) of the oracle's program forward+backward (the crate's
    single-threaded CPU path) with the MSE cotangent of the targets."""
    import numpy as np
    import oracle_ffi as orc
    prog, x, t, params = mlp_inputs(wl)
    x, t, params = x.numpy(), t.numpy(), params.numpy()
    y = orc.program_forward_backward(prog, x, params)[0]
    dy = (2.0 * (y - t) / y.size).astype(np.float32)
    n, t0 = 0, time.perf_counter()
    while True:
        orc.program_forward_backward(prog, x, params, dy=dy)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            return n, el


def _program_worker(args):
    wl, seconds = args
    return cpu_program_sample(wl, seconds)


def run_program(a):
    """A kernel.rs program workload: one step = forward, MSE head, backward of
    the compiled program, replayed from a CUDA graph; every rank runs its own
    replica (the program has no data-parallel exchange)."""
    import torch
    import torch.distributed as dist
    from dop import kernel as K
    from dop import parallel

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    world, rank = parallel.init_from_env("nccl", timeout_s=600, device=dev)
    wl = WORKLOADS[a.workload]
    prog, hx, ht, hp = mlp_inputs(wl)
    cp = K.CompiledProgram(prog)
    X, Tt, P = hx.to(dev), ht.to(dev), hp.to(dev)
    stream = torch.cuda.Stream(dev)
    rows = wl["batch"]

    def step(x, t, s):
        y = cp.forward(x, P, stream=s)
        loss, dy = K.mse_loss_grad(y, t, stream=s)
        dx, dp = cp.backward(P, dy, stream=s)
        return loss, dx, dp

    with torch.cuda.stream(stream):
        for _ in range(max(3, a.warmup)):
            step(X, Tt, stream)
    stream.synchronize()
    l_per = cp.launches()
    step(X, Tt, stream)
    stream.synchronize()
    l_per = cp.launches() - l_per + 1  # + the MSE head
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step(X, Tt, torch.cuda.current_stream(dev))
    for _ in range(a.warmup):
        graph.replay()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    cur = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(cur)
    for _ in range(a.steps):
        graph.replay()
    ev1.record(cur)
    torch.cuda.synchronize(dev)
    ms = parallel.max_over_ranks(ev0.elapsed_time(ev1) / a.steps, device=dev)
    value = world * rows / (ms / 1e3)
    # a step takes microseconds: a longer run of replays gives the clock
    # sampler something to see and a steady-state time beside the K steps
    reps = 20000
    with ClockSampler(local) as clk:
        ev0.record(cur)
        for _ in range(reps):
            graph.replay()
        ev1.record(cur)
        torch.cuda.synchronize(dev)
    steady_ms = parallel.max_over_ranks(ev0.elapsed_time(ev1) / reps, device=dev)

    # end to end through the public calls: x and targets from pinned host
    # memory, the loss read back, every step
    e2e = None
    if not a.no_e2e:
        px, pt = hx.pin_memory(), ht.pin_memory()
        hl = torch.empty(500, dtype=torch.float32).pin_memory()
        Xd, Td = torch.empty_like(X), torch.empty_like(Tt)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_e2e = 500
        with torch.cuda.stream(stream):
            e0.record(stream)
            for i in range(n_e2e):
                Xd.copy_(px, non_blocking=True)
                Td.copy_(pt, non_blocking=True)
                loss, _, _ = step(Xd, Td, stream)
                hl[i:i + 1].copy_(loss.view(1), non_blocking=True)
            e1.record(stream)
        torch.cuda.synchronize(dev)
        ems = parallel.max_over_ranks(e0.elapsed_time(e1) / n_e2e, device=dev)
        e2e = {"value": world * rows / (ems / 1e3), "unit": "tokens/s", "steps": n_e2e,
               "h2d_bytes_per_step": (hx.numel() + ht.numel()) * 4, "d2h_bytes_per_step": 4,
               "note": "eager public calls (CompiledProgram.forward, mse_loss_grad, backward)"}
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        n, sec = cpu_program_sample(wl, seconds=10.0)
        cpu = {"value": n * rows / sec, "unit": "tokens/s", "cores": 1, "kind": "port",
               "sample": f"{n} forward+backward passes of the program (batch {rows}) with the "
                         "MSE cotangent, single thread"}
    if rank == 0:
        tflops = mlp_flops(wl) / (ms / 1e3) / 1e12
        print(json.dumps({
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True,
            "steady_state": {"steps": reps, "ms_per_step": steady_ms,
                             "value": world * rows / (steady_ms / 1e3)},
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (x, targets ~ N(0,1); W ~ N(0, 1/fan_in); b = 0; seed 0)",
            "config": arm_config(a, wl, world),
            "tflops": tflops,
            "roofline": {"bound": "latency", "kernel": "whole step", "achieved": tflops,
                         "peak": None, "unit": "TFLOP/s", "frac": None, "traffic": None,
                         "note": f"{l_per} dependent launches of kernels that each take "
                                 "a few microseconds or less; no throughput roof applies"},
            "e2e": e2e, "gpu_launches": l_per * a.steps, "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }), flush=True)
    cp.close()
    if world > 1:
        torch.cuda.synchronize(dev)
        dist.barrier()
        dist.destroy_process_group()


def run_reference_program(a, wl, cores, world):
    """The oracle's program forward+backward on every host core: one
    independent replica per worker process, each step a 1 s sample."""
    import multiprocessing as mp
    steps = max(1, a.steps)
    ctx = mp.get_context("spawn")
    with ctx.Pool(cores) as pool:
        pool.map(_program_worker, [(wl, 0.2)] * cores)  # warm-up
        per_step = []
        for _ in range(steps):
            res = pool.map(_program_worker, [(wl, 1.0)] * cores)
            per_step.append(sum(n for n, _ in res) * wl["batch"] / max(t for _, t in res))
    v = sum(per_step) / steps
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": a.warmup, "ms_per_step": wl["batch"] / v * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": arm_config(a, wl, world),
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{cores} workers, each 1 s of forward+backward passes"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_gemm(a):
    """The tensor-core GEMM (dop_gemm_bf16: bf16 A [M, K], the crate's W[k * N
    + n] layout for B, bf16 C) on one shape, K timed launches between CUDA
    events, beside torch.matmul (cuBLAS) on the same operands."""
    import torch
    from dop._lib import check, lib
    if int(os.environ.get("RANK", "0")) != 0:
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    M, N, K, b_t = WORKLOADS[a.workload]["gemm"]
    g = torch.Generator(device=dev).manual_seed(0)
    A = torch.randn(M, K, generator=g, device=dev).bfloat16()
    # B(k, n) = Bs[k * N + n] (b_t = 0) or Bs[n * K + k] (b_t = 1)
    Bs = (torch.randn(N if b_t else K, K if b_t else N, generator=g, device=dev) * 0.02).bfloat16()
    Bm = Bs.t() if b_t else Bs
    C = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    stream = torch.cuda.current_stream(dev)

    def ours():
        check(lib().dop_gemm_bf16(M, N, K, A.data_ptr(), K, 0, Bs.data_ptr(), K if b_t else N, b_t,
                                  C.data_ptr(), N, 0, 0, stream.cuda_stream))

    def timed(fn):
        for _ in range(max(3, a.warmup)):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(a.steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / a.steps

    with ClockSampler(0) as clk:
        ms = timed(ours)
        ms_cublas = timed(lambda: torch.matmul(A, Bm, out=C))
    flops = 2 * M * N * K
    print(json.dumps({
        "metric": "bf16 GEMM TFLOP/s (tensor-core kernel alone)", "value": flops / ms / 1e9,
        "unit": "TFLOP/s", "n_gpus": 1, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms,
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": a.workload, "M": M, "N": N, "K": K, "b_t": b_t},
        "cublas_same_shape": {"ms": ms_cublas, "tflops": flops / ms_cublas / 1e9},
        "clocks": clk.summary(),
    }), flush=True)


def run_attention(a):
    """The tensor-core flash attention alone: dop_gqa_forward and
    dop_gqa_backward (bf16 q, k, v, o, dO; fp32 lse, delta, dq, dk, dv) on
    one shape, K timed calls of each between CUDA events; a step is one
    forward and one backward.  FLOPs count the visible (query, key) pairs:
    4 hd per pair forward, 2.5 times that backward."""
    import numpy as np
    import torch
    from dop._lib import DOP_BF16, check, lib
    if int(os.environ.get("RANK", "0")) != 0:
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, S, H, KV, hd, W = WORKLOADS[a.workload]["attention"]
    T = B * S
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(T, H, hd, generator=g, device=dev).bfloat16()
    k = torch.randn(T, KV, hd, generator=g, device=dev).bfloat16()
    v = torch.randn(T, KV, hd, generator=g, device=dev).bfloat16()
    do = torch.randn(T, H, hd, generator=g, device=dev).bfloat16()
    o, lse = torch.empty_like(q), torch.empty(B, H, S, device=dev)
    dq = torch.empty(T, H, hd, device=dev)
    dk, dv = torch.empty(T, KV, hd, device=dev), torch.empty(T, KV, hd, device=dev)
    delta = torch.empty(B * H * S, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def fwd():
        check(lib().dop_gqa_forward(B, S, H, KV, hd, W, DOP_BF16, q.data_ptr(), k.data_ptr(),
                                    v.data_ptr(), o.data_ptr(), lse.data_ptr(), sp))

    def bwd():
        check(lib().dop_gqa_backward(B, S, H, KV, hd, W, DOP_BF16, q.data_ptr(), k.data_ptr(),
                                     v.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(),
                                     delta.data_ptr(), dq.data_ptr(), dk.data_ptr(),
                                     dv.data_ptr(), sp))

    def timed(fn):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(a.steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / a.steps

    for _ in range(max(1, a.warmup)):
        fwd()
        bwd()
    torch.cuda.synchronize(dev)
    with ClockSampler(0) as clk:
        ms_f = timed(fwd)
        ms_b = timed(bwd)
    pairs = float(np.minimum(np.arange(S) + 1, W).sum()) * B * H
    ff = 4 * hd * pairs
    hbm, peak, peak_sus, src = measured_peaks()
    print(json.dumps({
        "metric": "attention fwd+bwd tokens/s (tensor-core kernels alone)",
        "value": T / ((ms_f + ms_b) / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": ms_f + ms_b, "higher_is_better": True, "dtype": "bf16",
        "data": "synthetic N(0,1) q, k, v, dO",
        "config": {"workload": a.workload, "batch": B, "seq": S, "heads": H, "kv_heads": KV,
                   "head_dim": hd, "window": W},
        "phases_ms": {"attn_fwd": ms_f, "attn_bwd": ms_b},
        "tflops": {"fwd": ff / ms_f / 1e9, "bwd": 2.5 * ff / ms_b / 1e9},
        "frac_of_bf16_peak": {"fwd": ff / ms_f / 1e9 / peak, "bwd": 2.5 * ff / ms_b / 1e9 / peak},
        "peak_source": f"{src} bf16_tflops (burst; kernels timed alone)",
        "clocks": clk.summary(),
    }), flush=True)


def _trace(msg):
    if os.environ.get("DOP_BENCH_TRACE"):
        sys.stderr.write(f"[bench {time.strftime('%H:%M:%S')}] {msg}\n")
        sys.stderr.flush()


def run_stack(a):
    """The staged block stack: plan with dop.cluster.stage_mixtral over the
    job's GPUs, run with dop.cluster.run_plan (one process per GPU, NCCL hops
    between stages, replicas' adjoints all-reduced).  A step is the whole
    global batch through every block, forward and backward."""
    import torch
    import torch.distributed as dist
    from dop import DOP_BF16, cluster, parallel
    from dop.mixtral import Block, MixtralConfig

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    world, rank = parallel.init_from_env("nccl", timeout_s=600, device=dev)
    wl = WORKLOADS[a.workload]
    gb, seq, M = wl["batch"], wl["seq"], wl["micro_batches"]
    cfg = MixtralConfig(**wl["cfg"])
    one = dict(wl["cfg"], layers=1)
    cap = int(torch.cuda.get_device_properties(dev).total_memory * 0.92)
    plan = cluster.stage_mixtral(cfg, gb, seq, M, DOP_BF16, cluster.b200s(world, cap))
    assert len(plan.stage_groups()) == math.gcd(cfg.layers, world)
    groups = {}
    for g in plan.stage_groups():  # every rank creates every group, in the same order
        grp = dist.new_group(g) if world > 1 and len(g) > 1 else None
        groups[tuple(g)] = grp
    mine = sorted(h.layer for h in plan.homes if h.device == rank and h.kind == cluster.HOME_PARAM)
    params, dparams, lenses = {}, {}, {}
    for l in mine:
        _, ll, params[l] = make_params(one, "bf16", seed=l, device=dev)
        dparams[l] = torch.zeros(ll.total, dtype=torch.float32, device=dev)
    one_cfg = MixtralConfig(**one)
    mb = gb // M
    for l, n_slots in plan.slots(rank).items():
        for k in range(n_slots):
            lenses[(l, k)] = cluster.BlockLens(Block(one_cfg, mb, seq, DOP_BF16))
    my_micro = sorted({w.micro for w in plan.windows if w.device == rank and w.micro >= 0})
    first, last = 0 in mine, cfg.layers - 1 in mine
    g = torch.Generator(device=dev).manual_seed(1000)
    xs = {m: torch.randn(mb * seq, cfg.dim, generator=g, device=dev) for m in my_micro} if first else {}
    dys = {m: torch.randn(mb * seq, cfg.dim, generator=g, device=dev) for m in my_micro} if last else {}
    buf = lambda r, c: torch.empty(r, c, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(inputs, cots):
        for t in dparams.values():
            t.zero_()
        return cluster.run_plan(plan, rank, lambda l, k: lenses[(l, k)], params, dparams, inputs,
                                cots, buf, groups=groups)

    def launches():
        return sum(x.block.launches() for x in lenses.values())

    _trace("stack plan, parameters and inputs ready")
    for _ in range(a.warmup):
        step(xs, dys)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    l0 = launches()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        ev0.record(stream)
        for _ in range(a.steps):
            step(xs, dys)
        ev1.record(stream)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
    n_launch = launches() - l0
    ms = parallel.max_over_ranks(ev0.elapsed_time(ev1) / a.steps, device=dev)
    value = gb * seq / (ms / 1e3)
    # end to end: each step's stack inputs and output cotangents copied in
    # from pinned host memory, the input gradients read back
    e2e = None
    if not a.no_e2e:
        hx = {m: t.cpu().pin_memory() for m, t in xs.items()}
        hdy = {m: t.cpu().pin_memory() for m, t in dys.items()}
        hdx = {m: torch.empty(mb * seq, cfg.dim).pin_memory() for m in xs}
        h2d = sum(t.numel() * 4 for t in hx.values()) + sum(t.numel() * 4 for t in hdy.values())
        d2h = sum(t.numel() * 4 for t in hdx.values())

        def e2e_step():
            ins = {m: t.to(dev, non_blocking=True) for m, t in hx.items()}
            cts = {m: t.to(dev, non_blocking=True) for m, t in hdy.items()}
            out = step(ins, cts)
            for m, t in out["input_grads"].items():
                hdx[m].copy_(t, non_blocking=True)
        e2e_step()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_e2e = max(1, min(3, a.steps))
        e0.record(stream)
        for _ in range(n_e2e):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ems = parallel.max_over_ranks(e0.elapsed_time(e1) / n_e2e, device=dev)
        h2d = int(parallel.max_over_ranks(h2d, device=dev) if world > 1 else h2d)
        e2e = {"value": gb * seq / (ems / 1e3), "unit": "tokens/s", "steps": n_e2e,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "note": "bytes of one rank (the largest)"}
    clk_summary = clk.summary()
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cs = wl["cpu_seq"]
        ts, used = cpu_oracle_sample(one, cs, seed=0, repeats=1)
        cpu = {"value": cs / (cfg.layers * ts[0]), "unit": "tokens/s", "cores": used,
               "kind": "port",
               "sample": f"batch 1, seq {cs} through one block at the full widths, "
                         f"{used} host threads, time x {cfg.layers} blocks"}
    if rank == 0:
        hbm, peak, peak_sus, src = measured_peaks()
        flops = cfg.layers * flops_per_step(one, gb, seq)
        tflops = flops / (ms / 1e3) / 1e12
        out = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02^2) weights, N(0,1) x and dy)",
            "config": arm_config(a, wl, world),
            "tflops": tflops, "frac_of_bf16_peak": tflops / (world * peak),
            "frac_of_bf16_sustained": tflops / (world * peak_sus),
            "roofline": {"bound": "tensor", "kernel": "whole stack step", "achieved": tflops / world,
                         "peak": peak_sus, "unit": "TFLOP/s", "frac": tflops / world / peak_sus,
                         "traffic": None,
                         "peak_source": f"{src} bf16_tflops_sustained (per GPU)"},
            "e2e": e2e, "gpu_launches": n_launch, "clocks": clk_summary, "cpu_baseline": cpu,
        }
        print(json.dumps(out), flush=True)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
        for grp in groups.values():
            if grp is not None:
                dist.destroy_process_group(grp)
        dist.destroy_process_group()


def run_ours(a):
    import torch
    import torch.distributed as dist
    from dop import DOP_BF16, DOP_F32
    from dop.mixtral import Block

    from dop import parallel
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    world, rank = parallel.init_from_env("nccl", timeout_s=600, device=dev)
    wl = WORKLOADS[a.workload]
    batch, seq = wl["batch"], wl["seq"]
    T = batch * seq
    cfg, ll, P = make_params(wl["cfg"], wl["precision"], seed=0, device=dev)  # same weights on every rank
    prec = DOP_BF16 if wl["precision"] == "bf16" else DOP_F32
    ep = use_expert_parallel(a, wl, world)
    if a.parallel == "ep" and world > 1 and not ep:
        raise SystemExit(f"--parallel ep needs bf16 and experts % {world} == 0")
    blk = Block(cfg, batch, seq, prec, ep=(rank, world) if ep else None)
    if ep:
        parallel.connect_expert_parallel(blk, device=dev)
    bias = None
    if wl["skew"]:
        bias = zipf_bias(cfg.experts).to(dev)
        blk.set_router_bias(bias)
    g = torch.Generator(device=dev).manual_seed(1000 + rank)  # each rank its own batch
    X = torch.randn(T, cfg.dim, generator=g, device=dev)
    DY = torch.randn(T, cfg.dim, generator=g, device=dev)
    Y = torch.empty_like(X)
    DX = torch.empty_like(X)
    dP = torch.zeros(ll.total, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    # data parallel: the experts' adjoints (the slice from gate0 on) are
    # reduced on a side stream while the attention half of the backward runs.
    # Expert parallel: each rank's experts' adjoints are complete on that
    # rank; only the shared slice is summed.
    side = torch.cuda.Stream(dev) if world > 1 and not ep else None
    if side is not None:
        blk.set_adjoint_stream(side)
    x0 = ll.gate0

    def reduce_dp(buf):
        if side is not None:
            with torch.cuda.stream(side):
                parallel.reduce_adjoint(buf[x0:])
        parallel.reduce_adjoint(buf[:x0])
        if side is not None:
            stream.wait_stream(side)

    def step():
        dP.zero_()
        blk.forward(P, X, Y, stream=stream)
        blk.backward(P, DY, dP, DX, stream=stream)
        if world > 1:
            reduce_dp(dP)

    _trace("params and inputs ready")
    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize(dev)
    _trace("warm-up done")
    if world > 1:
        dist.barrier()
    blk.set_timing(True)
    launches0 = blk.launches()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    phase_acc = {}
    with ClockSampler(local) as clk:
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        ev0.record(stream)
        for _ in range(a.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    # per-phase CUDA events of the last timed step (recorded on `stream`
    # inside it; read after the loop so the timed region has no host sync)
    for name, pms in blk.phase_times():
        phase_acc.setdefault(name, []).append(pms)
    _trace("timed loop done")
    launches = blk.launches() - launches0
    blk.set_timing(False)
    clk_summary = clk.summary()
    ms = parallel.max_over_ranks(ev0.elapsed_time(ev1) / a.steps, device=dev)
    value = world * T / (ms / 1e3)

    # End to end through the public call: every step copies its x and dy from
    # pinned host memory and reads the step's whole result back: y, dx and
    # the fp32 parameter adjoint.  The copies run on two copy streams and
    # every device buffer is double-buffered, so step i+1's inputs travel
    # while step i computes and step i's results return during step i+1.
    e2e = None
    if not a.no_e2e:
        hx = torch.randn(T, cfg.dim, generator=torch.Generator().manual_seed(7)).pin_memory()
        hdy = torch.randn(T, cfg.dim, generator=torch.Generator().manual_seed(8)).pin_memory()
        hy = torch.empty(T, cfg.dim, pin_memory=True)
        hdx = torch.empty(T, cfg.dim, pin_memory=True)
        hdP = torch.empty(ll.total, dtype=torch.float32, pin_memory=True)
        Xb, DYb, DXb = [X, torch.empty_like(X)], [DY, torch.empty_like(DY)], [DX, torch.empty_like(DX)]
        Yb, dPb = [Y, torch.empty_like(Y)], [dP, torch.empty_like(dP)]
        h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        ev = lambda: torch.cuda.Event()
        in_ready, step_done, out_done = [ev(), ev()], [ev(), ev()], [ev(), ev()]

        def e2e_run(n, start):
            h2d.wait_event(start)
            with torch.cuda.stream(h2d):
                Xb[0].copy_(hx, non_blocking=True)
                DYb[0].copy_(hdy, non_blocking=True)
                in_ready[0].record(h2d)
            for i in range(n):
                b = i % 2
                if i + 1 < n:  # prefetch step i+1 into the other buffer set
                    with torch.cuda.stream(h2d):
                        if i >= 1:
                            h2d.wait_event(step_done[1 - b])
                        Xb[1 - b].copy_(hx, non_blocking=True)
                        DYb[1 - b].copy_(hdy, non_blocking=True)
                        in_ready[1 - b].record(h2d)
                stream.wait_event(in_ready[b])
                if i >= 2:  # step i-2's results have left this buffer set
                    stream.wait_event(out_done[b])
                dPb[b].zero_()
                blk.forward(P, Xb[b], Yb[b], stream=stream)
                blk.backward(P, DYb[b], dPb[b], DXb[b], stream=stream)
                if world > 1:
                    reduce_dp(dPb[b])
                step_done[b].record(stream)
                with torch.cuda.stream(d2h):
                    d2h.wait_event(step_done[b])
                    hy.copy_(Yb[b], non_blocking=True)
                    hdx.copy_(DXb[b], non_blocking=True)
                    hdP.copy_(dPb[b], non_blocking=True)
                    out_done[b].record(d2h)
            stream.wait_event(out_done[(n - 1) % 2])
            if n >= 2:
                stream.wait_event(out_done[(n - 2) % 2])

        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        e2e_run(2, e0)  # warm-up of the copy path
        torch.cuda.synchronize(dev)
        _trace("e2e warm-up done")
        if world > 1:
            dist.barrier()
        n_e2e = max(2, min(a.steps, 6))
        e0.record(stream)
        e2e_run(n_e2e, e0)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ems = parallel.max_over_ranks(e0.elapsed_time(e1) / n_e2e, device=dev)
        e2e = {"value": world * T / (ems / 1e3), "unit": "tokens/s", "steps": n_e2e,
               "h2d_bytes_per_step": 2 * T * cfg.dim * 4,
               "d2h_bytes_per_step": 2 * T * cfg.dim * 4 + ll.total * 4,
               "result": "y, dx and the fp32 parameter adjoint read back every step",
               "overlap": "double-buffered device buffers and copy streams"}

    flops = flops_per_step(wl["cfg"], batch, seq)
    hbm, peak, peak_sus, src = measured_peaks()
    # dominant kernel: the expert gate/up grouped GEMM (2 * rows * D * 2I FLOPs)
    gu = phase_acc.get("expert_gate_up", [float("nan")])
    gu_ms = sum(gu) / len(gu)
    gu_flops = 2 * T * cfg.top_k * cfg.dim * 2 * cfg.intermediate
    achieved = gu_flops / (gu_ms / 1e3) / 1e12
    phases = {k: round(sum(v) / len(v), 3) for k, v in phase_acc.items()}
    gu_peak, gu_peak_src = peak_sus, f"{src} bf16_tflops_sustained (kernel timed inside a long step)"
    if wl["precision"] == "f32":
        # 3xTF32: three tf32 products per fp32 product, tf32 at half the bf16
        # dense rate (NVIDIA's B200 figures: 1.1 / 2.25 PFLOP/s)
        gu_peak = peak_sus * (1.1 / 2.25) / 3
        gu_peak_src = (f"{src} bf16_tflops_sustained x 1.1/2.25 (tf32 / bf16 dense) / 3 "
                       "(three tf32 products per fp32 product)")

    _trace("e2e done")
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cs = wl["cpu_seq"]
        ts, used = cpu_oracle_sample(wl["cfg"], cs, seed=0, repeats=1)
        cpu = {"value": cs / ts[0], "unit": "tokens/s", "cores": used, "kind": "port",
               "sample": f"batch 1, seq {cs} at the full widths of {a.workload}, "
                         f"one fwd+bwd on {used} host threads"}

    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": wl["precision"],
            "data": "synthetic (seeded N(0,0.02^2) weights, N(0,1) x and dy)",
            "config": arm_config(a, wl, world),
            "tflops": flops / (ms / 1e3) / 1e12,
            "frac_of_bf16_peak": flops / (ms / 1e3) / 1e12 / peak,
            "frac_of_bf16_sustained": flops / (ms / 1e3) / 1e12 / peak_sus,
            # the gate/up GEMM is timed inside a long step: sustained peak
            "roofline": {"bound": "tensor", "kernel": "expert_gate_up", "achieved": achieved,
                         "peak": gu_peak, "unit": "TFLOP/s", "frac": achieved / gu_peak,
                         "traffic": (GATE_UP_TRAFFIC
                                     if a.workload in ("mixtral8x7b_block",
                                                       "mixtral8x7b_block_skewed") else None),
                         "traffic_source": ("dram bytes read + written by one launch at batch 8, "
                                            "seq 4096 (one-pass ncu capture, -c 1); algorithmic "
                                            "8.16e9 B: rows 0.55, weights 1.88, g/u/h 5.73"),
                         "peak_source": gu_peak_src},
            "phases_ms": phases,
            "e2e": e2e, "gpu_launches": launches // max(1, a.steps) * a.steps,
            "clocks": clk_summary, "cpu_baseline": cpu,
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        # every rank's kernels are done before any rank unmaps or frees a
        # workspace its peers read
        torch.cuda.synchronize(dev)
        dist.barrier()
        blk.close()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--parallel", default="auto", choices=["auto", "dp", "ep"],
                    help="N > 1: expert parallel (auto when the experts split evenly over "
                         "the ranks and the lens is bf16) or data parallel")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="profiler run: no CPU baseline, no e2e, warm-up may be < 3")
    a = ap.parse_args()
    if a.profile:
        a.no_cpu_baseline = a.no_e2e = True
    elif a.warmup < 3 and a.impl == "ours":
        a.warmup = 3
    if a.impl == "reference":
        run_reference(a)
    elif WORKLOADS[a.workload].get("program"):
        run_program(a)
    elif WORKLOADS[a.workload].get("gemm"):
        run_gemm(a)
    elif WORKLOADS[a.workload].get("attention"):
        run_attention(a)
    elif WORKLOADS[a.workload].get("stack"):
        run_stack(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
