"""Benchmark of the SPARC hot path on B200 (one JSON line on rank 0).

Default workload (the configuration the metric is quoted on): one
SPARCMixer(512) layer, forward + backward of sum(y * g), B=8 x T=2048 tokens per GPU, float32,
parameters from the default init under torch.manual_seed(0), synthetic x, g ~ N(0, 1).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload layer|layer5|stack|real|decode|projection|projection16|rtrl|complex]

Multi-GPU: one process per GPU (torchrun), batch-sharded data parallelism (each rank runs the
per-GPU batch: weak scaling), parameter gradients summed every step by the library's
gradient reduction kernel, which also sums them over the ranks through NVLink peer memory
(`--allreduce peer`: a separate peer-memory all-reduce kernel; `nccl`: NCCL's all-reduce);
timing is the max over ranks of per-step CUDA-event times.

Timing: W untimed warm-up steps; the step is captured once in a CUDA graph and replayed. Before
every timed step L2 is flushed by writing a 512 MiB buffer (the config-2 inputs fit in L2);
CUDA events bracket the step only, and K steps are bracketed by a barrier and a device
synchronise. `e2e` repeats the step through the public module API from pinned host buffers
(the host->device copy of the batch x, forward, a loss (a fixed linear readout of y resident on
the device, whose gradient is the device-timed step's g), backward and the device->host read of
the loss inside the timed region).

`--impl reference` times the reference algorithm's CPU restatement (the oracle) on the host
cores instead (the reference itself is Python/Triton with no CPU kernel for this path).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import json
import math
import multiprocessing as mp
import os
import re
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

WORKLOADS = {
    "layer": dict(workload="sparc_mixer_layer_fwd_bwd", batch=8, seq_len=2048, width=512,
                  dtype="float32", config_index=1),
    "layer5": dict(workload="sparc_mixer_layer_fwd_bwd_config5_share", batch=8, seq_len=16384, width=2048,
                   dtype="bfloat16", config_index=4),
    "stack": dict(workload="sparc_4layer_rmsnorm_residual_stack_fwd_bwd", batch=64, seq_len=16384,
                  width=2048, dtype="bfloat16", layers=4, config_index=4),
    "real": dict(workload="real_scan_fwd_bwd", batch=16, seq_len=8192, channels=16384,
                 dtype="bfloat16", config_index=2),
    "decode": dict(workload="sparc_decode_step", batch=256, width=2048, steps=1024,
                   dtype="bfloat16", config_index=3),
    # the projection variant (JAX sequence layer) at config 2's token count and state size
    "projection": dict(workload="sparc_sequence_layer_fwd_bwd", batch=8, seq_len=2048, width=512, modes=256,
                       dtype="float32", config_index=0),
    # the same in bfloat16: the products on the tensor cores (tcgen05)
    "projection16": dict(workload="sparc_sequence_layer_fwd_bwd_bf16", batch=8, seq_len=16384, width=2048,
                         modes=1024, dtype="bfloat16", config_index=0),
    # the generic complex scan (the reference's complex_scan, its "triton" backend for more than
    # 512 modes) at the config-5 layer's mode count, float32
    "complex": dict(workload="complex_scan_fwd_bwd", batch=8, seq_len=8192, modes=1024, dtype="float32",
                    config_index=4),
    # one RTRL cell step (trace update + trace gradients) at a size whose traces exceed L2
    "rtrl": dict(workload="sparc_rtrl_cell_step_fwd_bwd", batch=64, width=512, modes=512,
                 dtype="float32", config_index=0),
}
METRIC = "SPARC layer fwd+bwd tokens/sec and % HBM roofline at 1/2/4/8 B200"


# ----------------------------------------------------------------------------- helpers
def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _bf16_peak(sustained=False):
    """Measured dense bf16 TFLOP/s: the burst figure (a product timed alone) or, with `sustained`,
    the figure of back-to-back products under the power cap (a product inside a long step)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        if sustained and "bf16_tflops_sustained" in d:
            return float(d["bf16_tflops_sustained"])
        return float(d["bf16_tflops"])
    return 1400.0 if sustained else 1590.0


# Kernels one mixer fwd+bwd launches: fwd summary, carry scan, replay; bwd summary, carry scan,
# gradients, parameter-gradient reduction.
MIXER_LAUNCHES = 7


def mixer_kernel_bytes(B, T, W, s, chunk):
    """Algorithmic DRAM bytes of each mixer kernel per launch: every input it must read once and
    every output it must write once (activations W*s bytes per token, saved controls 32 bytes
    per token, chunk maps 16 bytes and chunk states 8 bytes per chunk and mode). The replay also
    writes every token's state (W*s per token) for the gradient kernel, which reads them with x
    and dy instead of replaying the recurrence."""
    M = W // 2
    bt = B * T
    chunks = -(-T // chunk)
    act = W * s * bt
    ctl = 32 * bt
    agg = 16 * B * chunks * M
    car = 8 * B * chunks * M
    return {"mixer_fwd_summary_kernel": act + ctl + agg,
            "mixer_carry_scan_kernel(fwd)": agg + car,
            "mixer_fwd_replay_kernel": 3 * act + ctl + car,
            "mixer_bwd_summary_kernel": 2 * act + ctl + agg,
            "mixer_carry_scan_kernel(bwd)": agg + car,
            "mixer_bwd_grad_kernel": 4 * act + ctl + 2 * car}


def profile_value(kernel: str, workload: str, key: str = "traffic_bytes_per_launch"):
    """A per-launch figure of `kernel` (DRAM bytes, warp instructions) from the committed ncu
    summary, if there is one."""
    path = os.path.join(ROOT, "profiles", f"{kernel}_{workload}.md")
    if not os.path.exists(path):
        return None
    m = re.search(key + r":\s*([0-9.eE+]+)", open(path).read())
    return float(m.group(1)) if m else None


def profile_traffic(kernel: str, workload: str):
    return profile_value(kernel, workload)


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms while running."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            t0 = time.time()
            while not self.lines and time.time() - t0 < 2.0:  # short regions: keep one sample
                time.sleep(0.02)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                smax = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": smax, "reasons": [], "samples": 0}
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


_REDUCERS = []


def make_reducer(args, params, fused_ok=False):
    """The per-step exchange of the parameter gradients for N > 1: inside the mixer kernels'
    gradient reduction (`fused`, the default where every parameter is a mixer / block parameter),
    the library's peer-memory all-reduce kernel after the backward (`peer`), or NCCL's all-reduce
    of the packed gradients (`nccl`). Returns the callable to run after the backward, or None."""
    import torch.distributed as dist

    if not dist.is_initialized() or dist.get_world_size() == 1:
        return None
    from sparc_b200.ddp import FusedGradExchange, GradAllReduce, PeerGradAllReduce

    params = [p for p in params if p.requires_grad]
    mode = args.allreduce
    if mode == "fused" and not fused_ok:
        mode = "peer"
    if mode == "fused" and dist.get_world_size() <= 8:
        _REDUCERS.append(FusedGradExchange())
        return None
    if mode == "peer" and dist.get_world_size() <= 8 and len(params) <= 64:
        r = PeerGradAllReduce(params)
        _REDUCERS.append(r)
        return r
    return GradAllReduce(params)


# ----------------------------------------------------------------------------- CPU oracle
def _oracle_rows(args):
    """float64 oracle forward+backward of a block of batch rows (run in a worker process)."""
    import numpy as np
    from threadpoolctl import threadpool_limits

    from oracle import sparc_oracle as O

    seed, seq_len, width, params = args
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((1, seq_len, width))
    g = rng.standard_normal((1, seq_len, width))
    with threadpool_limits(1):
        P = O.Params.from_mapping(params)
        y, _, _ = O.sparc_forward(x, P)
        grads = O.sparc_backward(x, P, g)
    return float(np.abs(y).sum()), {k: grads[k] for k in O.PARAM_NAMES}


class OraclePool:
    """Spawned worker processes that run the float64 oracle forward+backward, one batch row of
    the layer workload per task (each worker draws its row's x and g from the row's seed); a
    round is every row of the batch (the pool starts before any timing and before GPU work)."""

    def __init__(self, batch, seq_len, width, workers, seed=0):
        import torch

        from oracle import sparc_oracle as O

        torch.manual_seed(seed)
        params = O.init_params(width, lambda n: torch.rand(n).numpy())
        self.rows = [(seed * 1000003 + i, seq_len, width, params) for i in range(batch)]
        self.seq_len = seq_len
        self.ex = cf.ProcessPoolExecutor(max_workers=workers, mp_context=mp.get_context("spawn"))
        list(self.ex.map(_oracle_rows, self.rows[:1]))  # start the workers

    def round(self):
        """One round over the rows; returns (seconds, tokens)."""
        t0 = time.perf_counter()
        list(self.ex.map(_oracle_rows, self.rows))
        return time.perf_counter() - t0, len(self.rows) * self.seq_len

    def close(self):
        self.ex.shutdown()


def cpu_oracle_layer(batch, seq_len, width, workers, seconds, seed=0):
    """Time the CPU oracle on the layer workload for about `seconds` (at least one round).
    Returns (tokens/s, tokens processed, rows per round)."""
    pool = OraclePool(batch, seq_len, width, workers, seed)
    el, tokens = 0.0, 0
    while True:
        s, t = pool.round()
        el += s
        tokens += t
        if el >= seconds:
            break
    pool.close()
    return tokens / el, tokens, len(pool.rows)


# ----------------------------------------------------------------------------- our arm
def _dist():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def _time_steps(step_fn, steps, flush, world, device, soak_s=0.3):
    """Per-step CUDA event times (ms) of `step_fn`, L2 flushed before each step; max over
    ranks of the summed time. Untimed steps for about `soak_s` seconds come first (the same
    count on every rank), so that the clock sampler around this call sees the GPU under load."""
    import torch
    import torch.distributed as dist

    if soak_s > 0:
        torch.cuda.synchronize(device)
        t0 = time.time()
        flush()
        step_fn()
        torch.cuda.synchronize(device)
        n = torch.tensor([int(min(4000, soak_s / max(time.time() - t0, 1e-5)))], device=device)
        if world > 1:
            dist.all_reduce(n, op=dist.ReduceOp.MAX)
        for _ in range(int(n.item())):
            flush()
            step_fn()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    for i in range(steps):
        flush()
        starts[i].record()
        step_fn()
        ends[i].record()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    per = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total = torch.tensor([sum(per)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(total, op=dist.ReduceOp.MAX)
    return float(total.item()), per


def run_layer(args, wl, world, rank, local):
    import torch
    import torch.distributed as dist

    import sparc_b200
    from sparc_b200 import _lib

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    B, T, W = wl["batch"], wl["seq_len"], wl["width"]
    dtype = getattr(torch, wl["dtype"])
    torch.manual_seed(0)
    model = sparc_b200.SPARCMixer(W).to(device)
    gen = torch.Generator(device=device).manual_seed(1000 + rank)
    x = torch.randn(B, T, W, generator=gen, device=device).to(dtype)
    g = torch.randn(B, T, W, generator=gen, device=device).to(dtype)
    reducer = make_reducer(args, model.parameters(), fused_ok=True)
    s = 4 if dtype == torch.float32 else 2
    small = 2 * B * T * W * s < (256 << 20)  # inputs that could sit in the 126 MB L2
    flush_buf = torch.empty(512 << 20 if small else 16, dtype=torch.uint8, device=device)

    def flush():
        if small:
            flush_buf.fill_(1)

    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            model.zero_grad(set_to_none=True)
            y, _ = model(x)
            y.backward(g)
            if reducer is not None:
                reducer()  # also initialises the NCCL communicator before the graph capture
    torch.cuda.current_stream(device).wait_stream(stream)
    torch.cuda.synchronize(device)
    model.zero_grad(set_to_none=True)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        y, _ = model(x)
        y.backward(g)
        if reducer is not None:
            reducer()  # the one exchange step (NCCL all-reduce of the parameter gradients)
    del y  # drop the captured autograd graph (its gradient-accumulation nodes belong to `stream`)

    def step():
        graph.replay()

    for _ in range(args.warmup):
        flush()
        step()
    with ClockSampler(local) as clocks:
        total_ms, per = _time_steps(step, args.steps, flush, world, device)
    ms = total_ms / args.steps
    tokens_step = B * T * world
    value = tokens_step / (ms / 1e3)

    # per-kernel device time from the library's CUDA-event timing (sparc_timing_*), same inputs,
    # outside the graph; the roofline line is the dominant kernel's
    peak, peak_kind = measured_peaks()
    L = _lib.lib()
    chunk = int(L.sparc_mixer_chunk_tokens(_lib.dtype_code(dtype)))
    kbytes = mixer_kernel_bytes(B, T, W, s, chunk)
    xr = x.clone().requires_grad_(True)
    for _ in range(2):
        yy, _ = model(xr)
        yy.backward(g)
    torch.cuda.synchronize(device)
    L.sparc_timing_enable(1)
    _lib.kernel_times(reset_only=True)
    for _ in range(args.steps):
        flush()
        yy, _ = model(xr)
        flush()
        yy.backward(g)
        xr.grad = None
        model.zero_grad(set_to_none=True)
    torch.cuda.synchronize(device)
    times = _lib.kernel_times()
    L.sparc_timing_enable(0)
    kern = {}
    for name, (tot, cnt) in times.items():
        kms = tot / cnt
        kb = kbytes.get(name)
        kern[name] = {"ms": round(kms, 4), "launches_per_step": round(cnt / args.steps, 2), "algorithmic_bytes": kb,
                      "GBps": round(kb / (kms / 1e3) / 1e9, 1) if kb else None}
    # the dominant kernel among those with algorithmic bytes (with N ranks, the reduction kernel
    # also waits for the other ranks' gradients, so its time is not a bandwidth figure)
    dom = max((k for k in kern if kern[k]["GBps"]), key=lambda k: kern[k]["ms"])
    achieved = kern[dom]["GBps"]
    traffic = profile_traffic(dom, f"layer_b{B}_t{T}_w{W}_{'fp32' if s == 4 else 'bf16'}")
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic, "kernel": dom,
                "peak_source": peak_kind, "kernels": kern,
                "step_frac": round(5 * W * s * B * T / (ms / 1e3) / 1e9 / peak, 4)}
    # the ceiling that binds these kernels: instruction issue (148 SMs x 4 schedulers x one
    # warp-instruction per cycle), with the dominant kernel's instruction count from its ncu
    # summary and the SM clock sampled under load
    inst = profile_value(dom, f"layer_b{B}_t{T}_w{W}_{'fp32' if s == 4 else 'bf16'}", "warp_instructions_per_launch")
    sm_mhz = (clocks.summary() or {}).get("sm_mhz")
    if inst and sm_mhz and kern[dom]["ms"]:
        issue_us = inst / (148 * 4) / (sm_mhz * 1e6) * 1e6
        roofline["issue"] = {"kernel": dom, "warp_instructions": int(inst), "issue_bound_us": round(issue_us, 2),
                             "measured_us": round(kern[dom]["ms"] * 1e3, 2),
                             "frac": round(issue_us / (kern[dom]["ms"] * 1e3), 4), "sm_mhz": sm_mhz}

    # end to end through the public API: every step copies its batch x from pinned host memory
    # (on a copy stream, double-buffered, so that step i+1's copy overlaps step i's compute),
    # runs forward, a loss and backward, and reads the loss back to pinned host memory. The loss
    # is a fixed linear readout of y, sum(y * g) (g resident on the device, like the weights of
    # a head), so its gradient is the same g as the device-timed step's
    xh = x.cpu().pin_memory()
    gd = g.float()
    loss_h = torch.empty((), dtype=torch.float32).pin_memory()
    main = torch.cuda.current_stream(device)
    copy_stream = torch.cuda.Stream(device)
    bufs = [torch.empty_like(x) for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    for e in free:
        e.record(main)

    def h2d(i):
        k = i % 2
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(free[k])
            bufs[k].copy_(xh, non_blocking=True)
            copied[k].record(copy_stream)

    def e2e_steps(n):
        h2d(0)
        for i in range(n):
            if i + 1 < n:
                h2d(i + 1)
            k = i % 2
            main.wait_event(copied[k])
            xd = bufs[k]
            yy, _ = model(xd)
            loss = (yy.float() * gd).sum()
            loss.backward()
            if reducer is not None:
                reducer()
            free[k].record(main)
            loss_h.copy_(loss.detach(), non_blocking=True)
            model.zero_grad(set_to_none=True)

    e2e_steps(2)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(main)
    e2e_steps(args.steps)
    ev1.record(main)
    torch.cuda.synchronize(device)
    e2e_ms = torch.tensor([ev0.elapsed_time(ev1) / args.steps], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())
    e2e = {"value": round(tokens_step / (e2e_ms / 1e3), 1), "unit": "tokens/s",
           "h2d_bytes_per_step": int(B * T * W * s), "d2h_bytes_per_step": 4,
           "ms_per_step": round(e2e_ms, 4),
           "path": "SPARCMixer.forward, loss sum(y * g) (g resident), backward, from pinned host x "
                   "(copies double-buffered on a copy stream); loss read back"}
    sparc_b200.check_status()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        workers = min(8, os.cpu_count() or 1)
        tps, toks, rows = cpu_oracle_layer(B, T, W, workers, seconds=args.cpu_seconds)
        cpu = {"value": round(tps, 1), "unit": "tokens/s", "cores": workers, "kind": "port",
               "sample": f"{toks} tokens: float64 numpy oracle fwd+bwd, {rows} batch rows of "
                         f"T={T}, W={W} per round, one row per process"}
    del graph
    return dict(value=value, ms=ms, roofline=roofline, e2e=e2e, cpu=cpu, clocks=clocks.summary(),
                launches=MIXER_LAUNCHES * args.steps, per_step_ms=per, tokens_step=tokens_step, chunk=chunk)


def run_stack(args, wl, world, rank, local):
    import torch

    import sparc_b200
    from sparc_b200.stack import SPARCStack

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    gb, T, W, L = wl["batch"], wl["seq_len"], wl["width"], wl["layers"]
    B = gb // world
    torch.manual_seed(0)
    model = SPARCStack(W, L).to(device)
    gen = torch.Generator(device=device).manual_seed(1000 + rank)
    x = torch.randn(B, T, W, generator=gen, device=device).to(torch.bfloat16)
    g = torch.randn(B, T, W, generator=gen, device=device).to(torch.bfloat16)
    reducer = make_reducer(args, model.parameters(), fused_ok=True)

    def step():
        model.zero_grad(set_to_none=True)
        out = model(x)
        out.backward(g)
        if reducer is not None:
            reducer()

    for _ in range(max(3, args.warmup)):
        step()

    def noflush():
        pass

    with ClockSampler(local) as clocks:
        total_ms, per = _time_steps(step, args.steps, noflush, world, device)
    ms = total_ms / args.steps
    value = gb * T / (ms / 1e3)
    peak, kind = measured_peaks()
    fused_min = L * 5 * W * 2 * gb * T / world
    # as implemented: every block kernel's algorithmic bytes (saved controls, chunk maps and
    # states included); the block's reverse summary reads the relu bits the replay wrote
    # (W/8 bytes per token each way) instead of the mixer's output y
    per_layer = sum(mixer_kernel_bytes(B, T, W, 2, 16).values()) - W * 2 * B * T + 2 * (W // 8) * B * T
    roofline = {"bound": "hbm", "achieved": round(fused_min / (ms / 1e3) / 1e9, 1), "peak": peak,
                "unit": "GB/s", "frac": round(fused_min / (ms / 1e3) / 1e9 / peak, 4), "traffic": None,
                "kernel": "whole step (L*5*W*s bytes/token)", "peak_source": kind,
                "bytes_per_token": {"fused_minimum": L * 5 * W * 2,
                                    "as_implemented": round(L * per_layer / (B * T), 1)}}
    sparc_b200.check_status()
    return dict(value=value, ms=ms, roofline=roofline, e2e=None, cpu=None, clocks=clocks.summary(),
                launches=MIXER_LAUNCHES * L * args.steps, per_step_ms=per, tokens_step=gb * T)


def run_complex(args, wl, world, rank, local):
    """complex_scan forward + backward (sparc_b200.complex: chunk maps, cluster carry scan,
    replay; the backward in reverse) on [B, L, M] float32 operands larger than L2."""
    import torch

    import sparc_b200
    from sparc_b200 import _lib

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    B, T, M = wl["batch"], wl["seq_len"], wl["modes"]
    gen = torch.Generator(device=device).manual_seed(rank)
    rad = 0.99 + 0.0099 * torch.rand(B, T, M, generator=gen, device=device)
    ang = 0.3 * torch.randn(B, T, M, generator=gen, device=device)
    ops = [(rad * torch.cos(ang)), (rad * torch.sin(ang)), 0.5 * torch.randn(B, T, M, generator=gen, device=device),
           0.5 * torch.randn(B, T, M, generator=gen, device=device)]
    del rad, ang
    gr, gi = torch.randn(B, T, M, generator=gen, device=device), torch.randn(B, T, M, generator=gen, device=device)
    for t in ops:
        t.requires_grad_(True)

    def step():
        for t in ops:
            t.grad = None
        out_r, out_i = sparc_b200.complex_scan(*ops)
        torch.autograd.backward((out_r, out_i), (gr, gi))

    for _ in range(max(3, args.warmup)):
        step()
    with ClockSampler(local) as clocks:
        total_ms, per = _time_steps(step, args.steps, lambda: None, world, device)
    ms = total_ms / args.steps
    peak, kind = measured_peaks()
    L = _lib.lib()
    torch.cuda.synchronize(device)
    L.sparc_timing_enable(1)
    _lib.kernel_times(reset_only=True)
    for _ in range(args.steps):
        step()
    torch.cuda.synchronize(device)
    times = _lib.kernel_times()
    L.sparc_timing_enable(0)
    n = B * T * M * 4  # bytes of one float32 [B, L, M] array
    # algorithmic bytes per launch: summaries read a, b (fwd) / a, grad_out (bwd): 4 arrays;
    # the replay reads a, b and writes out: 6; the gradient kernel reads a, grad_out, out and
    # writes four gradients: 10; the carry scans read the chunk maps (16 bytes per (row, chunk,
    # mode)) and write the carries (8)
    maps = B * -(-T // 32) * M * 24
    kbytes = {"complex_fwd_summary_kernel": 4 * n, "complex_fwd_replay_kernel": 6 * n,
              "complex_bwd_summary_kernel": 4 * n, "complex_bwd_grad_kernel": 10 * n,
              "complex_carry_scan(fwd)": maps, "complex_carry_scan(bwd)": maps}
    kern = {}
    for name, (tot, cnt) in times.items():
        kms = tot / cnt
        kb = kbytes.get(name)
        kern[name] = {"ms": round(kms, 4), "launches_per_step": round(cnt / args.steps, 2), "algorithmic_bytes": kb,
                      "GBps": round(kb / (kms / 1e3) / 1e9, 1) if kb else None}
    dom = max((k for k in kern if kern[k]["GBps"]), key=lambda k: kern[k]["ms"])
    achieved = kern[dom]["GBps"]
    # the step's minimum: forward reads a, b and writes out (6 arrays), backward reads a, out,
    # grad_out and writes four gradients (10)
    step_bytes = 16 * n
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "traffic": None, "kernel": dom, "peak_source": kind, "kernels": kern,
                "step_frac": round(step_bytes / (ms / 1e3) / 1e9 / peak, 4)}
    return dict(value=B * T * world / (ms / 1e3), ms=ms, roofline=roofline, e2e=None, cpu=None,
                clocks=clocks.summary(), launches=6 * args.steps, per_step_ms=per, tokens_step=B * T * world)


def run_real(args, wl, world, rank, local):
    import torch

    import sparc_b200

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    B, T, D = wl["batch"], wl["seq_len"], wl["channels"]
    gen = torch.Generator(device=device).manual_seed(rank)
    a = torch.sigmoid(torch.logit(0.9 + 0.099 * torch.rand(B, T, D, generator=gen, device=device))).to(torch.bfloat16)
    b = (0.5 * torch.randn(B, T, D, generator=gen, device=device)).to(torch.bfloat16)
    g = torch.randn(B, T, D, generator=gen, device=device).to(torch.bfloat16)
    a.requires_grad_(True)
    b.requires_grad_(True)

    def step():
        a.grad = None
        b.grad = None
        out = sparc_b200.real_chunk_scan(a, b, 128)
        out.backward(g)

    for _ in range(max(3, args.warmup)):
        step()
    with ClockSampler(local) as clocks:
        total_ms, per = _time_steps(step, args.steps, lambda: None, world, device)
    ms = total_ms / args.steps
    peak, kind = measured_peaks()
    byts = 16 * D * B * T
    # per-kernel device time from the library's CUDA-event timing, same inputs (larger than L2):
    # forward 3 D s bytes per token (read a, b; write out), backward 5 D s (read a, b, grad_out;
    # write grad_a, grad_b); the line's roofline is the dominant kernel's
    from sparc_b200 import _lib

    L = _lib.lib()
    torch.cuda.synchronize(device)
    L.sparc_timing_enable(1)
    _lib.kernel_times(reset_only=True)
    for _ in range(args.steps):
        step()
    torch.cuda.synchronize(device)
    times = _lib.kernel_times()
    L.sparc_timing_enable(0)
    kbytes = {"real_fwd_kernel": 3 * 2 * D * B * T, "real_bwd_kernel": 5 * 2 * D * B * T}
    kern = {}
    for name, (tot, cnt) in times.items():
        kms = tot / cnt
        kb = kbytes.get(name)
        kern[name] = {"ms": round(kms, 4), "launches_per_step": round(cnt / args.steps, 2), "algorithmic_bytes": kb,
                      "GBps": round(kb / (kms / 1e3) / 1e9, 1) if kb else None}
    dom = max((k for k in kern if kern[k]["GBps"]), key=lambda k: kern[k]["ms"])
    achieved = kern[dom]["GBps"]
    traffic = profile_traffic(dom, f"real_b{B}_t{T}_c{D}_bf16")
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "traffic": traffic, "kernel": dom, "peak_source": kind, "kernels": kern,
                "step_frac": round(byts / (ms / 1e3) / 1e9 / peak, 4)}
    # end to end through real_chunk_scan: a, b and grad_out copied from pinned host memory every step,
    # out's sum read back (the host link bounds it: 6 bytes per element cross PCIe)
    ah, bh, gh = (t.detach().cpu().pin_memory() for t in (a, b, g))
    loss_h = torch.empty((), dtype=torch.float32).pin_memory()
    ad, bd, gd = torch.empty_like(a), torch.empty_like(b), torch.empty_like(g)

    def e2e_step():
        ad.copy_(ah, non_blocking=True)
        bd.copy_(bh, non_blocking=True)
        gd.copy_(gh, non_blocking=True)
        aa = ad.detach().requires_grad_(True)
        bb = bd.detach().requires_grad_(True)
        out = sparc_b200.real_chunk_scan(aa, bb, 128)
        out.backward(gd)
        loss_h.copy_(out.detach().float().sum(), non_blocking=True)

    e2e_step()
    e_steps = max(2, min(args.steps, 5))
    e_ms, _ = _time_steps(e2e_step, e_steps, lambda: None, world, device)
    e_ms /= e_steps
    e2e = {"value": round(B * T * world / (e_ms / 1e3), 1), "unit": "tokens/s",
           "h2d_bytes_per_step": 3 * 2 * B * T * D, "d2h_bytes_per_step": 4, "ms_per_step": round(e_ms, 4),
           "path": "real_chunk_scan forward/backward from pinned host a, b, grad_out"}
    return dict(value=B * T * world / (ms / 1e3), ms=ms, roofline=roofline, e2e=e2e, cpu=None,
                clocks=clocks.summary(), launches=2 * args.steps, per_step_ms=per, tokens_step=B * T * world)


def run_decode(args, wl, world, rank, local):
    import torch

    import sparc_b200

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    B, W, S = wl["batch"], wl["width"], wl["steps"]
    torch.manual_seed(0)
    m = sparc_b200.SPARCMixer(W).to(device)
    m.prepare_inference()
    gen = torch.Generator(device=device).manual_seed(rank)
    xs = torch.randn(S, B, W, generator=gen, device=device).to(torch.bfloat16)
    st0 = (torch.zeros(B, W // 2, device=device), torch.zeros(B, W // 2, device=device))

    def roll():
        st = st0
        for s in range(S):
            _, st = m.step(xs[s], st, None)
        return st

    roll()
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        roll()
    torch.cuda.current_stream(device).wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        roll()
    for _ in range(args.warmup):
        graph.replay()
    with ClockSampler(local) as clocks:
        total_ms, per = _time_steps(graph.replay, args.steps, lambda: None, world, device)
    ms = total_ms / args.steps
    us_step = ms * 1e3 / S
    peak, kind = measured_peaks()
    byts = 12 * W * B
    roofline = {"bound": "hbm", "achieved": round(byts / (us_step / 1e6) / 1e9, 1), "peak": peak, "unit": "GB/s",
                "frac": round(byts / (us_step / 1e6) / 1e9 / peak, 4), "traffic": None,
                "kernel": "decode_kernel", "peak_source": kind, "us_per_step": round(us_step, 3)}
    del graph
    return dict(value=B * S * world / (ms / 1e3), ms=ms, roofline=roofline, e2e=None, cpu=None,
                clocks=clocks.summary(), launches=S * args.steps, per_step_ms=per, tokens_step=B * S * world)


def run_projection(args, wl, world, rank, local):
    """SPARCSequenceLayer forward + backward (content / projection / readout products and the
    recurrence in the mixer kernels' projection mode), captured in a CUDA graph."""
    import torch

    import sparc_b200
    from sparc_b200 import _lib

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    B, T, W, M = wl["batch"], wl["seq_len"], wl["width"], wl["modes"]
    torch.manual_seed(0)
    layer = sparc_b200.SPARCSequenceLayer(W, M).to(device)
    gen = torch.Generator(device=device).manual_seed(1000 + rank)
    dtype = getattr(torch, wl["dtype"])
    x = torch.randn(B, T, W, generator=gen, device=device).to(dtype)
    g = torch.randn(B, T, W, generator=gen, device=device).to(dtype)
    reducer = make_reducer(args, layer.parameters())
    flush_buf = torch.empty(512 << 20, dtype=torch.uint8, device=device)
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            layer.zero_grad(set_to_none=True)
            layer(x).backward(g)
            if reducer is not None:
                reducer()
    torch.cuda.current_stream(device).wait_stream(stream)
    torch.cuda.synchronize(device)
    layer.zero_grad(set_to_none=True)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        layer(x).backward(g)
        if reducer is not None:
            reducer()
    for _ in range(args.warmup):
        flush_buf.fill_(1)
        graph.replay()
    with ClockSampler(local) as clocks:
        total_ms, per = _time_steps(graph.replay, args.steps, lambda: flush_buf.fill_(1), world, device)
    ms = total_ms / args.steps
    # per-kernel times of the recurrence (library timing, outside the graph)
    L = _lib.lib()
    L.sparc_timing_enable(1)
    _lib.kernel_times(reset_only=True)
    for _ in range(args.steps):
        flush_buf.fill_(1)
        layer(x).backward(g)
        layer.zero_grad(set_to_none=True)
    torch.cuda.synchronize(device)
    times = _lib.kernel_times()
    L.sparc_timing_enable(0)
    kern = {k: round(t / n, 4) for k, (t, n) in times.items()}
    peak, kind = measured_peaks()
    # the recurrence's algorithmic bytes: content u (2M values per token) read by the forward
    # summary and replay, states h written; u, dh read and du written by the backward
    byts = 5 * 2 * M * x.element_size() * B * T
    rec_ms = sum(v for k, v in kern.items() if k.startswith("mixer_"))
    roofline = {"bound": "hbm", "achieved": round(byts / (rec_ms / 1e3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                "frac": round(byts / (rec_ms / 1e3) / 1e9 / peak, 4), "traffic": None,
                "kernel": "the seven recurrence kernels (projection mode), 5 x 2M x s bytes per token",
                "peak_source": kind, "kernels_ms": kern, "recurrence_ms": round(rec_ms, 4)}
    if "proj_gemm_kernel" in times:  # tensor-core products: 2 x 2M x W flops per token each, six per step
        # a product's time includes its split-k finish launch where it has one
        tot, n = times["proj_gemm_kernel"]
        tot += times.get("proj_gemm_finish_kernel", (0.0, 0))[0]
        gms = tot / n
        split = 3 if x.dtype == torch.float32 else 1  # float32 operands: three bf16 terms along k
        tf = 2.0 * 2 * M * W * B * T * split / (gms / 1e3) / 1e12
        # the products run back to back inside the step (milliseconds long, under the power cap):
        # the sustained measured peak is the denominator; the burst one is reported beside it
        roofline["tensor"] = {"kernel": "proj_gemm_kernel (+ proj_gemm_finish_kernel)", "ms_per_launch": round(gms, 4),
                              "TFLOPs": round(tf, 1), "peak_TFLOPs": _bf16_peak(sustained=True),
                              "peak_kind": "sustained (measured)", "frac": round(tf / _bf16_peak(sustained=True), 4),
                              "peak_burst_TFLOPs": _bf16_peak(), "frac_of_burst": round(tf / _bf16_peak(), 4),
                              "flops": "2 x tokens x 2M x W per product" + (" x 3 (bf16 split of float32)" if split == 3 else "")}
    del graph
    # every launch of the library in the timed steps (the colsum entry times its two launches
    # as one pair)
    launches = sum(n for _, n in times.values()) + times.get("proj_colsum_kernel", (0, 0))[1]
    return dict(value=B * T * world / (ms / 1e3), ms=ms, roofline=roofline, e2e=None, cpu=None,
                clocks=clocks.summary(), launches=launches, per_step_ms=per,
                tokens_step=B * T * world)


def run_rtrl(args, wl, world, rank, local):
    """One SPARCRTRLCell step with a loss on its output (trace update, trace gradients and the
    content / projection products), batch rows as tokens; traces live in HBM (> L2)."""
    import torch

    import sparc_b200
    from sparc_b200 import _lib

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    B, W, M = wl["batch"], wl["width"], wl["modes"]
    torch.manual_seed(0)
    cell = sparc_b200.SPARCRTRLCell(W, M).to(device)
    gen = torch.Generator(device=device).manual_seed(1000 + rank)
    xs = torch.randn(8, B, W, generator=gen, device=device)
    w = torch.randn(B, 2 * M, generator=gen, device=device)
    carry = cell.initial_carry(B)
    state = {"carry": carry, "i": 0}

    def step():
        cell.zero_grad(set_to_none=True)
        nxt, out = cell(state["carry"], xs[state["i"] % 8])
        (out * w).sum().backward()
        state["carry"] = nxt
        state["i"] += 1

    for _ in range(max(3, args.warmup)):
        step()
    with ClockSampler(local) as clocks:
        total_ms, per = _time_steps(step, args.steps, lambda: None, world, device)
    ms = total_ms / args.steps
    L = _lib.lib()
    L.sparc_timing_enable(1)
    _lib.kernel_times(reset_only=True)
    for _ in range(args.steps):
        step()
    torch.cuda.synchronize(device)
    times = _lib.kernel_times()
    L.sparc_timing_enable(0)
    kern = {k: round(t / n, 4) for k, (t, n) in times.items()}
    peak, kind = measured_peaks()
    # step kernel: four [B, W(+1), M] complex traces read and written (64 bytes per (b, j, m)),
    # five modal traces; gradient kernel: the nine new traces read once (32 bytes per (b, j, m))
    step_bytes = 64 * B * W * M + 32 * B * M + 80 * B * M
    grad_bytes = 32 * B * W * M + 40 * B * M
    st_ms = kern.get("rtrl_step_kernel")
    gr_ms = kern.get("rtrl_grad_kernel")
    roofline = {"bound": "hbm", "achieved": round(step_bytes / (st_ms / 1e3) / 1e9, 1), "peak": peak,
                "unit": "GB/s", "frac": round(step_bytes / (st_ms / 1e3) / 1e9 / peak, 4), "traffic": None,
                "kernel": "rtrl_step_kernel", "peak_source": kind, "kernels_ms": kern,
                "grad_kernel_GBps": round(grad_bytes / (gr_ms / 1e3) / 1e9, 1) if gr_ms else None}
    return dict(value=B * world / (ms / 1e3), ms=ms, roofline=roofline, e2e=None, cpu=None,
                clocks=clocks.summary(), launches=2 * args.steps, per_step_ms=per, tokens_step=B * world)


# ----------------------------------------------------------------------------- reference arm
_PER_GPU_BATCH = ("layer", "layer5", "real", "decode", "projection", "projection16", "rtrl", "complex")


def workload_config(workload: str, wl: dict, world: int) -> dict:
    """The workload part of the JSON line's `config`, the same for both arms: the batch is the
    job's global batch (per-GPU batch x ranks for the data-parallel workloads)."""
    cfg = {"workload": wl["workload"], "baseline_config": wl["config_index"]}
    for k in ("batch", "seq_len", "width", "modes", "channels", "layers", "steps"):
        if k in wl:
            cfg["global_batch" if k == "batch" else k] = wl[k] * (world if k == "batch" and workload in _PER_GPU_BATCH else 1)
    return cfg


def line_config(args, wl: dict, world: int) -> dict:
    """The JSON line's `config`, identical for both arms (the reference arm processes the same
    global batch; how it runs is in its cpu_baseline block): the workload, its data-parallel
    layout, how L2 is kept out of the timing and how steps are timed on the GPU arm."""
    cfg = workload_config(args.workload, wl, world)
    cfg["parallelism"] = f"dp{world}" if world > 1 else "single"
    if world > 1:
        cfg["gradient_exchange"] = {
            "fused": "in the gradient reduction kernel over NVLink peer memory (CUDA IPC)",
            "peer": "peer-memory all-reduce kernel (NVLink, CUDA IPC)",
            "nccl": "NCCL all-reduce of the packed gradients"}[
                args.allreduce if args.allreduce != "fused" or args.workload in ("layer", "layer5", "stack") else "peer"]
    cfg["l2"] = ("flushed before every step (512 MiB write, outside the CUDA events)"
                 if args.workload in ("layer", "projection") else "inputs larger than L2")
    cfg["timing"] = ("per-step CUDA events, CUDA-graph replay"
                     if args.workload in ("layer", "layer5", "decode", "projection", "projection16")
                     else "per-step CUDA events")
    return cfg


def run_reference(args, wl, world=1):
    """The reference algorithm on the host cores: the float64 oracle restatement, one batch row
    per process over all host cores; each step is one round over the job's global batch
    (per-GPU batch x ranks, the rows the GPU arm processes in one step)."""
    workers = os.cpu_count() or 1
    B, T, W = wl["batch"] * world, wl["seq_len"], wl["width"]
    pool = OraclePool(B, T, W, min(workers, B))
    times = []
    for i in range(args.warmup + args.steps):
        sec, toks = pool.round()
        if i >= args.warmup:
            times.append(sec)
    pool.close()
    ms = sum(times) / len(times) * 1e3
    return toks / (ms / 1e3), ms, toks, len(pool.rows)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="layer")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--allreduce", choices=["fused", "peer", "nccl"], default="fused",
                    help="N > 1: gradient exchange fused into the gradient reduction kernel, by the "
                         "peer-memory all-reduce kernel, or by NCCL")
    ap.add_argument("--batch", type=int, default=None, help="override the per-GPU batch (profiling runs)")
    ap.add_argument("--seq-len", type=int, default=None, help="override the sequence length (profiling runs)")
    ap.add_argument("--channels", type=int, default=None,
                    help="real workload: override D (config 3 is quoted at D=16384 and D=1024)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    wl = dict(WORKLOADS[args.workload])
    if args.batch is not None:
        wl["batch"] = args.batch
    if args.seq_len is not None:
        wl["seq_len"] = args.seq_len
    if args.channels is not None:
        if "channels" not in wl:
            ap.error("--channels applies to the real workload")
        wl["channels"] = args.channels
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        if args.workload != "layer":
            print(json.dumps({"impl": "reference", "unavailable": "reference arm covers the layer workload"}))
            return
        value, ms, toks, cores = run_reference(args, wl, world)
        line = {"metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
                "data": "synthetic", "impl": "reference",
                "config": line_config(args, wl, world),
                "cpu_baseline": {"value": round(value, 1), "unit": "tokens/s", "cores": cores, "kind": "port",
                                 "sample": f"{toks} tokens per step: {wl['batch'] * world} batch rows of "
                                           f"T={wl['seq_len']}, W={wl['width']} (the job's global batch), float64 "
                                           f"numpy oracle fwd+bwd on {cores} host cores, one row per process, "
                                           f"wall clock per step"},
                "e2e": {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    world, rank, local = _dist()
    runner = {"layer": run_layer, "layer5": run_layer, "stack": run_stack, "real": run_real,
              "decode": run_decode, "projection": run_projection, "projection16": run_projection,
              "rtrl": run_rtrl, "complex": run_complex}[args.workload]
    r = runner(args, wl, world, rank, local)
    # a bounded wait of the cross-GPU gradient exchange that ran out means wrong gradient sums:
    # no number is published then (every rank learns of it through one collective)
    if world > 1:
        import torch
        import torch.distributed as dist

        bad = torch.tensor([int(any(x.timed_out() for x in _REDUCERS if hasattr(x, "timed_out")))],
                           device=torch.device("cuda", local))
        dist.all_reduce(bad, op=dist.ReduceOp.MAX)
        if int(bad.item()):
            for x in _REDUCERS:
                x.close()
            dist.barrier()
            dist.destroy_process_group()
            raise RuntimeError("a gradient exchange's bounded wait for a peer ran out: the step's gradient sums "
                               "are not valid, so no throughput is reported")
    if rank == 0:
        unit = "tokens/s"
        cfg = line_config(args, wl, world)
        if "chunk" in r:
            r["roofline"]["chunk"] = r["chunk"]
        line = {"metric": METRIC, "value": round(r["value"], 1), "unit": unit, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["ms"], 4),
                "higher_is_better": True,
                "scaling": "weak" if args.workload in _PER_GPU_BATCH else "strong", "vs_baseline": None,
                "dtype": "f32" if wl["dtype"] == "float32" else "bf16", "data": "synthetic",
                "config": cfg, "roofline": r["roofline"], "cpu_baseline": r["cpu"], "e2e": r["e2e"],
                "clocks": r["clocks"], "gpu_launches": r["launches"]}
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist

        for r in _REDUCERS:
            r.close()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
