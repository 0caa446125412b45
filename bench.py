#!/usr/bin/env python3
"""Benchmark of the layer-stack forward (BASELINE.json metric) on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c4]
                    [--impl ours|reference]

A step is one forward of the stack over one fixed global batch of the
workload. The default is c4, the largest configuration BASELINE.json runs
on one GPU (4 layers, B=64, S=2048, d=768, H=12, F=3072, causal, valid
lengths U[1, 2048]). Under torchrun the global batch (seed 0) is sharded
over the ranks -- equal row counts, cost-balanced assignment
(sharding.BatchShard), 64/32/16/8 rows at N = 1/2/4/8 -- and each rank runs
its rows on its own GPU with no collective in the forward (strong scaling);
the time is the max over ranks. A batch that does not split evenly (c1's
two rows over four GPUs) runs as replicas instead ("scaling": "weak").

Rank 0 prints one JSON line:
  value        useful TFLOP/s of the whole batch (valid tokens, valid causal
               pairs) with inputs resident in HBM: CUDA-graph replays timed
               with CUDA events, L2 flushed (256 MiB write) between steps;
  e2e          the same metric through the public API (submission's
               UserOptimizedTransformer in the serving loop): every step
               copies its rows from pinned host memory and its result back,
               inside the timed region;
  gather       (N > 1) the NCCL all-gather that assembles the whole [B,S,d]
               result on every rank, timed on its own (it is not part of a
               step: the forward needs no inter-GPU traffic);
  roofline     the dominant kernel (largest share of forward time, measured
               live with CUDA events around each launch of an eager forward),
               plus attention's own fraction;
  cpu_baseline the CPU oracle (reference layer restated in PyTorch) on a
               bounded sample, rank 0 at N=1;
  clocks       nvidia-smi samples taken during the timed region.

`--impl reference` times the reference's own CPU implementation of the path
(the oracle port; the Python reference cannot be installed on the GPU box)
on the host cores, same metric and config; only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from techjam2026_b200.configs import WORKLOADS, generate_case, make_state_dict  # noqa: E402
from techjam2026_b200.roofline import (dense_causal_flops, lengths_of,  # noqa: E402
                                       ln_bytes_per_forward, measured_peaks, profiled_traffic,
                                       useful_flops)

METRIC = "layer-stack fwd latency ms & TFLOP/s (% tcgen05 peak) at 1/2/4/8 B200 vs CPU ref"


def parse_args():
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--config", default="c4", choices=sorted(WORKLOADS))
    p.add_argument("--impl", default="ours", choices=("ours", "reference"))
    p.add_argument("--cpu-seconds", type=float, default=12.0,
                   help="budget of the CPU-baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-gather", action="store_true",
                   help="skip the timed NCCL all-gather of the outputs (N > 1)")
    p.add_argument("--batch-size", type=int, default=None,
                   help="global batch (default: the workload's); for bounded profiling")
    p.add_argument("--protocol", default="contract", choices=("contract", "organiser"),
                   help="organiser: time the public module the way the organiser's harness "
                        "does (fixed device input, per-call events, 3 rounds x 100, median)")
    p.add_argument("--seed", type=int, default=1234, help="organiser protocol seed")
    return p.parse_args()


def run_organiser_protocol(args, rank, world):
    """The organiser harness's timing, restated (torch_transformer_benchmark.py
    :477-583, defaults :617-624): the input is drawn once with seed+100000,
    the module is called `warmup` (20) times, then `rounds` (3) batches of
    `repeats` (100) calls, each call bracketed by CUDA events on the current
    stream with no cache flush and no synchronisation in between; the result
    is the median call latency. The module is the public drop-in
    (`submission.UserOptimizedTransformer`). Its accuracy trials (seeds
    seed..seed+4 against the fp32 reference layer) are the GPU test
    `test_organiser_accuracy_trials`. Each rank times its own GPU."""
    import submission
    torch.cuda.set_device(rank if world > 1 else 0)
    dev = torch.device("cuda", torch.cuda.current_device())
    w = WORKLOADS[args.config]
    cfg = w.cfg
    api = submission.UserOptimizedTransformer(cfg)
    api.load_state_dict(make_state_dict(cfg, 0), strict=True)
    api = api.to(dev).eval()
    x_cpu, mask_cpu = generate_case(cfg, args.seed + 100000, w.padding_ratio, w.input_scale)
    x, mask = x_cpu.to(dev), mask_cpu.to(dev)
    warmup, repeats, rounds = 20, 100, 3
    samples = []
    with torch.inference_mode():
        for _ in range(warmup):
            api(x, mask)
        torch.cuda.synchronize(dev)
        for _ in range(rounds):
            starts = [torch.cuda.Event(enable_timing=True) for _ in range(repeats)]
            ends = [torch.cuda.Event(enable_timing=True) for _ in range(repeats)]
            torch.cuda.synchronize(dev)
            for i in range(repeats):
                starts[i].record()
                api(x, mask)
                ends[i].record()
            torch.cuda.synchronize(dev)
            samples.extend(a.elapsed_time(b) for a, b in zip(starts, ends))
    assert api._impl is not None, "public API fell back: nothing of ours was timed"
    med = statistics.median(samples)
    flops = useful_flops(cfg, lengths_of(mask_cpu, cfg.batch_size, cfg.seq_len))
    line = {"metric": METRIC, "protocol": "organiser", "value": round(flops / (med / 1e3) / 1e12, 3),
            "unit": "TFLOP/s", "median_ms": round(med, 4),
            "min_ms": round(min(samples), 4), "samples": len(samples),
            "tokens_per_s": round(cfg.batch_size * cfg.seq_len * 1000.0 / med, 1),
            "n_gpus": world, "dtype": "f32", "data": "synthetic",
            "config": {"workload": args.config, "signature": sig(cfg), "seed": args.seed + 100000,
                       "warmup": warmup, "repeats": repeats, "rounds": rounds}}
    if rank == 0:
        print(json.dumps(line))
    return 0


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


# ----------------------------------------------------------------- CPU legs

def cpu_sample(w, seconds: float, seed: int = 0):
    """Time the CPU oracle on single sequences of the workload until `seconds`
    elapse (at least one). Returns (useful TFLOP/s, sample description, threads)."""
    import oracle
    threads = max(1, os.cpu_count() or 1)
    torch.set_num_threads(threads)
    cfg = w.cfg
    sd = make_state_dict(cfg, 0)
    x, mask = generate_case(cfg, seed, w.padding_ratio, w.input_scale)
    qc = 1024 if cfg.seq_len > 4096 else None
    one = lambda b: oracle.forward(sd, cfg.num_layers, cfg.num_heads, x[b:b + 1],  # noqa: E731
                                   mask[b:b + 1], causal=cfg.causal, query_chunk=qc)
    if cfg.seq_len > 8192:
        # c5-sized sequences: one prefix of 8192 tokens is the bounded unit.
        P = 8192
        one = lambda b: oracle.forward(sd, cfg.num_layers, cfg.num_heads,  # noqa: E731
                                       x[b:b + 1, :P], mask[b:b + 1, :P], causal=cfg.causal,
                                       query_chunk=1024)
    one(0)  # warm-up
    flops, t_total, n, b = 0.0, 0.0, 0, 0
    t_end = time.perf_counter() + seconds
    while n == 0 or time.perf_counter() < t_end:
        t0 = time.perf_counter_ns()
        one(b)
        t_total += (time.perf_counter_ns() - t0) / 1e9
        L = mask[b]
        if cfg.seq_len > 8192:
            L = L[:8192]
        flops += useful_flops(cfg, [int(L.sum())])
        n += 1
        b = (b + 1) % cfg.batch_size
    desc = (f"oracle fp32 on {n} single sequence(s) of {w.name} "
            f"({'prefix 8192 of ' if cfg.seq_len > 8192 else ''}S={cfg.seq_len}), "
            f"{t_total:.1f} s, torch threads={threads}")
    return flops / t_total / 1e12, desc, threads, t_total / n * 1e3


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    w = WORKLOADS[args.config]
    for _ in range(max(0, args.warmup)):
        pass  # the sample itself includes a warm-up forward
    per_step = max(2.0, min(20.0, 120.0 / max(1, args.steps)))
    vals, descs = [], []
    threads = 1
    for _ in range(args.steps):
        v, desc, threads, ms = cpu_sample(w, per_step, seed=0)
        vals.append(v)
        descs.append(desc)
    value = statistics.median(vals)
    line = {
        "metric": METRIC, "value": round(value, 6), "unit": "TFLOP/s", "impl": "reference",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded generate_random_case draws, Xavier weights)",
        "config": {"workload": w.name, "signature": sig(w.cfg),
                   "global_batch": w.cfg.batch_size, "seq_len": w.cfg.seq_len,
                   "parallelism": "one CPU process (host cores); GPUs unused"},
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": threads,
                         "kind": "port", "sample": descs[-1], "cpu_model": cpu_model()},
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def sig(cfg):
    from techjam2026_b200.configs import signature
    return signature(cfg)


# ----------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi samples every 10 ms; summary() keeps those stamped inside the
    timed window (mark_start/mark_end), falling back to the nearest ones when
    the window is shorter than the sampling period."""
    FIELDS = ("timestamp,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,"
              "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    @staticmethod
    def _bus(s: str) -> str:
        # "00000000:1B:00.0" (nvidia-smi) and "0000:1b:00.0" (torch) -> "1b:00.0"
        return s.strip().lower().split(":", 1)[-1]

    def __init__(self, gpu_index: int):
        # nvidia-smi numbers GPUs physically; match this process's GPU by its
        # PCI bus id, whatever CUDA_VISIBLE_DEVICES remaps.
        try:
            self.bus = self._bus(torch.cuda.get_device_properties(gpu_index).pci_bus_id)
        except Exception:
            self.bus = None
        self.proc = None
        self.path = None
        self.t0 = self.t1 = None

    def mark_start(self):
        self.t0 = datetime.datetime.now()

    def mark_end(self):
        self.t1 = datetime.datetime.now()

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="kf_clocks_", suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "10"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 10:
                    continue
                if self.bus and self._bus(parts[1]) != self.bus:
                    continue
                try:
                    ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f")
                except ValueError:
                    ts = None
                try:
                    rows.append((ts, float(parts[2]), float(parts[3]),
                                 [n for n, v in zip(names, parts[6:10]) if v.lower() == "active"]))
                except ValueError:
                    continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        stamped = [r for r in rows if r[0] is not None]
        inside = [r for r in stamped if self.t0 and self.t1 and self.t0 <= r[0] <= self.t1]
        window = "inside the timed region"
        if not inside and self.t0 and stamped:
            after = [r for r in stamped if r[0] >= self.t0][:2]
            before = [r for r in stamped if r[0] < self.t0][-1:]
            inside, window = before + after, "nearest to the timed region (shorter than 10 ms)"
        if not inside:
            inside, window = rows, "whole sampling period"
        return {"sm_mhz": statistics.median(r[1] for r in inside),
                "sm_max_mhz": max(r[2] for r in inside), "samples": len(inside),
                "window": window, "reasons": sorted({n for r in inside for n in r[3]})}


# ----------------------------------------------------------------- GPU legs

class LaunchTimer:
    """Brackets each C-ABI launch of an eager forward with CUDA events."""

    def __init__(self):
        self.records = []

    def __call__(self, kind: str):
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        self.records.append((kind, start, end))
        return start, end


def kernel_breakdown(model, x, keep, ws, weights, repeats: int = 5):
    """Per-kind average launch time (ms) from events around every launch.

    A 10 ms device spin is queued first, so the host has enqueued the whole
    instrumented forward before the GPU reaches it: events then bracket
    device execution, not host launch gaps."""
    out = torch.empty_like(x)
    totals, counts = {}, {}
    for _ in range(repeats):
        timer = LaunchTimer()
        torch.cuda._sleep(20_000_000)
        model.launch(x, keep, out, ws, weights, timer=timer)
        torch.cuda.synchronize()
        for kind, s, e in timer.records:
            totals[kind] = totals.get(kind, 0.0) + s.elapsed_time(e)
            counts[kind] = counts.get(kind, 0) + 1
    return {k: (totals[k] / counts[k], counts[k] // repeats) for k in totals}


def kernel_work(kind: str, cfg, B: int, S: int, lengths) -> tuple:
    """Algorithmic work of ONE launch of `kind`: (amount, unit, bound).

    GEMMs count the valid tokens T only (2*T*N*K): padded rows are not
    algorithmic work, so skipping them cannot raise the fraction. Attention
    counts valid causal pairs; the norm counts the bytes of valid rows
    (roofline.ln_bytes_per_forward, averaged over its 2L+1 launches)."""
    d, F, H = cfg.d_model, cfg.ffn_dim, cfg.num_heads
    M = B * S
    T = float(sum(lengths))
    if kind == "qkv":
        return 2.0 * T * 3 * d * d, "flop", "tensor"
    if kind == "out_proj":
        return 2.0 * T * d * d, "flop", "tensor"
    if kind == "ffn1":
        return 2.0 * T * F * d, "flop", "tensor"
    if kind == "ffn2":
        return 2.0 * T * d * F, "flop", "tensor"
    if kind == "attention":
        pairs = sum(n * (n + 1) // 2 for n in lengths) if cfg.causal else sum(n * n for n in lengths)
        return 4.0 * d * pairs, "flop", "tensor"
    if kind == "ln":
        # average over the forward's 2L+1 norm launches, valid rows only
        return ln_bytes_per_forward(cfg, lengths) / (2 * cfg.num_layers + 1), "byte", "hbm"
    if kind == "keep_bits":
        return float(M + 4 * B * ((S + 31) // 32)), "byte", "hbm"
    return 0.0, "flop", "tensor"


def _timed_gather(shard, out_local, dev, world, repeats: int = 5) -> dict:
    """The optional NCCL all-gather of every rank's output rows into one
    [B, S, d] tensor in batch order (sharding.BatchShard.gather), timed on
    its own with CUDA events (median of `repeats`, max over ranks), and
    checked: this rank's rows of the gathered tensor equal its own output
    bit for bit on every rank."""
    import torch.distributed as dist
    for _ in range(2):
        shard.gather(out_local)
    torch.cuda.synchronize()
    ts = []
    for _ in range(repeats):
        dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        full = shard.gather(out_local)
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    ok = torch.tensor([1 if torch.equal(shard.take(full), out_local) else 0],
                      dtype=torch.int32, device=dev)
    t = torch.tensor([statistics.median(ts)], dtype=torch.float64, device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    nbytes = full.numel() * full.element_size()
    ms = float(t.item())
    return {"ms": round(ms, 4), "bytes": int(nbytes),
            "algbw_gbs": round(nbytes / (ms / 1e3) / 1e9, 1),
            "collective": "all_gather_into_tensor (NCCL) + un-permute to batch order",
            "rows_match": bool(ok.item())}


def main():
    args = parse_args()
    rank, world, local = dist_env()
    if world != args.gpus:
        args.gpus = world if world > 1 else args.gpus
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.protocol == "organiser":
        return run_organiser_protocol(args, rank, world)

    import dataclasses

    import torch.distributed as dist
    from techjam2026_b200 import _lib
    from techjam2026_b200.dispatch import DispatchTable, probe
    from techjam2026_b200.fused import FusedTransformer
    from techjam2026_b200.sharding import BatchShard

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    # Several ranks on one host: each stays on its GPU's NUMA node. (One rank
    # keeps every core: the CPU baseline runs there.)
    host_binding = bind_host_to_gpu(local) if world > 1 else {"bound": False,
                                                              "why": "one rank"}
    if world > 1:
        dist.init_process_group("nccl", device_id=dev,
                                timeout=datetime.timedelta(seconds=120))

    w = WORKLOADS[args.config]
    if args.batch_size:
        w = dataclasses.replace(w, cfg=dataclasses.replace(w.cfg, batch_size=args.batch_size))
    cfg_g = w.cfg
    B_g, S = cfg_g.batch_size, cfg_g.seq_len
    # One global batch (the workload's first seed), drawn identically on every
    # rank; each rank keeps its share of the rows.
    x_all, mask_all = generate_case(cfg_g, w.seeds[0], w.padding_ratio, w.input_scale)
    lengths_all = lengths_of(mask_all, B_g, S)
    strong = B_g % world == 0
    if strong:
        shard = BatchShard(lengths_all, world, rank, cfg_g.d_model, cfg_g.ffn_dim, cfg_g.causal)
        x_cpu, mask_cpu = shard.take(x_all), shard.take(mask_all)
        lengths = shard.local_lengths()
    else:
        # Replicas: a batch that does not split over the ranks runs whole on each.
        shard = None
        x_cpu, mask_cpu, lengths = x_all, mask_all, lengths_all
    del x_all
    cfg = dataclasses.replace(cfg_g, batch_size=x_cpu.shape[0])
    spec = probe(local)
    plan, source = DispatchTable.load_for(spec).lookup(spec.arch, torch.float32, cfg)
    model = FusedTransformer(cfg, plan)
    model.load_state_dict(make_state_dict(cfg, 0), strict=True)
    model.eval()

    flops_rank = useful_flops(cfg, lengths)
    x = x_cpu.to(dev)
    mask = mask_cpu.to(dev)

    runner = model.graph_runner(x, mask)
    runner.load_inputs(x, mask)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    for _ in range(max(3, args.warmup)):
        runner.replay()
    torch.cuda.synchronize()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        time.sleep(0.3)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        clocks.mark_start()
        for k in range(args.steps):
            flush.zero_()                       # evict L2 between steps (untimed)
            starts[k].record()
            runner.replay()
            ends[k].record()
        torch.cuda.synchronize()
        clocks.mark_end()
        if world > 1:
            dist.barrier()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    ms_total = sum(step_ms)
    t = torch.tensor([ms_total], dtype=torch.float64, device=dev)
    f = torch.tensor([flops_rank], dtype=torch.float64, device=dev)
    per_rank = [ms_total]
    if world > 1:
        every = torch.empty(world, dtype=torch.float64, device=dev)
        dist.all_gather_into_tensor(every, t)
        per_rank = [float(v) for v in every.tolist()]
        dist.all_reduce(f, op=dist.ReduceOp.SUM)
    ms_total_max = max(per_rank)
    flops_all = float(f.item())
    ms_per_step = ms_total_max / args.steps
    value = flops_all / (ms_per_step / 1e3) / 1e12
    status = _lib.lib().kf_device_status(local)

    # ---- the optional all-gather of the outputs (N > 1), timed on its own
    gather = None
    if world > 1 and strong and not args.no_gather:
        gather = _timed_gather(shard, runner.static_out, dev, world)

    # ---- e2e through the public API (pinned host buffers, copies timed)
    e2e = None
    if not args.no_e2e:
        import submission
        api = submission.UserOptimizedTransformer(cfg)
        api.load_state_dict(model.state_dict(), strict=True)
        api = api.to(dev).eval()
        xh = x_cpu.pin_memory()
        mh = mask_cpu.pin_memory()
        oh = torch.empty_like(x_cpu).pin_memory()
        with torch.inference_mode():
            for _ in range(max(3, args.warmup)):
                oh.copy_(api(xh.to(dev, non_blocking=True), mh.to(dev, non_blocking=True)),
                         non_blocking=True)
            torch.cuda.synchronize()
            e_s = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
            e_e = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
            if world > 1:
                dist.barrier()
            for k in range(args.steps):
                flush.zero_()
                e_s[k].record()
                xd = xh.to(dev, non_blocking=True)
                md = mh.to(dev, non_blocking=True)
                oh.copy_(api(xd, md), non_blocking=True)
                e_e[k].record()
            torch.cuda.synchronize()
        assert api._impl is not None, "public API fell back: e2e would not measure the GPU path"
        e_ms = torch.tensor([sum(s.elapsed_time(e) for s, e in zip(e_s, e_e))],
                            dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
        serial_step = float(e_ms.item()) / args.steps
        # The serving loop (techjam2026_b200.serving.StreamedForward): the
        # upload of step k+1 and the download of result k-1 overlap forward
        # k; every step still copies its inputs from pinned host memory and
        # its result back. L2 flushed before every forward, as above.
        from techjam2026_b200.serving import StreamedForward
        pipe = StreamedForward(api._impl, xh.to(dev), mh.to(dev))
        xs, ms = [xh] * args.steps, [mh] * args.steps
        outs = [oh, torch.empty_like(oh).pin_memory()] * ((args.steps + 1) // 2)
        outs = outs[:args.steps]
        with torch.inference_mode():
            pipe.run(xs[:min(args.steps, 3)], ms[:min(args.steps, 3)], outs[:min(args.steps, 3)])
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            p0 = torch.cuda.Event(enable_timing=True)
            p1 = torch.cuda.Event(enable_timing=True)
            p0.record()
            pipe.run(xs, ms, outs, before_step=lambda k: flush.zero_())
            p1.record()
            torch.cuda.synchronize()
        p_ms = torch.tensor([p0.elapsed_time(p1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(p_ms, op=dist.ReduceOp.MAX)
        e_step = float(p_ms.item()) / args.steps
        # The L2 flush before each forward sits inside this timed region (it
        # is queued on the compute stream between the steps): its own time,
        # so the loop's overhead over the forward can be read off.
        f_ts = []
        for _ in range(5):
            f0 = torch.cuda.Event(enable_timing=True)
            f1 = torch.cuda.Event(enable_timing=True)
            f0.record()
            flush.zero_()
            f1.record()
            torch.cuda.synchronize()
            f_ts.append(f0.elapsed_time(f1))
        # Bytes the loop moved per step: each row's valid prefix (prefix masks)
        # plus the mask; whole tensors otherwise.
        h2d = int(pipe.last_h2d_bytes)
        d2h = int(pipe.last_d2h_bytes)
        e2e = {"value": round(flops_all / (e_step / 1e3) / 1e12, 3), "unit": "TFLOP/s",
               "ms_per_step": round(e_step, 4),
               "l2_flush_ms_per_step_inside": round(statistics.median(f_ts), 4),
               "h2d_bytes_per_step": h2d * world,
               "d2h_bytes_per_step": d2h * world,
               "h2d_bytes_per_rank": h2d, "d2h_bytes_per_rank": d2h,
               "h2d_d2h_gbs_per_rank": round((h2d + d2h) / (e_step / 1e3) / 1e9, 2),
               "loop": ("StreamedForward: copies on two streams overlap the forward; "
                        + ("valid row prefixes only" if pipe.packed else "whole tensors")),
               "serial_ms_per_step": round(serial_step, 4),
               "serial_value": round(flops_all / (serial_step / 1e3) / 1e12, 3)}

    # ---- live per-kernel breakdown (eager forward, events around each launch)
    ws = runner.ws
    bd = kernel_breakdown(model, runner.static_x, runner.static_keep, ws, runner.weights)
    shares = {k: ms * n for k, (ms, n) in bd.items()}
    total = sum(shares.values())
    dom = max(shares, key=shares.get)
    peaks = measured_peaks()
    # A step of 100 ms or more keeps a 1 kW B200 at its power cap for most of
    # the step, so its tensor kernels are held to the sustained GEMM rate
    # (the seconds-long cuBLAS loop); shorter steps to the burst rate.
    long_step = ms_per_step >= 100.0

    def kernel_roof(kind):
        amount, unit, bound = kernel_work(kind, cfg, cfg.batch_size, cfg.seq_len, lengths)
        k_ms = bd[kind][0]
        if bound == "tensor":
            achieved = amount / (k_ms / 1e3) / 1e12
            peak = peaks["tf32_tflops_sustained" if long_step else "tf32_tflops"]
            return bound, achieved, peak, "TFLOP/s", k_ms
        return bound, amount / (k_ms / 1e3) / 1e9, peaks["hbm_gbs"], "GB/s", k_ms

    bound, achieved, peak, r_unit, dom_ms = kernel_roof(dom)
    # DRAM bytes of one launch of the dominant kernel, from the committed ncu
    # capture of this workload under the same plan (null otherwise).
    prof = profiled_traffic(w.name, cfg.batch_size, dom, plan.describe())
    roofline = {"kernel": dom, "bound": bound, "achieved": round(achieved, 2),
                "peak": round(peak, 1), "unit": r_unit, "frac": round(achieved / peak, 4),
                "traffic": prof["bytes"] if prof and prof["plan_match"] else None,
                "traffic_source": (f"{prof['source']} (ncu dram__bytes_read.sum + "
                                   "dram__bytes_write.sum, one launch)"
                                   + ("" if prof["plan_match"] else
                                      ": captured under another plan, not used"))
                if prof else "no committed capture of this workload and kernel",
                "algorithmic": kernel_work(dom, cfg, cfg.batch_size, cfg.seq_len, lengths)[0],
                "peak_source": (f"{peaks['source']} "
                                f"{'sustained' if long_step else 'burst'} "
                                f"(TF32 = measured dense BF16 / 2; step {ms_per_step:.1f} ms)")
                if bound == "tensor" else peaks["source"],
                "frac_of_burst": round(achieved / peaks["tf32_tflops"], 4)
                if bound == "tensor" else None,
                "launch_ms": round(dom_ms, 5),
                "share": {k: round(v / total, 4) for k, v in sorted(shares.items())}}
    # Per-kernel fractions: attention against the burst TF32 rate, the GEMMs
    # against the TF32-equivalent rate, the norm against HBM.
    kernels = {}
    for kind in sorted(bd):
        if kind == "keep_bits":
            continue
        kb_, ka, kp, ku, kms = kernel_roof(kind)
        kernels[kind] = {"launch_ms": round(kms, 5), "achieved": round(ka, 2), "unit": ku,
                         "frac": round(ka / kp, 4),
                         "frac_of_burst": round(ka / peaks["tf32_tflops"], 4)
                         if kb_ == "tensor" else None,
                         "launches_per_step": bd[kind][1]}
    roofline["kernels"] = kernels
    if "attention" in kernels:
        roofline["attention"] = dict(kernels["attention"], peak=round(peaks["tf32_tflops"], 1),
                                     peak_source=f"{peaks['source']} burst (TF32 = dense BF16 / 2)")

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            v, desc, threads, ms = cpu_sample(w, args.cpu_seconds)
            cpu = {"value": round(v, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                   "sample": desc, "ms_per_sequence": round(ms, 2), "cpu_model": cpu_model()}
        clk = clocks.summary()
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "strong" if strong else "weak",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded generate_random_case draws, Xavier weights)",
            "config": {"workload": w.name, "signature": sig(cfg_g),
                       "global_batch": B_g if strong else B_g * world, "seq_len": S,
                       "rows_per_rank": cfg.batch_size,
                       "parallelism": (f"batch sharded over {world} rank(s): equal row counts, "
                                       "cost-balanced assignment, no collective in the forward"
                                       if strong else f"{world} replicas of the whole batch"),
                       "modeled_imbalance": round(shard.imbalance, 4) if shard else None,
                       "per_rank_ms_per_step": [round(v / args.steps, 4) for v in per_rank],
                       "plan": plan.describe(), "plan_source": source,
                       "l2": "flushed between steps (256 MiB write)",
                       "valid_tokens": int(sum(lengths_all)),
                       "valid_tokens_rank0": int(sum(lengths)),
                       "dense_causal_tflop": round(dense_causal_flops(cfg_g) / 1e12, 4),
                       "useful_tflop": round(flops_all / 1e12, 4)},
            "tc_frac_of_tf32_peak": round(value / world / peaks["tf32_tflops"], 4),
            "gpu_launches": int(runner.launches * args.steps),
            "e2e": e2e, "gather": gather, "host_binding": host_binding,
            "roofline": roofline, "cpu_baseline": cpu,
            "clocks": clk, "device_status": status,
        }
        print(json.dumps(line), flush=True)
    runner = None
    model.release_buffers()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def bind_host_to_gpu(device_index: int) -> dict:
    """Pin this process to the CPU cores NVML reports as nearest to the GPU
    (its NUMA node), so the pinned host buffers of the e2e leg live on, and
    are copied from, that node when several ranks share the host. Only NVML
    queries are made and only this process's CPU affinity changes."""
    try:
        import pynvml
        import torch
        pynvml.nvmlInit()
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            try:
                h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-")
                                                     else "GPU-" + uuid)
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            n = os.cpu_count() or 1
            words = pynvml.nvmlDeviceGetCpuAffinity(h, (n + 63) // 64)
            try:
                node = int(pynvml.nvmlDeviceGetNumaNodeId(h))
            except Exception:
                node = None
        finally:
            pynvml.nvmlShutdown()
    except Exception as e:  # no NVML: leave the affinity alone
        return {"bound": False, "why": f"NVML: {e}"[:100]}
    near = {64 * i + b for i, w in enumerate(words) for b in range(64) if (int(w) >> b) & 1}
    cores = near & set(os.sched_getaffinity(0))
    if not cores:
        return {"bound": False, "why": "no allowed core near the GPU"}
    os.sched_setaffinity(0, cores)
    return {"bound": True, "cores": len(cores), "numa_node": node}


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo", encoding="utf-8") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


if __name__ == "__main__":
    sys.exit(main())
