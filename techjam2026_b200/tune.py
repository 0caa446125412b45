"""Populate the sm_100 dispatch table by measurement (gate, then time).

    python -m techjam2026_b200.tune --config c4 [--shards 8] [--write]

For one BASELINE configuration -- or, with --shards N, the share of its
batch that one rank runs when the batch is split over N GPUs
(sharding.BatchShard, rank 0) -- on the current GPU:

1. Build the forward with the table's current plan for that shape and keep
   its output on a seeded input as the reference.
2. For each GEMM of the layer (qkv, out, ffn1, ffn2) and each N tile the
   kernels offer (one CTA, or a CTA pair for bf16x3 at 128/256), build the
   forward with only that choice changed. The gate: its output must be
   bit-identical to the reference (a tile only decides which CTA computes an
   output element, never the order of its accumulation), so a candidate
   that changes any bit is rejected as a bug. The attention kernel (one CTA
   per query tile, or the persistent kernel over a work list) is a candidate
   of the same kind: the forward's output is bit-identical either way.
3. Time every surviving candidate as a CUDA-graph replay (median of
   `--repeats`, L2 flushed before each), keep the fastest tile per GEMM, and
   confirm the combined plan against the reference and the current plan.
4. With --write, store the combined plan as the exact entry for the shape
   when it is faster than the current one.

This is the sm_100 counterpart of the reference's plan search and
`verify --demote` (kernelforge/search.py:131-351, cli.py:149-260), limited
to the choices that cannot change numerics.
"""
from __future__ import annotations

import argparse
import dataclasses
import gc
import json
import statistics
import sys
from typing import Dict, List, Tuple

import torch

from .configs import WORKLOADS, generate_case, make_state_dict, signature
from .dispatch import DispatchTable, Entry, Plan, probe
from .fused import FusedTransformer

GEMMS = ("qkv", "out", "ffn1", "ffn2")
TILES = {"bf16x3": (64, 96, 112, 128, 256), "3xtf32": (64, 128, 256), "tf32": (64, 128, 256)}
# N tile 112 needs an fp32 output (FFN1 writes bf16 planes for FFN2).
NO_112 = ("ffn1",)
# bf16x3 GEMMs also run as 256 x bn tiles on CTA pairs for these N tiles.
PAIR_TILES = (128, 256)


def candidates(prec: str, gemm: str = "") -> List[Tuple[int, bool]]:
    """(N tile, CTA pair) choices of one GEMM; none of them changes a bit."""
    out = [(bn, False) for bn in TILES[prec] if not (bn == 112 and gemm in NO_112)]
    if prec == "bf16x3":
        out += [(bn, True) for bn in PAIR_TILES]
    return out


def _forward(cfg, sd, plan: Plan, x, mask) -> Tuple[FusedTransformer, torch.Tensor]:
    m = FusedTransformer(cfg, plan)
    m.load_state_dict(sd, strict=True)
    m = m.to(x.device).eval()
    runner = m.graph_runner(x, mask)
    runner.load_inputs(x, mask)
    runner.replay()
    torch.cuda.synchronize()
    return m, runner.static_out.clone()


def _time(model: FusedTransformer, x, mask, repeats: int, flush: torch.Tensor) -> float:
    runner = model.graph_runner(x, mask)
    runner.load_inputs(x, mask)
    for _ in range(3):
        runner.replay()
    times = []
    for _ in range(repeats):
        flush.zero_()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        runner.replay()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    return statistics.median(times)


def tune(name: str, repeats: int = 10, seed: int = 0, log=print, shards: int = 1) -> Dict:
    w = WORKLOADS[name]
    cfg = w.cfg
    x_cpu, m_cpu = generate_case(cfg, seed, w.padding_ratio, w.input_scale)
    if shards > 1:
        from .sharding import BatchShard
        shard = BatchShard(m_cpu.sum(1).tolist(), shards, 0, cfg.d_model, cfg.ffn_dim,
                           cfg.causal)
        x_cpu, m_cpu = shard.take(x_cpu), shard.take(m_cpu)
        cfg = dataclasses.replace(cfg, batch_size=shard.local_batch)
    spec = probe()
    table = DispatchTable.load_for(spec)
    base, source = table.lookup(spec.arch, torch.float32, cfg)
    sd = make_state_dict(cfg, seed)
    dev = torch.device("cuda", torch.cuda.current_device())
    x, mask = x_cpu.to(dev), m_cpu.to(dev)
    flush = torch.empty(64 * 1024 * 1024, device=dev)

    model, ref = _forward(cfg, sd, base, x, mask)
    t_base = _time(model, x, mask, repeats, flush)
    model.release_buffers()
    del model
    gc.collect()
    torch.cuda.empty_cache()
    log(f"{name} {signature(cfg)}: current plan ({source}) {base.describe()}: {t_base:.3f} ms")
    best = {}
    results: List[dict] = []
    for g in GEMMS:
        field, pfield = f"bn_{g}", f"pair_{g}"
        prec = getattr(base, f"prec_{g}")
        timed = []
        for bn, pair in candidates(prec, g):
            cand = dataclasses.replace(base, **{field: bn, pfield: pair})
            model, out = _forward(cfg, sd, cand, x, mask)
            exact = torch.equal(out, ref)
            t = _time(model, x, mask, repeats, flush) if exact else float("inf")
            model.release_buffers()  # the captured graph holds its memory pool
            del model, out
            gc.collect()
            torch.cuda.empty_cache()
            results.append({"gemm": g, "bn": bn, "pair": pair, "ms": t, "bit_exact": exact})
            tag = f"bn={bn:3d}{' pair' if pair else '     '}"
            log(f"  {g:5s} {tag}: {'%.3f ms' % t if exact else 'REJECTED (output differs)'}")
            if exact:
                timed.append((t, bn, pair))
        if timed:
            _, bn_best, pair_best = min(timed)
            best[field], best[pfield] = bn_best, pair_best
        else:
            best[field], best[pfield] = getattr(base, field), getattr(base, pfield)
    # The attention kernel, with the GEMM tiles chosen above.
    timed = []
    for persistent in (False, True):
        cand = dataclasses.replace(base, **best, attn_persistent=persistent)
        model, out = _forward(cfg, sd, cand, x, mask)
        exact = torch.equal(out, ref)
        t = _time(model, x, mask, repeats, flush) if exact else float("inf")
        model.release_buffers()
        del model, out
        gc.collect()
        torch.cuda.empty_cache()
        results.append({"gemm": "attention", "persistent": persistent, "ms": t,
                        "bit_exact": exact})
        log(f"  attention {'persistent' if persistent else 'one CTA per query tile'}: "
            f"{'%.3f ms' % t if exact else 'REJECTED (output differs)'}")
        if exact:
            timed.append((t, persistent))
    best["attn_persistent"] = min(timed)[1] if timed else base.attn_persistent
    tuned = dataclasses.replace(base, **best)
    model, out = _forward(cfg, sd, tuned, x, mask)
    exact = torch.equal(out, ref)
    t_tuned = _time(model, x, mask, repeats, flush) if exact else float("inf")
    log(f"  combined {tuned.describe()}: {t_tuned:.3f} ms, bit-exact {exact}")
    label = name if shards == 1 else f"{name}, one rank's rows of {shards} (cost-balanced shard)"
    return {"config": name, "label": label, "signature": signature(cfg), "base_ms": t_base,
            "tuned_ms": t_tuned, "bit_exact": exact, "plan": tuned, "base": base,
            "candidates": results}


def write_entry(result: Dict, arch: str = "sm_100") -> str:
    table = DispatchTable.load(arch)
    sig = result["signature"]
    tuned: Plan = result["plan"]
    note = (f"tiles tuned by measurement: {result['tuned_ms']:.3f} ms "
            f"(was {result['base_ms']:.3f} ms); all candidates bit-exact")
    for e in table.entries:
        if e.signature == sig and e.dtype == "float32":
            keep = e.note.split(";")[0]
            e.plan = dataclasses.replace(tuned, name=e.plan.name)
            e.note = f"{keep}; {note}"
            break
    else:
        table.entries.append(Entry(sig, "float32", "sm_100", tuned,
                                   f"{result.get('label', result.get('config', sig))}; {note}"))
    return table.save(arch)


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--config", action="append", choices=sorted(WORKLOADS), required=True)
    p.add_argument("--repeats", type=int, default=10)
    p.add_argument("--shards", type=int, action="append", default=None,
                   help="tune the shard one rank runs when the batch is split over N GPUs")
    p.add_argument("--write", action="store_true", help="store faster plans in the table")
    args = p.parse_args(argv)
    for name in args.config:
        for shards in (args.shards or [1]):
            r = tune(name, args.repeats, shards=shards)
            # Written when faster; a shard shape's measured plan is also written
            # when it is the plan the table would give it anyway.
            same = r["plan"] == r["base"]
            if args.write and r["bit_exact"] and (r["tuned_ms"] < r["base_ms"]
                                                  or (shards > 1 and same)):
                print(f"  written to {write_entry(r)}")
            print(json.dumps({k: (dataclasses.asdict(v) if isinstance(v, Plan) else v)
                              for k, v in r.items() if k != "candidates"}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
