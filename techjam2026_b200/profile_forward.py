"""Eager forwards of one workload, for running under a profiler.

    python -m techjam2026_b200.profile_forward --config c4 [--batch-size 8]
                                               [--forwards 2]

Builds the stack for a BASELINE configuration (its dispatch-table plan, the
workload's seeded batch, optionally only its first `--batch-size` rows) and
runs `--forwards` whole forwards launch by launch (no CUDA graph), so a
profiler sees every kernel as its own launch. The first forward is the
warm-up; the launch order of one forward is printed first, so a profiler's
`-s` (launches to skip) and `-c` (launches to capture) can be read off it:
the launches of forward f are [f * n, (f + 1) * n).
"""
from __future__ import annotations

import argparse
import dataclasses
import sys


def main(argv=None) -> int:
    import torch

    from .configs import WORKLOADS, generate_case, make_state_dict
    from .dispatch import DispatchTable, probe
    from .fused import FusedTransformer

    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--config", default="c4", choices=sorted(WORKLOADS))
    p.add_argument("--batch-size", type=int, default=None)
    p.add_argument("--forwards", type=int, default=2)
    args = p.parse_args(argv)
    w = WORKLOADS[args.config]
    cfg = w.cfg
    x, mask = generate_case(cfg, w.seeds[0], w.padding_ratio, w.input_scale)
    if args.batch_size:
        cfg = dataclasses.replace(cfg, batch_size=args.batch_size)
        x, mask = x[:args.batch_size].contiguous(), mask[:args.batch_size].contiguous()
    spec = probe(0)
    plan, source = DispatchTable.load_for(spec).lookup(spec.arch, torch.float32, cfg)
    model = FusedTransformer(cfg, plan)
    model.load_state_dict(make_state_dict(cfg, 0), strict=True)
    model.eval()
    xd, md = x.cuda(), mask.cuda()
    w_ = model.prepare(xd.device)
    ws = model.workspace(cfg.batch_size, cfg.seq_len, xd.device)
    out = torch.empty_like(xd)
    kinds = []
    model.launch(xd, model._keep_u8(md), out, ws, w_,
                 timer=lambda kind: (kinds.append(kind), (_NoEvent(), _NoEvent()))[1])
    torch.cuda.synchronize()
    print(f"{args.config} B={cfg.batch_size} plan ({source}): {plan.describe()}")
    print(f"{len(kinds)} launches per forward: " + " ".join(kinds))
    for _ in range(args.forwards - 1):
        model.launch(xd, model._keep_u8(md), out, ws, w_)
    torch.cuda.synchronize()
    from . import _lib
    status = _lib.lib().kf_device_status(0)
    print(f"{args.forwards} forwards done, device status {status}")
    return 0 if status == 0 else 1


class _NoEvent:
    def record(self):
        pass


if __name__ == "__main__":
    sys.exit(main())
