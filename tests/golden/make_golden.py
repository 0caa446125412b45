"""Generate the golden vectors under tests/golden/ from the REFERENCE itself.

Run in a container where the reference checkout is available:

    KF_REFERENCE_DIR=/path/to/techjam2026 python tests/golden/make_golden.py

For each case it imports the organiser's torch_transformer_benchmark.py from
the reference checkout, builds its BaselineTransformer, applies the benchmark
weight convention (Xavier-uniform weights, zero biases, LayerNorm 1/0, in
named_parameters() order from one seeded CPU generator), draws x and
valid_token_mask with the reference's own generate_random_case on the CPU,
and records the reference's fp32 CPU output. Nothing from the reference is
copied; only its outputs are stored.

Files: golden_<case>.pt = {config, seed, padding_ratio, state_dict, x, mask,
out}; golden_inputs.json = lengths and x checksums of the larger BASELINE
configs (inputs only, to pin the generator at full size).
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from techjam2026_b200.configs import WORKLOADS, init_params_  # noqa: E402

CASES = {
    # name: (B, S, d, H, F, L, causal, padding_ratio, seed)
    "c1": (2, 64, 128, 4, 512, 1, True, 0.5, 0),
    "mini_s333": (2, 333, 64, 4, 128, 2, True, 0.5, 7),
    "mini_dh8_noncausal": (3, 40, 32, 4, 64, 2, False, 0.6, 5),
    "mini_nopad": (2, 96, 64, 2, 128, 2, True, 0.0, 11),
    # a long ragged row: S = 4097 (one query row past 32 tiles of 128),
    # head_dim 8, as the chunked oracle restatement is pinned at this length
    "mini_s4097": (1, 4097, 16, 2, 32, 1, True, 0.5, 17),
    # bfloat16 I/O: the reference module cast to bf16, inputs drawn in bf16
    # (the harness's --dtype bfloat16), output in bf16.
    "mini_bf16": (2, 96, 64, 2, 128, 2, True, 0.5, 13),
}
DTYPES = {"mini_bf16": torch.bfloat16}


def x_checksum(x: torch.Tensor) -> str:
    return hashlib.sha256(x.contiguous().numpy().tobytes()).hexdigest()


def main() -> None:
    ref_dir = os.environ.get("KF_REFERENCE_DIR")
    if not ref_dir:
        raise SystemExit("set KF_REFERENCE_DIR to a checkout of the reference "
                         "(the directory holding torch_transformer_benchmark.py)")
    sys.path.insert(0, ref_dir)
    import torch_transformer_benchmark as ref

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    only = set(sys.argv[1:])  # optional case names: regenerate just those
    for name, (B, S, d, H, F, L, causal, pad, seed) in CASES.items():
        if only and name not in only:
            continue
        dtype = DTYPES.get(name, torch.float32)
        cfg = ref.TransformerConfig(B, S, d, H, F, L, causal)
        model = init_params_(ref.BaselineTransformer(cfg), seed).eval().to(dtype)
        x, mask = ref.generate_random_case(cfg, torch.device("cpu"), dtype, seed, pad, 1.0)
        with torch.inference_mode():
            out = model(x, mask)
        blob = {"config": [B, S, d, H, F, L, causal], "seed": seed, "padding_ratio": pad,
                "state_dict": {k: v.clone() for k, v in model.state_dict().items()},
                "x": x.clone(), "mask": mask.clone(), "out": out.clone()}
        if dtype != torch.float32:
            blob["dtype"] = str(dtype).replace("torch.", "")
        path = os.path.join(HERE, f"golden_{name}.pt")
        torch.save(blob, path)
        print(f"{name}: out[{tuple(out.shape)}] -> {path} ({os.path.getsize(path)} bytes)")

    if only:
        return
    inputs = {}
    for wname, w in WORKLOADS.items():
        cfg = ref.TransformerConfig(**{f: getattr(w.cfg, f) for f in (
            "batch_size", "seq_len", "d_model", "num_heads", "ffn_dim", "num_layers", "causal")})
        for seed in w.seeds:
            if wname == "c5":
                B = 2  # first two sequences only (the draw order makes them a prefix)
            else:
                B = cfg.batch_size
            small = ref.TransformerConfig(B, cfg.seq_len, cfg.d_model, cfg.num_heads,
                                          cfg.ffn_dim, cfg.num_layers, cfg.causal)
            x, mask = ref.generate_random_case(small, torch.device("cpu"), torch.float32,
                                               seed, w.padding_ratio, w.input_scale)
            inputs[f"{wname}/seed{seed}/B{B}"] = {
                "lengths": mask.sum(1).tolist(), "x_sha256": x_checksum(x)}
    with open(os.path.join(HERE, "golden_inputs.json"), "w", encoding="utf-8") as f:
        json.dump(inputs, f, indent=1, sort_keys=True)
        f.write("\n")
    print(f"inputs: {len(inputs)} entries")


if __name__ == "__main__":
    main()
