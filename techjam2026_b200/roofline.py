"""Work and traffic formulas used for roofline fractions.

Useful FLOPs of one forward (the figure `roofline.achieved` uses):

    sum over layers of  2*T*(4d^2 + 2dF)  +  4*d*sum_b L_b(L_b+1)/2

T = sum_b L_b valid tokens; the attention term counts only valid causal
(query, key) pairs of valid queries, 2*Dh FLOPs each for QK^T and PV over
all heads. Padded rows, skipped tiles and head-dim padding are not counted,
so skipping them raises the achieved rate and cannot push it past 100%.
The dense-causal count (all M = B*S rows, S(S+1)/2 pairs per sequence) is
the reference's roofline.stack_flops convention (kernelforge/roofline.py:
96-116, attention halved for causal).

LayerNorm traffic: 16*d bytes per row per add+mask+LN call (read x and y,
write s and h, fp32), 2L+1 calls per forward (`norm_bytes`, every row: an
upper bound); `ln_bytes_per_forward` counts what the calls must move when
padded rows are skipped (the roofline's algorithmic bytes).
"""
from __future__ import annotations

import json
import os
from typing import Iterable, List, Optional

import torch


def lengths_of(mask: Optional[torch.Tensor], B: int, S: int) -> List[int]:
    if mask is None:
        return [S] * B
    return [int(v) for v in mask.to(torch.int64).sum(dim=1).tolist()]


def gemm_flops_per_token(cfg) -> float:
    d, F = cfg.d_model, cfg.ffn_dim
    return 2.0 * (4 * d * d + 2 * d * F)


def attn_pairs(lengths: Iterable[int], causal: bool = True, S: Optional[int] = None) -> float:
    if causal:
        return float(sum(n * (n + 1) // 2 for n in lengths))
    return float(sum(n * n for n in lengths))


def useful_flops(cfg, lengths: Iterable[int]) -> float:
    lengths = list(lengths)
    T = float(sum(lengths))
    return cfg.num_layers * (T * gemm_flops_per_token(cfg)
                             + 4.0 * cfg.d_model * attn_pairs(lengths, cfg.causal))


def useful_attention_flops(cfg, lengths: Iterable[int]) -> float:
    return cfg.num_layers * 4.0 * cfg.d_model * attn_pairs(list(lengths), cfg.causal)


def dense_causal_flops(cfg) -> float:
    B, S = cfg.batch_size, cfg.seq_len
    M = B * S
    pairs = B * S * (S + 1) / 2 if cfg.causal else B * S * S
    return cfg.num_layers * (M * gemm_flops_per_token(cfg) + 4.0 * cfg.d_model * pairs)


def norm_bytes(cfg) -> float:
    M = cfg.batch_size * cfg.seq_len
    return 16.0 * cfg.d_model * M * (2 * cfg.num_layers + 1)


def ln_bytes_per_forward(cfg, lengths: Iterable[int]) -> float:
    """Algorithmic DRAM bytes of the 2L+1 add+mask+LayerNorm calls of one
    forward, the norms touching valid rows only (padded rows are skipped,
    except that the final norm writes them as zeros):
      entry norm        read x, write s and h     12*d bytes per valid row
      2L-1 middle norms read x, y, write s, h     16*d
      final norm        read x, y, write h        8*d, plus 4*d per padded row
    """
    T = float(sum(lengths))
    M = float(cfg.batch_size * cfg.seq_len)
    d, L = cfg.d_model, cfg.num_layers
    return 12.0 * d * T + (2 * L - 1) * 16.0 * d * T + 8.0 * d * T + 4.0 * d * (M - T)


def ln_call_bytes(M: int, d: int, has_y: bool = True, writes_s: bool = True) -> float:
    return 4.0 * d * M * (1 + int(has_y) + int(writes_s) + 1)


def measured_peaks(path: Optional[str] = None) -> dict:
    """MEASURED_PEAKS.json (driver-written) or the pool's stated fallback.
    TF32 tensor peak = half the measured dense BF16 GEMM rate (tcgen05 TF32
    issues at half the BF16 rate)."""
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    path = path or os.path.join(here, "MEASURED_PEAKS.json")
    out = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
           "source": "fallback"}
    try:
        with open(path, encoding="utf-8") as f:
            blob = json.load(f)
        for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained"):
            if k in blob:
                out[k] = float(blob[k])
        out["source"] = "measured"
    except Exception:
        pass
    out["tf32_tflops"] = out["bf16_tflops"] / 2.0
    out["tf32_tflops_sustained"] = out["bf16_tflops_sustained"] / 2.0
    return out


def plan_tag(plan_description: str) -> str:
    """Short stable tag of a plan (its `Plan.describe()` text)."""
    import hashlib
    return hashlib.sha1(plan_description.encode("utf-8")).hexdigest()[:12]


def profiled_traffic(workload: str, batch: int, kind: str, plan_description: str,
                     folder: Optional[str] = None) -> Optional[dict]:
    """DRAM bytes per launch of `kind` on `workload` at `batch` rows, from an
    ncu capture.

    Reads the `traffic <workload> <batch> <kind> <bytes> <plan tag>` lines of
    the committed capture summaries (profiles/traffic_*.md:
    dram__bytes_read.sum + dram__bytes_write.sum per launch, one ncu pass
    over one forward). Returns {"bytes", "source", "plan_match"} -- a capture
    taken under another plan is reported as such and must not be used -- or
    None when no capture covers the workload, batch and kernel."""
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    folder = folder or os.path.join(here, "profiles")
    try:
        names = sorted(n for n in os.listdir(folder)
                       if n.startswith("traffic_") and n.endswith(".md"))
    except OSError:
        return None
    want = plan_tag(plan_description)
    found = None
    for name in names:
        with open(os.path.join(folder, name), encoding="utf-8") as f:
            for line in f:
                parts = line.split()
                if (len(parts) == 6 and parts[0] == "traffic" and parts[1] == workload
                        and parts[2] == str(batch) and parts[3] == kind):
                    hit = {"bytes": int(parts[4]), "source": f"profiles/{name}",
                           "plan_match": parts[5] == want}
                    if hit["plan_match"]:
                        return hit
                    found = found or hit
    return found
