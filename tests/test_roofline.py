"""Roofline bookkeeping used by bench.py: FLOP counts and the traffic table."""
import torch

from techjam2026_b200.configs import WORKLOADS
from techjam2026_b200.roofline import (dense_causal_flops, lengths_of, plan_tag,
                                       profiled_traffic, useful_flops)


def test_useful_flops_counts_valid_causal_pairs():
    cfg = WORKLOADS["c1"].cfg
    full = useful_flops(cfg, [cfg.seq_len] * cfg.batch_size)
    assert abs(full - dense_causal_flops(cfg)) <= 1e-6 * full
    half = useful_flops(cfg, [cfg.seq_len // 2] * cfg.batch_size)
    assert half < full / 2


def test_lengths_of_mask():
    # True marks a valid (kept) token
    m = torch.ones(2, 8, dtype=torch.bool)
    m[0, 5:] = False
    assert lengths_of(m, 2, 8) == [5, 8]
    assert lengths_of(None, 3, 4) == [4, 4, 4]


def test_profiled_traffic_parses_lines_and_checks_the_plan(tmp_path):
    tag = plan_tag("plan A")
    (tmp_path / "traffic_x.md").write_text(
        f"text\n```\ntraffic w 8 k 123 {tag}\ntraffic w 8 k2 7 {tag}\n"
        f"traffic w 64 k 555 {tag}\ntraffic w 8 k3 9 {plan_tag('plan B')}\n```\n")
    (tmp_path / "other.md").write_text(f"traffic w 8 k 999 {tag}\n")
    hit = profiled_traffic("w", 8, "k", "plan A", str(tmp_path))
    assert hit["bytes"] == 123 and hit["plan_match"]
    assert profiled_traffic("w", 64, "k", "plan A", str(tmp_path))["bytes"] == 555
    assert profiled_traffic("w", 8, "k4", "plan A", str(tmp_path)) is None
    stale = profiled_traffic("w", 8, "k3", "plan A", str(tmp_path))
    assert stale["bytes"] == 9 and not stale["plan_match"]
    assert profiled_traffic("w", 16, "k", "plan A", str(tmp_path)) is None


def test_norm_bytes_count_valid_rows():
    from techjam2026_b200.roofline import ln_bytes_per_forward
    cfg = WORKLOADS["c2"].cfg
    d, L, M = cfg.d_model, cfg.num_layers, cfg.batch_size * cfg.seq_len
    full = ln_bytes_per_forward(cfg, [cfg.seq_len] * cfg.batch_size)
    assert full == (12 + (2 * L - 1) * 16 + 8) * d * M
    half = ln_bytes_per_forward(cfg, [cfg.seq_len // 2] * cfg.batch_size)
    assert half == (12 + (2 * L - 1) * 16 + 8) * d * M / 2 + 4 * d * M / 2


def test_committed_c4_capture_matches_the_tables_plan():
    """profiles/traffic_c4.md was captured under the plan the dispatch table
    gives c4 today, for every kernel kind of the forward; a plan change
    without a new capture fails here (bench.py would report no traffic)."""
    from techjam2026_b200.dispatch import DispatchTable
    cfg = WORKLOADS["c4"].cfg
    plan, source = DispatchTable.load("sm_100").lookup("sm_100", torch.float32, cfg)
    assert source == "exact"
    for kind in ("qkv", "attention", "out_proj", "ln", "ffn1", "ffn2"):
        hit = profiled_traffic("c4", cfg.batch_size, kind, plan.describe())
        assert hit is not None and hit["plan_match"], kind
        assert hit["source"] == "profiles/traffic_c4.md"
