"""Roofline bookkeeping used by bench.py: FLOP counts and the traffic table."""
import torch

from techjam2026_b200.configs import WORKLOADS
from techjam2026_b200.roofline import (dense_causal_flops, lengths_of, profiled_traffic,
                                       useful_flops)


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


def test_profiled_traffic_reads_committed_capture():
    t = profiled_traffic("c2", "ffn1")
    assert t is not None and t["source"].startswith("profiles/traffic_")
    # the capture's DRAM read of one FFN1 launch: W1 planes (4.19 MB) plus live A rows
    assert 2048 * 512 * 4 < t["bytes"] < 2048 * 512 * 4 + 4096 * 512 * 4
    assert profiled_traffic("c2", "no_such_kernel") is None


def test_profiled_traffic_parses_lines(tmp_path):
    (tmp_path / "traffic_x.md").write_text("text\n```\ntraffic w k 123\ntraffic w k2 7\n```\n")
    (tmp_path / "other.md").write_text("traffic w k 999\n")
    assert profiled_traffic("w", "k", str(tmp_path))["bytes"] == 123
    assert profiled_traffic("w", "k3", str(tmp_path)) is None
