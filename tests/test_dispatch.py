"""Dispatch table: sm_100 keys, reference signature format, lookup order
exact -> nearest -> default (kernelforge/dispatch.py:254-288). CPU only."""
from __future__ import annotations

import dataclasses

import pytest
import torch

from techjam2026_b200.configs import WORKLOADS, TransformerConfig, signature
from techjam2026_b200.dispatch import (CONSERVATIVE_PLAN, DEFAULT_PLAN, DispatchTable, Entry,
                                       Plan)


def test_signature_format_matches_reference():
    cfg = TransformerConfig(8, 512, 512, 8, 2048, 6, True)
    assert signature(cfg) == "B8-S512-d512-H8-F2048-L6-causal"
    assert signature(dataclasses.replace(cfg, causal=False)) == "B8-S512-d512-H8-F2048-L6"


def test_shipped_table_covers_every_baseline_config():
    table = DispatchTable.load("sm_100")
    for w in WORKLOADS.values():
        plan, src = table.lookup("sm_100", torch.float32, w.cfg)
        assert src == "exact", w.name


def test_lookup_order():
    cfg = TransformerConfig(2, 64, 128, 4, 512, 1, True)
    special = Plan(name="special", bn_qkv=64)
    t = DispatchTable([Entry(signature(cfg), "float32", "sm_100", special)])
    assert t.lookup("sm_100a", torch.float32, cfg) == (special, "exact")
    other = TransformerConfig(2, 64, 128, 4, 512, 2, True)
    assert t.lookup("sm_100", torch.float32, other) == (CONSERVATIVE_PLAN, "nearest")
    assert DispatchTable([]).lookup("sm_100", torch.float32, other) == (DEFAULT_PLAN, "default")


def test_nearest_keeps_the_plan_of_the_same_layer_at_the_closest_batch():
    """A batch slice or one rank's shard of a configuration keeps that
    configuration's measured plan; another layer shape does not."""
    big = Plan(name="b16", bn_qkv=256, pair_qkv=True)
    small = Plan(name="b2", bn_qkv=128)
    t = DispatchTable([
        Entry(signature(TransformerConfig(16, 1024, 1024, 4, 4096, 2, True)), "float32", "sm_100", big),
        Entry(signature(TransformerConfig(2, 1024, 1024, 4, 4096, 2, True)), "float32", "sm_100", small),
    ])
    for B, want in ((8, big), (32, big), (4, small), (1, small)):
        cfg = TransformerConfig(B, 1024, 1024, 4, 4096, 2, True)
        assert t.lookup("sm_100", torch.float32, cfg) == (want, "nearest"), B
    other = TransformerConfig(8, 1024, 1024, 4, 4096, 2, False)      # not causal
    assert t.lookup("sm_100", torch.float32, other) == (CONSERVATIVE_PLAN, "nearest")
    # the shipped table: one c5 shard (2 sequences) keeps the c5 plan
    from techjam2026_b200.configs import WORKLOADS
    import dataclasses
    c5 = WORKLOADS["c5"].cfg
    shipped = DispatchTable.load()
    assert shipped.lookup("sm_100", torch.float32, dataclasses.replace(c5, batch_size=2))[0] == \
        shipped.lookup("sm_100", torch.float32, c5)[0]


def test_other_arches_and_dtypes_are_refused():
    cfg = TransformerConfig(2, 64, 128, 4, 512, 1, True)
    with pytest.raises(RuntimeError):
        DispatchTable([]).lookup("sm_90", torch.float32, cfg)
    with pytest.raises(RuntimeError):
        DispatchTable([]).lookup("sm_100", torch.float64, cfg)


def test_narrow_dtypes_get_the_exact_reference_plan():
    """fp16/bf16 I/O: only the reference's exact arithmetic passes the gate,
    so every shape maps to the exact-reference graph plan."""
    from techjam2026_b200.dispatch import EXACT_PLAN
    cfg = TransformerConfig(2, 64, 128, 4, 512, 1, True)
    for dt in (torch.float16, torch.bfloat16):
        plan, src = DispatchTable.load().lookup("sm_100", dt, cfg)
        assert plan is EXACT_PLAN and src == "exact-dtype" and plan.exact_reference
        assert plan.describe() == "exact-reference+cuda-graph"
    plan, _ = DispatchTable.load().lookup("sm_100", torch.float32, cfg)
    assert not plan.exact_reference


def test_table_round_trips(tmp_path, monkeypatch):
    import techjam2026_b200.dispatch as D
    monkeypatch.setattr(D, "TABLE_DIR", str(tmp_path))
    cfg = TransformerConfig(2, 64, 128, 4, 512, 1, True)
    t = DispatchTable([Entry(signature(cfg), "float32", "sm_100", Plan(name="x", bn_out=128))])
    t.save("sm_100")
    back = DispatchTable.load("sm_100")
    assert back.lookup("sm_100", torch.float32, cfg)[0] == Plan(name="x", bn_out=128)


def test_workspace_estimate_matches_allocation():
    """The batch-streaming budget uses _Workspace.estimate; it must equal what
    the workspace really allocates, for every precision mix."""
    import dataclasses
    from techjam2026_b200.configs import WORKLOADS
    from techjam2026_b200.fused import _Workspace
    from techjam2026_b200.dispatch import DEFAULT_PLAN
    plans = [DEFAULT_PLAN,
             dataclasses.replace(DEFAULT_PLAN, prec_qkv="tf32", prec_out="3xtf32",
                                 prec_ffn1="tf32", prec_ffn2="bf16x3")]
    for name in ("c1", "c3a", "c2"):
        cfg = WORKLOADS[name].cfg
        for plan in plans:
            B, S = 2, min(cfg.seq_len, 96)
            ws = _Workspace(cfg, B, S, torch.device("cpu"), plan)
            assert _Workspace.estimate(cfg, B, S, plan) == ws.nbytes(), (name, plan.prec_qkv)


def test_batch_streaming_slice_rows_follow_the_budget():
    from techjam2026_b200.configs import WORKLOADS
    from techjam2026_b200.fused import FusedTransformer
    cfg = WORKLOADS["c2"].cfg
    m = FusedTransformer(cfg)
    per = m.bytes_per_sequence(cfg.seq_len)
    cpu = torch.device("cpu")
    for budget, rows in ((per * 3 + per // 2, 3), (per // 2, 1), (per * 100, 8)):
        m.memory_budget_bytes = budget
        m._slice_rows.clear()
        assert m.slice_rows(8, cfg.seq_len, cpu) == rows


def test_tune_write_entry_updates_exact_signature(tmp_path, monkeypatch):
    """tune.write_entry replaces the exact entry's tiles (keeping its name and
    the first part of its note) or appends a new entry; lookup then returns
    it as "exact"."""
    import dataclasses
    import shutil
    from techjam2026_b200 import dispatch, tune
    from techjam2026_b200.configs import WORKLOADS, signature
    shutil.copy(dispatch.DispatchTable.path_for("sm_100"), tmp_path / "dispatch_sm_100.json")
    monkeypatch.setattr(dispatch, "TABLE_DIR", str(tmp_path))
    cfg = WORKLOADS["c4"].cfg
    base, _ = dispatch.DispatchTable.load().lookup("sm_100", torch.float32, cfg)
    tuned = dataclasses.replace(base, bn_ffn1=96, bn_ffn2=64)
    tune.write_entry({"signature": signature(cfg), "plan": tuned, "tuned_ms": 1.0,
                      "base_ms": 2.0})
    plan, src = dispatch.DispatchTable.load().lookup("sm_100", torch.float32, cfg)
    assert src == "exact" and plan.bn_ffn1 == 96 and plan.bn_ffn2 == 64
    assert plan.name == base.name
    odd = dataclasses.replace(cfg, batch_size=3)
    tune.write_entry({"signature": signature(odd), "plan": tuned, "tuned_ms": 1.0,
                      "base_ms": 2.0})
    plan, src = dispatch.DispatchTable.load().lookup("sm_100", torch.float32, odd)
    assert src == "exact" and plan.bn_ffn2 == 64


def test_tune_candidates_include_cta_pairs_for_bf16x3_only():
    from techjam2026_b200 import tune
    bf = tune.candidates("bf16x3")
    assert (256, True) in bf and (128, True) in bf and (96, False) in bf
    assert all(not pair for _, pair in tune.candidates("tf32"))
    assert all(bn in (128, 256) for bn, pair in bf if pair)


def test_plan_pair_fields_round_trip_and_describe():
    import dataclasses
    from techjam2026_b200.dispatch import DEFAULT_PLAN, Entry, Plan
    p = dataclasses.replace(DEFAULT_PLAN, bn_qkv=256, pair_qkv=True)
    e = Entry("sig", "float32", "sm_100", p, "note")
    assert Entry.from_json(e.to_json()).plan == p
    assert "cta-pair=y/n/n/n" in p.describe()
    # entries written before the pair fields existed still load
    d = dataclasses.asdict(DEFAULT_PLAN)
    for k in ("pair_qkv", "pair_out", "pair_ffn1", "pair_ffn2"):
        d.pop(k)
    assert Plan(**d).pair_qkv is False


def test_stream_k_workspace_keeps_partials_and_counters_apart():
    """One workspace serves stream-K GEMMs of several shapes: the largest
    partial area comes first and the largest counter area last, so no GEMM's
    partials overlap any GEMM's counters (placed at the buffer's end)."""
    import dataclasses
    from techjam2026_b200.configs import WORKLOADS
    from techjam2026_b200.dispatch import DEFAULT_PLAN
    from techjam2026_b200.fused import _Workspace
    cfg = WORKLOADS["c2"].cfg
    M = cfg.batch_size * cfg.seq_len
    plan = dataclasses.replace(DEFAULT_PLAN, bn_qkv=128, bn_out=128, bn_ffn1=128, bn_ffn2=64,
                               sk_qkv=True, sk_out=True, sk_ffn1=True, sk_ffn2=True)
    size = _Workspace.sk_bytes(cfg, M, plan)
    assert size % 4 == 0
    ends, starts = [], []
    for n, bn in ((3 * cfg.d_model, 128), (cfg.d_model, 128), (cfg.ffn_dim, 128),
                  (cfg.d_model, 64)):
        tiles = ((M + 127) // 128) * ((n + bn - 1) // bn)
        ends.append(tiles * 2 * 128 * bn * 4)
        starts.append((size - tiles * 2 * 4) & ~15)
        assert starts[-1] + tiles * 8 <= size
    assert max(ends) <= min(starts)
    assert _Workspace.sk_bytes(cfg, M, DEFAULT_PLAN) == 0
