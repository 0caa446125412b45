"""Batch sharding host logic, on CPU: cost-balanced equal-count assignment,
and a 2-rank gloo run whose gathered, un-permuted result equals the
single-process oracle result bit for bit. No GPU."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from techjam2026_b200.configs import WORKLOADS, generate_case
from techjam2026_b200.sharding import assign_rows, imbalance, permutation, row_cost


def test_assignment_is_equal_count_and_balanced():
    w = WORKLOADS["c4"]
    _, mask = generate_case(w.cfg, 0, w.padding_ratio)
    lengths = mask.sum(1).tolist()
    for world in (2, 4, 8):
        rows = assign_rows(lengths, world, w.cfg.d_model, w.cfg.ffn_dim)
        assert sorted(b for r in rows for b in r) == list(range(64))
        assert all(len(r) == 64 // world for r in rows)
        naive = [list(range(i * 64 // world, (i + 1) * 64 // world)) for i in range(world)]
        bal = imbalance(lengths, rows, w.cfg.d_model, w.cfg.ffn_dim)
        assert bal < 1.05, bal
        assert bal <= imbalance(lengths, naive, w.cfg.d_model, w.cfg.ffn_dim)


def test_permutation_round_trips():
    rows = [[3, 0], [1, 2]]
    perm, inv = permutation(rows)
    x = torch.arange(4) * 10
    assert torch.equal(x[perm][inv], x)


def test_uneven_batch_is_refused():
    with pytest.raises(ValueError):
        assign_rows([5, 6, 7], 2, 64, 128)


def test_costs_grow_with_length():
    assert row_cost(2048, 768, 3072) > row_cost(1, 768, 3072) > 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    import oracle
    from golden_cases import load_case
    from techjam2026_b200.sharding import BatchShard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = load_case("mini_s333")
        cfg, x, mask = case["cfg"], case["x"], case["mask"]
        lengths = mask.sum(1).tolist()
        shard = BatchShard(lengths, world, rank, cfg.d_model, cfg.ffn_dim, cfg.causal)
        assert shard.local_batch == len(lengths) // world
        out_local = oracle.forward(case["state_dict"], cfg.num_layers, cfg.num_heads,
                                   shard.take(x), shard.take(mask), causal=cfg.causal)
        full = shard.gather(out_local)
        assert torch.equal(shard.take(full), out_local)
        if rank == 0:
            # By value (a numpy array is pickled whole): a tensor would travel
            # as a shared-memory handle that dies with this process.
            q.put(full.numpy().copy())
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_gather_matches_single_process():
    from golden_cases import load_case
    import oracle
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = torch.from_numpy(q.get(timeout=300))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    case = load_case("mini_s333")
    cfg = case["cfg"]
    want = oracle.forward(case["state_dict"], cfg.num_layers, cfg.num_heads, case["x"],
                          case["mask"], causal=cfg.causal)
    assert torch.equal(got, want)


def test_batch_shard_single_rank_is_the_whole_batch():
    from techjam2026_b200.sharding import BatchShard
    w = WORKLOADS["c4"]
    _, mask = generate_case(w.cfg, 0, w.padding_ratio)
    lengths = mask.sum(1).tolist()
    shard = BatchShard(lengths, 1, 0, w.cfg.d_model, w.cfg.ffn_dim)
    assert shard.mine == list(range(64)) and shard.imbalance == 1.0
    t = torch.arange(64 * 3).view(64, 3)
    assert torch.equal(shard.take(t), t) and shard.gather(t) is t
    for world in (2, 4, 8):
        shards = [BatchShard(lengths, world, r, w.cfg.d_model, w.cfg.ffn_dim)
                  for r in range(world)]
        assert all(s.rows == shards[0].rows for s in shards), "every rank derives one plan"
        assert sorted(b for s in shards for b in s.mine) == list(range(64))
        assert sum(sum(s.local_lengths()) for s in shards) == sum(lengths)
    with pytest.raises(ValueError):
        BatchShard(lengths, 2, 2, w.cfg.d_model, w.cfg.ffn_dim)
    with pytest.raises(ValueError):
        shard.take(torch.zeros(3, 2))
