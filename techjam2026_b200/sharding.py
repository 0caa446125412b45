"""Batch sharding of the layer stack across GPUs (one process per GPU).

No op of the stack mixes batch elements (kernelforge/optimized.py:343-348),
so the forward needs no inter-GPU traffic: each rank runs the rows it owns
with its own CUDA graph. Two policies:

  * replicas: every rank runs a full batch of its own (used only when the
    batch does not split evenly, e.g. c1's two rows over four GPUs);
  * a fixed global batch split across ranks (`BatchShard`, the bench's
    mode: strong scaling): equal row counts per rank (one
    static shape, one graph) with a cost-balanced assignment -- greedy
    largest-first over the per-row cost 2*L*(4d^2+2dF) + 4d*L(L+1)/2 -- so the
    slowest rank is not the one that drew all the long sequences (lengths vary
    1..2048 in c4). The permutation is recorded and undone after the gather.

`gather_rows` is the optional all-gather that assembles a single result
tensor (torch.distributed.all_gather_into_tensor: NCCL over NVLink on GPUs,
gloo on CPU); it is the only collective, and the forward itself never calls
it.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

import torch


def row_cost(length: int, d: int, ffn: int, causal: bool = True) -> float:
    pairs = length * (length + 1) / 2 if causal else float(length * length)
    return 2.0 * length * (4 * d * d + 2 * d * ffn) + 4.0 * d * pairs


def assign_rows(lengths: Sequence[int], world: int, d: int, ffn: int,
                causal: bool = True) -> List[List[int]]:
    """Rows per rank: equal counts (B must divide by world), greedy
    largest-cost-first onto the least-loaded rank that still has room."""
    B = len(lengths)
    if world <= 0 or B % world:
        raise ValueError(f"batch {B} does not split evenly over {world} ranks")
    cap = B // world
    order = sorted(range(B), key=lambda b: (-row_cost(lengths[b], d, ffn, causal), b))
    load = [0.0] * world
    rows: List[List[int]] = [[] for _ in range(world)]
    for b in order:
        r = min((r for r in range(world) if len(rows[r]) < cap), key=lambda r: (load[r], r))
        rows[r].append(b)
        load[r] += row_cost(lengths[b], d, ffn, causal)
    return [sorted(r) for r in rows]


def imbalance(lengths: Sequence[int], rows: List[List[int]], d: int, ffn: int,
              causal: bool = True) -> float:
    """max(rank cost) / mean(rank cost); 1.0 is perfect balance."""
    costs = [sum(row_cost(lengths[b], d, ffn, causal) for b in r) for r in rows]
    mean = sum(costs) / len(costs)
    return max(costs) / mean if mean > 0 else 1.0


def permutation(rows: List[List[int]]) -> Tuple[torch.Tensor, torch.Tensor]:
    """(perm, inverse): concatenated rank order and the map back to batch order."""
    perm = torch.tensor([b for r in rows for b in r], dtype=torch.long)
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(perm.numel())
    return perm, inv


def gather_rows(local: torch.Tensor, rows: List[List[int]], group=None) -> torch.Tensor:
    """All-gather every rank's [B/world, ...] output into one [B, ...] tensor in
    the original batch order."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    full = torch.empty((local.shape[0] * world,) + tuple(local.shape[1:]), dtype=local.dtype,
                       device=local.device)
    dist.all_gather_into_tensor(full, local.contiguous(), group=group)
    _, inv = permutation(rows)
    return full[inv.to(full.device)]


class BatchShard:
    """This rank's share of one fixed global batch.

    Built from the global batch's valid lengths (every rank computes the same
    assignment from the same lengths, so no message is needed to agree on
    it): `rows` holds every rank's batch indices, `mine` this rank's, in
    ascending order. `take(t)` selects this rank's rows of any [B, ...]
    tensor (inputs on the host or the device), `gather(out)` runs the one
    collective and returns the whole [B, ...] result in batch order on every
    rank. With world == 1 the shard is the whole batch and `gather` is the
    identity."""

    def __init__(self, lengths: Sequence[int], world: int, rank: int, d: int, ffn: int,
                 causal: bool = True):
        if not 0 <= rank < world:
            raise ValueError(f"rank {rank} outside a world of {world}")
        self.world, self.rank = world, rank
        self.lengths = [int(v) for v in lengths]
        self.rows = assign_rows(self.lengths, world, d, ffn, causal)
        self.mine = self.rows[rank]
        self.imbalance = imbalance(self.lengths, self.rows, d, ffn, causal)
        self._index = torch.tensor(self.mine, dtype=torch.long)

    @property
    def local_batch(self) -> int:
        return len(self.mine)

    def local_lengths(self) -> List[int]:
        return [self.lengths[b] for b in self.mine]

    def take(self, t: torch.Tensor) -> torch.Tensor:
        if t.shape[0] != len(self.lengths):
            raise ValueError(f"expected a batch of {len(self.lengths)} rows, got {t.shape[0]}")
        return t.index_select(0, self._index.to(t.device)).contiguous()

    def gather(self, local: torch.Tensor, group=None) -> torch.Tensor:
        if self.world == 1:
            return local
        return gather_rows(local, self.rows, group)
