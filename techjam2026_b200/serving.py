"""Streamed forward over a sequence of host batches (the serving loop).

A serving process receives batches in host memory and returns results in
host memory. Run one after another, every batch pays its host->device copy,
the forward, and its device->host copy in turn. `StreamedForward` overlaps
them: while the forward of batch k runs on the caller's stream, the upload
of batch k+1 runs on one copy stream and the download of result k-1 on
another. PCIe is full duplex and the GPU has several copy engines, so in
steady state a batch costs the longest of the three, not their sum. Device
buffers are double-buffered; every batch still crosses PCIe both ways.

Padding stays on the host. With a bool prefix mask (each row's valid
tokens first, as the organiser's generator draws them) only each row's
valid prefix crosses PCIe in either direction: the forward never reads a
padded row of x (the first norm masks it by a select), and a padded row of
the result is exactly zero, which the loop writes into the host result
buffer itself (once per buffer, and again only where a row got shorter).
For c4 that is about half the bytes of the whole [B, S, d] tensors.

The forward itself is the model's CUDA graph, so results are bit-identical
to calling the model on each batch. For a `FusedTransformer` with a bool
mask (or none) there is one graph per buffer slot, captured on that slot's
upload and download buffers, so a step makes no device-side copy; other
models use their `graph_runner` and copy into and out of its buffers.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from .fused import FusedTransformer, GraphRunner, _Workspace


class StreamedForward:
    """Pipelined forward of one fixed batch shape.

    `x_example` / `mask_example` are device tensors of that shape (their
    values are not used). Host tensors passed to `run` should be pinned;
    otherwise the copies are synchronous and nothing overlaps."""

    def __init__(self, model: FusedTransformer, x_example: torch.Tensor,
                 mask_example: Optional[torch.Tensor] = None, packed: bool = True):
        if not x_example.is_cuda:
            raise ValueError("x_example must be a CUDA tensor of the batch shape")
        self.device = x_example.device
        self.with_mask = mask_example is not None
        self.xd = [torch.empty_like(x_example).contiguous() for _ in range(2)]
        self.md = ([torch.empty_like(mask_example).contiguous() for _ in range(2)]
                   if self.with_mask else [None, None])
        self.od = [torch.empty_like(x_example).contiguous() for _ in range(2)]
        self.up = torch.cuda.Stream(device=self.device)
        self.down = torch.cuda.Stream(device=self.device)
        self.bound = None
        self.runner = None
        if isinstance(model, FusedTransformer) and (
                mask_example is None or mask_example.dtype == torch.bool):
            B, S, _ = x_example.shape
            ws = _Workspace(model.config, B, S, self.device, model.plan)
            self.bound = [GraphRunner(model, self.xd[b], self.md[b], self.od[b], ws)
                          for b in range(2)]
        else:
            self.runner = model.graph_runner(x_example, mask_example)
        # Copies of valid prefixes only (fused model with a bool mask).
        self.packed = packed and self.bound is not None
        # Host result buffers: rows this loop has written per batch row
        # (None: unknown) and the event of the last download into each.
        self._out_rows = {}
        self._out_event = {}
        self.last_h2d_bytes = 0
        self.last_d2h_bytes = 0

    @staticmethod
    def prefix_lengths(mask: Optional[torch.Tensor]) -> Optional[List[int]]:
        """Valid length of every row of a host bool [B, S] mask whose valid
        tokens form a prefix of the row; None for any other mask."""
        if (mask is None or mask.is_cuda or mask.dtype != torch.bool or mask.dim() != 2):
            return None
        lens = mask.sum(dim=1)
        if not torch.equal(torch.arange(mask.shape[1])[None, :] < lens[:, None], mask):
            return None
        return [int(v) for v in lens.tolist()]

    def _clear_padding(self, out: torch.Tensor, lens: List[int]) -> None:
        """Make the padded rows of host result buffer `out` zero before a
        download of valid prefixes only: all of them the first time the
        buffer is seen, later only rows that were valid in its last use.
        Rows an earlier download may still be writing are cleared only after
        that download has finished."""
        key = (out.data_ptr(), tuple(out.shape))
        prev = self._out_rows.get(key)
        S = out.shape[1]
        todo = [(i, l, S if prev is None else prev[i]) for i, l in enumerate(lens)]
        todo = [(i, a, e) for i, a, e in todo if e > a]
        if todo:
            ev = self._out_event.get(key)
            if ev is not None:
                ev.synchronize()
            for i, a, e in todo:
                out[i, a:e].zero_()
        self._out_rows[key] = list(lens)

    def run(self, xs: Sequence[torch.Tensor], masks: Optional[Sequence[torch.Tensor]],
            outs: Sequence[torch.Tensor], before_step=None) -> None:
        """Forward xs[k] (with masks[k]) into outs[k] for every k.

        Everything is queued asynchronously; the caller's current stream
        waits for the last download, so outs are ready once that stream is
        synchronized. `before_step(k)`, if given, is called on the caller's
        stream just before forward k is queued (the benchmark flushes L2
        there). Host tensors must stay alive until then."""
        n = len(xs)
        if n == 0:
            return
        if len(outs) != n or (self.with_mask and (masks is None or len(masks) != n)):
            raise ValueError("xs, masks and outs must have the same length")
        comp = torch.cuda.current_stream(self.device)
        uploaded = [torch.cuda.Event() for _ in range(n)]
        loaded = [torch.cuda.Event() for _ in range(n)]
        computed = [torch.cuda.Event() for _ in range(n)]
        downloaded = [torch.cuda.Event() for _ in range(n)]
        self.up.wait_stream(comp)
        self.down.wait_stream(comp)
        memo = {}  # one prefix check per distinct mask tensor of the call

        def lengths_of(m):
            if id(m) not in memo:
                memo[id(m)] = self.prefix_lengths(m)
            return memo[id(m)]
        lens = [lengths_of(masks[k]) if (self.packed and masks is not None) else None
                for k in range(n)]
        row_bytes = xs[0].shape[-1] * xs[0].element_size()
        h2d = d2h = 0
        for k in range(n):
            full = xs[k].numel() * xs[k].element_size()
            h2d += full if lens[k] is None else sum(lens[k]) * row_bytes
            d2h += full if lens[k] is None else sum(lens[k]) * row_bytes
            if self.with_mask:
                h2d += masks[k].numel() * masks[k].element_size()
        self.last_h2d_bytes, self.last_d2h_bytes = h2d // n, d2h // n

        def upload(k: int) -> None:
            b = k % 2
            with torch.cuda.stream(self.up):
                if k >= 2:
                    self.up.wait_event(loaded[k - 2])  # forward k-2 has read buffer b
                if lens[k] is None:
                    self.xd[b].copy_(xs[k], non_blocking=True)
                else:
                    for i, l in enumerate(lens[k]):
                        if l:
                            self.xd[b][i, :l].copy_(xs[k][i, :l], non_blocking=True)
                if self.with_mask:
                    self.md[b].copy_(masks[k], non_blocking=True)
                uploaded[k].record(self.up)

        upload(0)
        for k in range(n):
            b = k % 2
            if k + 1 < n:
                upload(k + 1)
            if before_step is not None:
                before_step(k)
            comp.wait_event(uploaded[k])
            if self.bound is not None:
                if k >= 2:
                    comp.wait_event(downloaded[k - 2])  # result k-2 has left buffer b
                self.bound[b].replay()                  # reads xd[b], md[b]; writes od[b]
                loaded[k].record(comp)
            else:
                self.runner.load_inputs(self.xd[b], self.md[b])
                loaded[k].record(comp)
                self.runner.replay()
                if k >= 2:
                    comp.wait_event(downloaded[k - 2])  # result k-2 has left buffer b
                self.od[b].copy_(self.runner.static_out)
            computed[k].record(comp)
            with torch.cuda.stream(self.down):
                self.down.wait_event(computed[k])
                key = (outs[k].data_ptr(), tuple(outs[k].shape))
                if lens[k] is None:
                    outs[k].copy_(self.od[b], non_blocking=True)
                    self._out_rows[key] = None
                else:
                    self._clear_padding(outs[k], lens[k])
                    for i, l in enumerate(lens[k]):
                        if l:
                            outs[k][i, :l].copy_(self.od[b][i, :l], non_blocking=True)
                downloaded[k].record(self.down)
                self._out_event[key] = downloaded[k]
        comp.wait_event(downloaded[n - 1])

    def __call__(self, xs: List[torch.Tensor], masks: Optional[List[torch.Tensor]] = None
                 ) -> List[torch.Tensor]:
        """Convenience form: returns new pinned host outputs, synchronized."""
        outs = [torch.empty(x.shape, dtype=x.dtype, pin_memory=True) for x in xs]
        self.run(xs, masks, outs)
        torch.cuda.current_stream(self.device).synchronize()
        return outs
