"""Whole-forward CUDA graph around an exact reference forward (narrow dtypes).

At float16/bfloat16 I/O the organiser's gate compares against the reference
layer run in that dtype, whose own rounding (scores, probabilities, every
GEMM output and residual rounded to the I/O dtype) is amplified through the
stack. Any reassociation of those roundings fails the gate: the reference
measured envelopes of 2.2-3.0 (fp16) and 18-21 (bf16) for its fused QKV,
fused norm, SDPA and its own flash kernel, and 0.000 only for its
structurally rewritten but arithmetically identical path
(kernelforge docs/PRECISION.md:59-135; its dispatch table ships
"safe(exact)+graph" plans there, kernelforge/dispatch.py:315-318). The same
holds for any kernel of ours, so at those dtypes the admissible plan is the
reference's own forward, captured once per input shape into one CUDA graph
and replayed: the same library calls in the same order, so the output is
bit-identical to the eager forward, minus the per-op launch overhead.

float32 I/O never takes this path (it runs techjam2026_b200.fused).
"""
from __future__ import annotations

from typing import Callable, Dict, Optional, Tuple

import torch

NARROW_DTYPES = (torch.float16, torch.bfloat16)


class _Captured:
    def __init__(self, fn: Callable, x: torch.Tensor, mask: Optional[torch.Tensor]):
        self.static_x = x.detach().clone()
        self.static_mask = None if mask is None else mask.detach().clone()
        side = torch.cuda.Stream(device=x.device)
        side.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(side), torch.inference_mode():
            for _ in range(2):  # library handles, cuBLAS workspaces, lazy init
                fn(self.static_x, self.static_mask)
        torch.cuda.current_stream(x.device).wait_stream(side)
        torch.cuda.synchronize(x.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph), torch.inference_mode():
            self.static_out = fn(self.static_x, self.static_mask)

    def __call__(self, x: torch.Tensor, mask: Optional[torch.Tensor]) -> torch.Tensor:
        self.static_x.copy_(x, non_blocking=True)
        if self.static_mask is not None:
            self.static_mask.copy_(mask, non_blocking=True)
        self.graph.replay()
        return self.static_out.clone()


class ExactGraphForward:
    """`fn(x, mask) -> out` replayed from one CUDA graph per (shape, dtype,
    device, mask presence). `fn` must be the exact reference forward; inputs
    are copied into static buffers and the output is cloned (the next replay
    overwrites the static output)."""

    def __init__(self, fn: Callable):
        self.fn = fn
        self._graphs: Dict[Tuple, _Captured] = {}

    def __call__(self, x: torch.Tensor, mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        if not x.is_cuda:
            raise RuntimeError("ExactGraphForward captures CUDA graphs: CUDA inputs required")
        if mask is not None and mask.device != x.device:
            raise RuntimeError("valid_token_mask must be on the input's device")
        key = (tuple(x.shape), x.dtype, str(x.device), mask is None,
               None if mask is None else mask.dtype)
        cap = self._graphs.get(key)
        if cap is None:
            cap = _Captured(self.fn, x, mask)
            self._graphs[key] = cap
        return cap(x, mask)

    def clear(self) -> None:
        self._graphs.clear()
