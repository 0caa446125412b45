"""Drop-in entry: `UserOptimizedTransformer` for torch_transformer_benchmark.py.

Same contract as the reference's submission.py:40-106:
  * subclasses the organiser's BaselineTransformer, so parameter names are
    unchanged and `copy_model_weights(strict=True)` works;
  * picks a plan from the sm_100 dispatch table on the first forward (which
    falls inside the harness's warm-up) and runs the CUDA path
    (techjam2026_b200.fused.FusedTransformer, whole forward in one CUDA graph);
    at float16/bfloat16 I/O the plan is the organiser's own layer captured
    whole into one CUDA graph (techjam2026_b200.exact: the gate admits only
    its exact arithmetic there, as the reference's own table records);
  * if choosing or running the CUDA path raises, it says so on stdout and
    returns the organiser's baseline answer from then on (sticky), because the
    harness's accuracy gate is a hard failure. Nothing is silent;
  * the library's kernels never hang: a wait that gives up records a device
    status word instead. After every fused forward a 4-byte copy of that word
    is queued on a side stream (no synchronisation); the next call reads it
    and, if a kernel reported a failure, falls back the same way.

Use inside the organiser's harness either by replacing the class body with
`from submission import UserOptimizedTransformer`, or by assigning
`torch_transformer_benchmark.UserOptimizedTransformer = UserOptimizedTransformer`
before calling its main() (the reference's scripts/run_official.py:18-24).

Without the organiser's module on the path, the base class is
techjam2026_b200.model.LayerStack (same parameter tree, no forward of its
own): the fallback then raises instead of returning a baseline answer.
"""
from __future__ import annotations

import os
from typing import Optional

import torch

try:  # the organiser's harness: the normal way this class is used
    from torch_transformer_benchmark import BaselineTransformer, TransformerConfig  # noqa: F401
    HAS_ORGANISER_BASELINE = True
except Exception:  # standalone: parameter container with the same tree
    from techjam2026_b200.configs import TransformerConfig  # noqa: F401
    from techjam2026_b200.model import LayerStack as BaselineTransformer
    HAS_ORGANISER_BASELINE = False

from techjam2026_b200.dispatch import DispatchTable, Plan, probe
from techjam2026_b200.exact import ExactGraphForward
from techjam2026_b200.fused import FusedTransformer

_VERBOSE = os.environ.get("KF_VERBOSE", "") not in ("", "0")


class UserOptimizedTransformer(BaselineTransformer):
    """The submitted implementation (forward replaced, parameters unchanged)."""

    def __init__(self, config) -> None:
        super().__init__(config)
        self._impl = None  # FusedTransformer, or ExactGraphForward (fp16/bf16)
        self._plan: Optional[Plan] = None
        self._source = "uninitialized"
        self._failed = False
        self._status_host = None    # pinned int32: the device status word, read async
        self._status_stream = None
        self._status_event = None

    def _select(self, x: torch.Tensor) -> None:
        if self._impl is not None or self._failed:
            return
        try:
            if not x.is_cuda:
                raise RuntimeError("input is on the CPU; the fused path runs on sm_100 only")
            spec = probe(x.device.index)
            plan, source = DispatchTable.load_for(spec).lookup(
                spec.arch, x.dtype, self.config, spec.shared_mem_per_block_kb)
            if plan.exact_reference:
                # float16 / bfloat16: the organiser's own layer, whole forward
                # in one CUDA graph (bit-identical to its eager forward).
                if not HAS_ORGANISER_BASELINE:
                    raise RuntimeError(
                        f"{x.dtype} I/O runs the organiser's exact layer, and "
                        "torch_transformer_benchmark is not importable")
                base_forward = super().forward
                impl = ExactGraphForward(lambda xx, mm: base_forward(xx, mm))
            else:
                impl = FusedTransformer(self.config, plan)
                impl.load_state_dict(self.state_dict(), strict=True)
                impl.eval()
            self._impl, self._plan, self._source = impl, plan, source
            if _VERBOSE:
                print(f"[kf-b200] {spec.arch} {x.dtype} -> {plan.name} ({source}): "
                      f"{plan.describe()}")
        except Exception as e:
            self._failed = True
            print(f"[kf-b200] cannot use the sm_100 path ({type(e).__name__}: {e}); "
                  f"falling back to the reference implementation")

    def _reported_failure(self) -> int:
        """The library's device status word as of the previous fused forward
        (0 while its read has not landed yet)."""
        ev = self._status_event
        if ev is None or not ev.query():
            return 0
        return int(self._status_host[0])

    def _queue_status_read(self, device: torch.device) -> None:
        from techjam2026_b200 import _lib
        if self._status_host is None:
            self._status_host = torch.zeros(1, dtype=torch.int32).pin_memory()
            self._status_stream = torch.cuda.Stream(device=device)
        self._status_stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(self._status_stream):
            _lib.check(_lib.lib().kf_device_status_async(self._status_host.data_ptr(),
                                                         _lib.stream_ptr()),
                       "kf_device_status_async")
            ev = torch.cuda.Event()
            ev.record(self._status_stream)
        self._status_event = ev

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None
                ) -> torch.Tensor:
        self._select(x)
        if self._impl is None:
            return super().forward(x, valid_token_mask)
        fused = isinstance(self._impl, FusedTransformer)
        code = self._reported_failure() if fused else 0
        if code:
            self._failed, self._impl = True, None
            print(f"[kf-b200] the CUDA kernels reported device status {code} (a bounded wait "
                  f"gave up on this GPU)\n[kf-b200] falling back to the reference "
                  f"implementation for the rest of this run; results stay correct, speed does not.")
            return super().forward(x, valid_token_mask)
        try:
            out = self._impl(x, valid_token_mask)
            if fused:
                self._queue_status_read(x.device)
            return out
        except Exception as e:
            self._failed, self._impl = True, None
            print(f"[kf-b200] the fused path raised {type(e).__name__}: {e}\n"
                  f"[kf-b200] falling back to the reference implementation for the rest "
                  f"of this run; results stay correct, speed does not.")
            return super().forward(x, valid_token_mask)
