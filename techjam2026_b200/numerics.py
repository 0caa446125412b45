"""The accuracy gate of the organiser's harness, plus envelope utilisation.

Rule (torch_transformer_benchmark.py:309-316, restated by the reference in
kernelforge/numerics.py:98-152): every element must be finite and satisfy

    |opt - ref| <= atol   OR   |opt - ref| <= rtol * |ref|

which is stricter than torch.isclose (atol + rtol*|ref|). Defaults are the
script's: atol = 2e-3, rtol = 2e-2 (torch_transformer_benchmark.py:615-616).

Envelope utilisation = max(|err| / max(atol, rtol*|ref|)): < 1 passes, and the
reference admits a plan only below 0.80 (kernelforge/numerics.py:66-68).
"""
from __future__ import annotations

import dataclasses
from typing import Optional, Tuple

import torch

ATOL = 2e-3
RTOL = 2e-2
ADMISSION_MARGIN = 0.80


@dataclasses.dataclass
class CheckResult:
    passed: bool
    max_abs_error: float
    max_rel_error: float
    mean_abs_error: float
    failed_elements: int
    total_elements: int
    worst_index: Optional[Tuple[int, ...]]
    reference_at_worst: float
    optimized_at_worst: float
    envelope_utilization: float
    note: str = ""

    def __str__(self) -> str:
        status = "PASS" if self.passed else "FAIL"
        return (f"{status} | max_abs={self.max_abs_error:.3e} "
                f"max_rel={self.max_rel_error:.3e} "
                f"envelope={self.envelope_utilization:.3f} "
                f"failed={self.failed_elements}/{self.total_elements}"
                + (f" | {self.note}" if self.note else ""))


def check(reference: torch.Tensor, optimized: torch.Tensor, rtol: float = RTOL,
          atol: float = ATOL) -> CheckResult:
    """Apply the gate elementwise; both tensors are compared in fp32 on the
    reference's device (the candidate is moved there)."""
    if tuple(reference.shape) != tuple(optimized.shape):
        return CheckResult(False, float("inf"), float("inf"), float("inf"),
                           reference.numel(), reference.numel(), None, 0.0, 0.0,
                           float("inf"),
                           note=f"shape mismatch {tuple(reference.shape)} vs "
                                f"{tuple(optimized.shape)}")
    ref = reference.detach().float()
    opt = optimized.detach().float().to(ref.device)
    if ref.numel() == 0:
        return CheckResult(True, 0.0, 0.0, 0.0, 0, 0, None, 0.0, 0.0, 0.0)
    finite = torch.isfinite(ref) & torch.isfinite(opt)
    abs_err = (opt - ref).abs()
    passed_mask = finite & ((abs_err <= atol) | (abs_err <= rtol * ref.abs()))
    failed = int((~passed_mask).sum().item())
    allowed = torch.clamp(rtol * ref.abs(), min=atol)
    ratio = torch.where(finite, abs_err / allowed, torch.full_like(abs_err, float("inf")))
    utilization = float(ratio.max().item())
    safe_err = torch.where(finite, abs_err, torch.full_like(abs_err, float("inf")))
    flat_worst = int(safe_err.reshape(-1).argmax().item())
    idx, rem = [], flat_worst
    for size in reversed(ref.shape):
        idx.append(rem % size)
        rem //= size
    worst = tuple(reversed(idx))
    note = ""
    if not bool(finite.all()):
        note = f"{int((~finite).sum().item())} non-finite element(s)"
    return CheckResult(
        passed=failed == 0,
        max_abs_error=float(abs_err[finite].max().item()) if bool(finite.any()) else float("inf"),
        max_rel_error=float((abs_err / ref.abs().clamp_min(1e-12))[finite].max().item())
        if bool(finite.any()) else float("inf"),
        mean_abs_error=float(abs_err[finite].mean().item()) if bool(finite.any()) else float("inf"),
        failed_elements=failed,
        total_elements=ref.numel(),
        worst_index=worst,
        reference_at_worst=float(ref[worst].item()),
        optimized_at_worst=float(opt[worst].item()),
        envelope_utilization=utilization,
        note=note,
    )


def padded_rows_exactly_zero(out: torch.Tensor, valid_token_mask: torch.Tensor) -> bool:
    """Bit-exact mask handling: every row whose token is padding is +0.0/-0.0."""
    dead = ~valid_token_mask.to(out.device).bool()
    return int(torch.count_nonzero(out[dead]).item()) == 0
