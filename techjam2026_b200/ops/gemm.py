"""tcgen05 TF32 linear layer: out = epilogue(x @ weight^T + bias).

Replaces the cuBLAS `F.linear` calls of the reference's fused forward
(`kernelforge/optimized.py:441-446, 483, 573`); the GELU(erf) of FFN1
(`optimized.py:443`) is fused into the epilogue. Runs `kf_gemm_tf32`
(csrc/gemm_sm100.cu).
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import _lib


def linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
           gelu: bool = False, out: Optional[torch.Tensor] = None, round_tf32: bool = False,
           bn: int = 0, precision: str = "bf16x3") -> torch.Tensor:
    """x [M, K] fp32 (unit inner stride), weight [N, K] fp32 -> [M, N] fp32.

    precision
      "bf16x3": error-compensated hi*hi + hi*lo + lo*hi of a bf16 hi/lo split
                on the BF16 tensor path (~2^-17 relative, 1.5x one TF32 pass);
      "3xtf32": the same compensation with a TF32 split (~2^-20, 3x);
      "tf32":   one TF32 MMA per k step (the tensor core drops the low 13
                mantissa bits of each operand, ~2^-11)."""
    if precision not in _lib.GEMM_PRECISION_FLAGS:
        raise ValueError(f"precision must be one of {sorted(_lib.GEMM_PRECISION_FLAGS)}")
    if x.dtype != torch.float32 or weight.dtype != torch.float32:
        raise TypeError("linear: only float32 operands are implemented")
    if not x.is_cuda:
        raise RuntimeError("linear: CUDA tensors required (no CPU path)")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    weight = weight.contiguous()
    M, K = x2.shape
    N = weight.shape[0]
    assert weight.shape[1] == K, "weight must be [N, K]"
    if bias is not None:
        bias = bias.contiguous()
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=x.device)
    assert out.stride(-1) == 1
    rc = _lib.lib().kf_gemm_tf32(
        x2.data_ptr(), x2.stride(0), weight.data_ptr(), weight.stride(0),
        bias.data_ptr() if bias is not None else None,
        out.data_ptr(), out.stride(0), M, N, K,
        _lib.KF_EPI_BIAS_GELU if gelu else _lib.KF_EPI_BIAS,
        (_lib.KF_GEMM_ROUND_TF32 if round_tf32 else 0)
        | _lib.GEMM_PRECISION_FLAGS[precision], bn, 0, 0, None, None, _lib.stream_ptr())
    _lib.check(rc, "kf_gemm_tf32")
    return out.reshape(*lead, N)


def round_tf32(t: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Round fp32 values to the nearest TF32 value (weight preparation)."""
    t = t.contiguous()
    out = torch.empty_like(t) if out is None else out
    rc = _lib.lib().kf_round_tf32(t.data_ptr(), out.data_ptr(), t.numel(), _lib.stream_ptr())
    _lib.check(rc, "kf_round_tf32")
    return out
