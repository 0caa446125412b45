"""Fused residual-add + row-mask + LayerNorm, same call signature as the
reference's `kernelforge/ops/layernorm.py:101-156` (`add_mask_layernorm`).

    s = (x + y) masked by keep        (fp32)
    h = LayerNorm(s) * w + b          (biased variance, eps inside the sqrt)
    h = h masked by keep              (only with mask_out=True: the final norm,
                                       because LN of an all-zero row is `bias`)

Runs `kf_ln_add_mask` (csrc/ln_sm100.cu). fp32 I/O only: fp16/bf16 I/O is not
implemented and raises.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .. import _lib

HAS_KERNELS = True   # the reference exports HAS_TRITON; ours is the CUDA library

# The warp-per-row kernel keeps the row in registers up to d = 4096 and falls
# back to a three-pass kernel beyond that (still on the GPU).
MAX_D = 1 << 24


def supported(d_model: int) -> bool:
    return 0 < d_model <= MAX_D


def keep_as_u8(keep: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    """[M] keep flags as uint8 bytes (bool is reinterpreted without a copy)."""
    if keep is None:
        return None
    if keep.dtype == torch.bool:
        return keep.contiguous().view(torch.uint8)
    if keep.dtype == torch.uint8:
        return keep.contiguous()
    return (keep != 0).to(torch.uint8)


def add_mask_layernorm(
    x: torch.Tensor,                      # [M, d] residual stream in
    y: Optional[torch.Tensor],            # [M, d] sublayer output, or None
    keep: Optional[torch.Tensor],         # [M] 0/1 (float, bool or uint8), or None
    weight: torch.Tensor,
    bias: torch.Tensor,
    eps: float = 1e-5,
    mask_out: bool = False,
    out_dtype: Optional[torch.dtype] = None,
    residual_dtype: Optional[torch.dtype] = None,
    want_residual: bool = True,
    round_tf32: bool = False,
) -> Tuple[Optional[torch.Tensor], torch.Tensor]:
    """Returns (new_residual_stream or None, normalized_activation)."""
    assert x.dim() == 2, "pass [M, d]"
    M, d = x.shape
    out_dtype = out_dtype or x.dtype
    residual_dtype = residual_dtype or x.dtype
    for t, name in ((x, "x"), (y, "y"), (weight, "weight"), (bias, "bias")):
        if t is not None and t.dtype != torch.float32:
            raise TypeError(f"add_mask_layernorm: {name} must be float32, got {t.dtype}")
    if out_dtype != torch.float32 or residual_dtype != torch.float32:
        raise TypeError("add_mask_layernorm: only float32 outputs are implemented")
    if not x.is_cuda:
        raise RuntimeError("add_mask_layernorm: CUDA tensors required (no CPU path)")
    if x.stride(1) != 1:
        x = x.contiguous()
    if y is not None and y.stride(1) != 1:
        y = y.contiguous()
    weight = weight.contiguous()
    bias = bias.contiguous()
    k8 = keep_as_u8(keep)
    if k8 is not None:
        assert k8.numel() == M, "keep must have one entry per row"

    s_out = torch.empty((M, d), dtype=torch.float32, device=x.device) if want_residual else None
    h_out = torch.empty((M, d), dtype=torch.float32, device=x.device)
    flags = (_lib.KF_LN_MASK_OUT if mask_out else 0) | (_lib.KF_LN_ROUND_TF32 if round_tf32 else 0)
    rc = _lib.lib().kf_ln_add_mask(
        x.data_ptr(), x.stride(0),
        y.data_ptr() if y is not None else None, y.stride(0) if y is not None else 0,
        k8.data_ptr() if k8 is not None else None,
        weight.data_ptr(), bias.data_ptr(),
        s_out.data_ptr() if s_out is not None else None, d,
        h_out.data_ptr(), d, M, d, float(eps), flags, _lib.stream_ptr())
    _lib.check(rc, "kf_ln_add_mask")
    return s_out, h_out
