"""Masked FlashAttention forward, same call signature as the reference's
`kernelforge/ops/flash.py:363-422` (`flash_attention`).

    O = softmax(Q K^T * sm_scale + causal(-inf) + keypad(-inf)) V

per (batch, head), softmax in fp32; Q/K/V are strided [B, H, S, Dh] views
with unit stride on Dh (e.g. views into a fused [B, S, 3, H, Dh] QKV buffer).
Runs `kf_keep_bits`, `kf_attn_schedule` and the persistent
`kf_flash_fwd_tf32_sched` (csrc/flash_persist_sm100.cu), or with
`persistent=False` the one-CTA-per-query-tile `kf_flash_fwd_tf32`
(csrc/flash_sm100.cu); both give the same bits: TF32 tcgen05 contractions
with FP32 TMEM accumulators. A query row whose keys are all masked yields 0
(not NaN), as in the reference kernel (flash.py:241-243).

`smem_kb` and `block` are accepted for signature compatibility; the sm_100
kernel's tiling is fixed per head_dim. `round_scores_to` (fp16/bf16 score
rounding) only applies to narrow I/O dtypes, which are not implemented.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .. import _lib

HAS_KERNELS = True
MIN_HEAD_DIM = 16
SUPPORTED_HEAD_DIMS = (8, 16, 32, 64, 128, 256)


def flash_supported(head_dim: int) -> bool:
    return head_dim in SUPPORTED_HEAD_DIMS


def keep_bits(keep: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Pack a [B, S] keep mask into the kernel's [B, ceil(S/32)] bit words."""
    B, S = keep.shape
    if keep.dtype == torch.bool:
        k8 = keep.contiguous().view(torch.uint8)
    elif keep.dtype == torch.uint8:
        k8 = keep.contiguous()
    else:
        k8 = (keep != 0).to(torch.uint8).contiguous()
    words = int(_lib.lib().kf_keep_bits_words(B, S))
    if out is None:
        out = torch.empty(words, dtype=torch.int32, device=keep.device)
    rc = _lib.lib().kf_keep_bits(k8.data_ptr(), k8.stride(0), B, S, out.data_ptr(),
                                 _lib.stream_ptr())
    _lib.check(rc, "kf_keep_bits")
    return out


def flash_attention(
    q: torch.Tensor,                        # [B, H, S, Dh]
    k: torch.Tensor,
    v: torch.Tensor,
    keep: Optional[torch.Tensor] = None,    # [B, S] key validity, 0/1
    causal: bool = False,
    sm_scale: Optional[float] = None,
    smem_kb: float = 227.0,
    block: Optional[Tuple[int, int, int, int]] = None,
    out: Optional[torch.Tensor] = None,
    round_scores_to: Optional[torch.dtype] = None,
    skip_empty_queries: bool = False,
    round_tf32_out: bool = False,
    persistent: bool = True,
) -> torch.Tensor:
    B, H, S, Dh = q.shape
    assert flash_supported(Dh), f"unsupported head_dim {Dh}"
    for t in (q, k, v):
        if t.dtype != torch.float32:
            raise TypeError("flash_attention: only float32 Q/K/V are implemented")
        if not t.is_cuda:
            raise RuntimeError("flash_attention: CUDA tensors required (no CPU path)")
    if round_scores_to is not None:
        raise NotImplementedError("round_scores_to applies to fp16/bf16 I/O only")
    # The scale uses the ORIGINAL head_dim, before any padding.
    sm_scale = sm_scale if sm_scale is not None else Dh ** -0.5

    dh_store = Dh
    if Dh < MIN_HEAD_DIM:
        # The MMA needs >= 16 columns for O; zero padding is exact. (The layer
        # stack avoids this copy: its QKV GEMM writes the padded layout.)
        dh_store = MIN_HEAD_DIM
        q, k, v = (torch.nn.functional.pad(t, (0, MIN_HEAD_DIM - Dh)) for t in (q, k, v))
    assert q.stride(-1) == 1 and k.stride(-1) == 1 and v.stride(-1) == 1, \
        "flash_attention needs unit stride along head_dim"
    o = out if out is not None else torch.empty((B, H, S, Dh), dtype=torch.float32,
                                                device=q.device)
    assert o.stride(-1) == 1, "output needs unit stride along head_dim"

    bits = keep_bits(keep) if keep is not None else None
    flags = ((_lib.KF_ATTN_CAUSAL if causal else 0)
             | (_lib.KF_ATTN_SKIP_EMPTY_Q if skip_empty_queries else 0)
             | (_lib.KF_ATTN_ROUND_TF32 if round_tf32_out else 0))
    L = _lib.lib()
    st = _lib.stream_ptr()
    args = (q.data_ptr(), q.stride(0), q.stride(1), q.stride(2),
            k.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
            v.data_ptr(), v.stride(0), v.stride(1), v.stride(2),
            o.data_ptr(), o.stride(0), o.stride(1), o.stride(2),
            bits.data_ptr() if bits is not None else None)
    if persistent and B > 0 and H > 0 and S > 0:
        sched = attn_schedule(bits, B, H, S)
        rc = L.kf_flash_fwd_tf32_sched(*args, sched.data_ptr(), B, H, S, dh_store, Dh,
                                       float(sm_scale), flags, st)
        _lib.check(rc, "kf_flash_fwd_tf32_sched")
    else:
        rc = L.kf_flash_fwd_tf32(*args, B, H, S, dh_store, Dh, float(sm_scale), flags, st)
        _lib.check(rc, "kf_flash_fwd_tf32")
    return o


def attn_schedule(bits: Optional[torch.Tensor], B: int, H: int, S: int,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Work list of the persistent attention for key bits of [B, S] rows
    (None: every key valid) and H heads (kf_attn_schedule)."""
    L = _lib.lib()
    words = int(L.kf_attn_schedule_words(B, H, S))
    device = bits.device if bits is not None else torch.device("cuda", torch.cuda.current_device())
    if out is None:
        out = torch.empty(words, dtype=torch.int32, device=device)
    rc = L.kf_attn_schedule(bits.data_ptr() if bits is not None else None, B, H, S,
                            out.data_ptr(), _lib.stream_ptr())
    _lib.check(rc, "kf_attn_schedule")
    return out
