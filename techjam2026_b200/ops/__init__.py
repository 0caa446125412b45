"""The CUDA kernels, re-exported with the reference's ops surface
(`kernelforge/ops/__init__.py:7-11`) plus the tcgen05 linear layer."""
from .layernorm import add_mask_layernorm, HAS_KERNELS
from .flash import flash_attention, flash_supported
from .gemm import linear, round_tf32

__all__ = ["add_mask_layernorm", "flash_attention", "flash_supported", "linear",
           "round_tf32", "HAS_KERNELS"]
