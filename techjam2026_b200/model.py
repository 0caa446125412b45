"""Parameter container with the reference's module tree.

`LayerStack` has exactly the module names and parameter shapes of the
organiser's BaselineTransformer (torch_transformer_benchmark.py:59-172), so
its state_dict keys are identical and `copy_model_weights(strict=True)`
(:203-213) works in both directions:

    layers.{i}.norm1.{weight,bias}
    layers.{i}.attention.{q_proj,k_proj,v_proj,out_proj}.{weight,bias}
    layers.{i}.norm2.{weight,bias}
    layers.{i}.ffn_in.{weight,bias}, layers.{i}.ffn_out.{weight,bias}
    final_norm.{weight,bias}

It holds parameters only; its forward raises. The computation lives in
`techjam2026_b200.fused.FusedTransformer` (CUDA, sm_100a). When the
organiser's module is importable, `submission.py` subclasses that instead.
"""
from __future__ import annotations

import torch.nn as nn


class SelfAttentionParams(nn.Module):
    def __init__(self, d_model: int, num_heads: int) -> None:
        super().__init__()
        if d_model % num_heads:
            raise ValueError("d_model must be divisible by num_heads")
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.q_proj = nn.Linear(d_model, d_model)
        self.k_proj = nn.Linear(d_model, d_model)
        self.v_proj = nn.Linear(d_model, d_model)
        self.out_proj = nn.Linear(d_model, d_model)


class BlockParams(nn.Module):
    def __init__(self, d_model: int, num_heads: int, ffn_dim: int) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(d_model)
        self.attention = SelfAttentionParams(d_model, num_heads)
        self.norm2 = nn.LayerNorm(d_model)
        self.ffn_in = nn.Linear(d_model, ffn_dim)
        self.ffn_out = nn.Linear(ffn_dim, d_model)


class LayerStack(nn.Module):
    def __init__(self, config) -> None:
        super().__init__()
        self.config = config
        self.layers = nn.ModuleList(
            [BlockParams(config.d_model, config.num_heads, config.ffn_dim)
             for _ in range(config.num_layers)])
        self.final_norm = nn.LayerNorm(config.d_model)

    def forward(self, x, valid_token_mask=None):  # pragma: no cover - by design
        raise RuntimeError(
            "LayerStack only holds parameters; run the stack with "
            "techjam2026_b200.fused.FusedTransformer on an sm_100 GPU")
