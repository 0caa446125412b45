"""Workload definitions and the seeded input / weight generators.

`TransformerConfig` has the fields of the organiser's dataclass
(torch_transformer_benchmark.py:29-56); any object with those attributes is
accepted everywhere (the organiser's own instances included).

`generate_case` reproduces torch_transformer_benchmark.py:234-272
(`generate_random_case`) draw for draw on a CPU generator, so the same seed
gives the same x and valid_token_mask as the organiser's harness run with
device="cpu". Inputs are always drawn on the CPU and then moved: CPU and CUDA
generators produce different streams.

`init_params_` applies the weight convention the benchmark configurations
specify (Xavier-uniform weights, zero biases, LayerNorm gamma = 1, beta = 0)
in named_parameters() order from one seeded generator.
"""
from __future__ import annotations

import dataclasses
from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn


@dataclasses.dataclass(frozen=True)
class TransformerConfig:
    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool

    def validate(self) -> None:
        for name in ("batch_size", "seq_len", "d_model", "num_heads", "ffn_dim", "num_layers"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be positive")
        if self.d_model % self.num_heads != 0:
            raise ValueError(f"d_model ({self.d_model}) must be divisible by "
                             f"num_heads ({self.num_heads})")


def signature(cfg) -> str:
    """Shape signature in the reference's dispatch format (dispatch.py:40-44)."""
    return (f"B{cfg.batch_size}-S{cfg.seq_len}-d{cfg.d_model}-H{cfg.num_heads}"
            f"-F{cfg.ffn_dim}-L{cfg.num_layers}{'-causal' if cfg.causal else ''}")


@dataclasses.dataclass(frozen=True)
class Workload:
    """One BASELINE.json configuration: a model shape plus its input law."""
    name: str
    cfg: TransformerConfig
    padding_ratio: float          # lengths ~ U[max(1, round(S*(1-p))), S]
    seeds: Tuple[int, ...] = (0,)
    input_scale: float = 1.0
    note: str = ""


def _c(B, S, d, H, F, L) -> TransformerConfig:
    return TransformerConfig(B, S, d, H, F, L, True)


# BASELINE.json "configs", in order. All are causal with key padding; FFN is
# GELU(erf) as in the reference layer (torch_transformer_benchmark.py:141).
WORKLOADS: Dict[str, Workload] = {
    "c1": Workload("c1", _c(2, 64, 128, 4, 512, 1), 0.5, (0,),
                   note="1 layer, lengths U[32,64]"),
    "c2": Workload("c2", _c(8, 512, 512, 8, 2048, 6), 0.5, (0, 1, 2),
                   note="6-layer stack, lengths U[256,512]"),
    "c3a": Workload("c3a", _c(16, 1024, 128, 16, 512, 2), 0.5, (0,),
                    note="head_dim 8 (zero-padded to 16)"),
    "c3b": Workload("c3b", _c(16, 1024, 1024, 4, 4096, 2), 0.5, (0,),
                    note="head_dim 256"),
    "c4": Workload("c4", _c(64, 2048, 768, 12, 3072, 4), 0.9999, (0,),
                   note="heavy padding, lengths U[1,2048]"),
    "c5": Workload("c5", _c(16, 65536, 1024, 16, 1024, 2), 0.5, (0,),
                   note="long sequence, lengths U[32768,65536]"),
}


def generate_case(cfg, seed: int, padding_ratio: float, input_scale: float = 1.0,
                  batch_size: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """x [B,S,d] fp32 and valid_token_mask [B,S] bool, drawn on the CPU."""
    B = cfg.batch_size if batch_size is None else batch_size
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    x = torch.randn(B, cfg.seq_len, cfg.d_model, generator=g, dtype=torch.float32)
    x = x * input_scale
    if padding_ratio <= 0:
        return x, torch.ones(B, cfg.seq_len, dtype=torch.bool)
    min_valid = max(1, int(round(cfg.seq_len * (1.0 - padding_ratio))))
    lengths = torch.randint(low=min_valid, high=cfg.seq_len + 1, size=(B,), generator=g)
    mask = torch.arange(cfg.seq_len)[None, :] < lengths[:, None]
    x = x.masked_fill(~mask[..., None], 0)
    return x, mask


def init_params_(model: nn.Module, seed: int) -> nn.Module:
    """Xavier-uniform weights, zero biases, LayerNorm (1, 0); deterministic in
    named_parameters() order."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if p.dim() == 2:
                w = torch.empty(p.shape, dtype=torch.float32)
                nn.init.xavier_uniform_(w, generator=g)
                p.copy_(w)
            elif name.endswith("weight"):
                p.fill_(1.0)
            else:
                p.zero_()
    return model


def make_state_dict(cfg, seed: int) -> Dict[str, torch.Tensor]:
    """State dict of a freshly initialised stack (reference key names)."""
    from .model import LayerStack
    with torch.device("cpu"):
        m = LayerStack(cfg)
    return init_params_(m, seed).state_dict()
