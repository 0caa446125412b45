"""CPU oracle for the layer-stack forward -- TEST INFRASTRUCTURE ONLY.

Nothing in the product (techjam2026_b200/, submission.py) imports this
module; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline /
reference legs use it, as the checker or as the timed CPU arm.

It is a plain-PyTorch restatement, on CPU, of the reference's layer stack
(torch_transformer_benchmark.py:59-172), written against a state_dict so it
needs none of the reference's classes:

  per layer (BaselineTransformerBlock.forward, :134-145)
      x = x + MHA(LN1(x))                      (:140)
      x = x + W2 . gelu_erf(W1 . LN2(x) + b1) + b2    (:141)
      x[padded rows] = 0                       (:143-144)
  then LN_final(x) and x[padded rows] = 0      (:169-171)

  MHA (BaselineSelfAttention.forward, :86-122): separate q/k/v projections,
  scores = q k^T * Dh^-0.5, causal triu(1) -> -inf (:99-104), invalid keys
  -> -inf (:105-108), softmax in fp32 (:111), context = P v, out_proj, then
  invalid query rows -> 0 (:120-121).

Parity is pinned: tests/test_oracle.py checks this restatement against golden
outputs that tests/golden/make_golden.py produced by running the reference's
own BaselineTransformer in this container.

Differences from the reference's literal op sequence, all exact:
  * attention runs one batch element (and optionally one query chunk) at a
    time, so the [B, H, S, S] score tensor is never materialised (c4's is
    12.9 GB per layer, c5's 1.1 PB). Softmax rows are independent and no op
    mixes batch elements, so this changes no value (the reference's
    scripts/shape14.py:124-145 streams the same way; it omits the padding
    masks, which are restored here); with the causal mask a query chunk
    multiplies only the keys up to its last query, the rest being -inf
    (weight exactly 0) for every query of the chunk;
  * `dtype=torch.float64` runs the same math in double precision, used as a
    tighter reference when measuring error envelopes.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch
import torch.nn.functional as F

Params = Dict[str, torch.Tensor]


def _p(params: Params, key: str, dtype: torch.dtype) -> torch.Tensor:
    return params[key].to(dtype)


def _linear(x: torch.Tensor, params: Params, prefix: str, dtype: torch.dtype) -> torch.Tensor:
    return F.linear(x, _p(params, prefix + ".weight", dtype), _p(params, prefix + ".bias", dtype))


def _layer_norm(x: torch.Tensor, params: Params, prefix: str, dtype: torch.dtype,
                eps: float = 1e-5) -> torch.Tensor:
    return F.layer_norm(x, (x.shape[-1],), _p(params, prefix + ".weight", dtype),
                        _p(params, prefix + ".bias", dtype), eps)


def attention(h: torch.Tensor, params: Params, prefix: str, num_heads: int,
              valid_token_mask: Optional[torch.Tensor], causal: bool,
              dtype: torch.dtype = torch.float32, query_chunk: Optional[int] = None
              ) -> torch.Tensor:
    """BaselineSelfAttention.forward (torch_transformer_benchmark.py:86-122)."""
    B, S, d = h.shape
    Dh = d // num_heads
    scale = Dh ** -0.5
    q = _linear(h, params, prefix + ".q_proj", dtype)
    k = _linear(h, params, prefix + ".k_proj", dtype)
    v = _linear(h, params, prefix + ".v_proj", dtype)
    q = q.view(B, S, num_heads, Dh).transpose(1, 2)
    k = k.view(B, S, num_heads, Dh).transpose(1, 2)
    v = v.view(B, S, num_heads, Dh).transpose(1, 2)
    chunk = query_chunk or S
    ctx = torch.empty(B, num_heads, S, Dh, dtype=dtype, device=h.device)
    for b in range(B):
        kb, vb = k[b], v[b]
        key_ok = None if valid_token_mask is None else valid_token_mask[b]
        for i0 in range(0, S, chunk):
            i1 = min(S, i0 + chunk)
            # With the causal mask, keys past the chunk's last query are -inf
            # for every query of the chunk (weight exactly 0): leave them out.
            kend = i1 if causal else S
            scores = torch.matmul(q[b, :, i0:i1], kb[:, :kend].transpose(-2, -1)) * scale
            if causal:
                qi = torch.arange(i0, i1, device=h.device)[:, None]
                kj = torch.arange(kend, device=h.device)[None, :]
                scores = scores.masked_fill(kj > qi, float("-inf"))
            if key_ok is not None:
                scores = scores.masked_fill(~key_ok[None, None, :kend], float("-inf"))
            # softmax in fp32 whatever the I/O dtype (torch_transformer_benchmark.py:110-111)
            probs = torch.softmax(scores.float(), dim=-1).to(dtype)
            ctx[b, :, i0:i1] = torch.matmul(probs, vb[:, :kend])
    ctx = ctx.transpose(1, 2).reshape(B, S, d)
    out = _linear(ctx, params, prefix + ".out_proj", dtype)
    if valid_token_mask is not None:
        out = out.masked_fill(~valid_token_mask[..., None], 0)
    return out


def block(x: torch.Tensor, params: Params, i: int, num_heads: int,
          valid_token_mask: Optional[torch.Tensor], causal: bool,
          dtype: torch.dtype = torch.float32, query_chunk: Optional[int] = None
          ) -> torch.Tensor:
    """BaselineTransformerBlock.forward (torch_transformer_benchmark.py:134-145)."""
    pre = f"layers.{i}"
    x = x + attention(_layer_norm(x, params, pre + ".norm1", dtype), params, pre + ".attention",
                      num_heads, valid_token_mask, causal, dtype, query_chunk)
    hidden = F.gelu(_linear(_layer_norm(x, params, pre + ".norm2", dtype), params,
                            pre + ".ffn_in", dtype), approximate="none")
    x = x + _linear(hidden, params, pre + ".ffn_out", dtype)
    if valid_token_mask is not None:
        x = x.masked_fill(~valid_token_mask[..., None], 0)
    return x


@torch.no_grad()
def forward(params: Params, num_layers: int, num_heads: int, x: torch.Tensor,
            valid_token_mask: Optional[torch.Tensor] = None, causal: bool = True,
            dtype: torch.dtype = torch.float32, query_chunk: Optional[int] = None
            ) -> torch.Tensor:
    """BaselineTransformer.forward (torch_transformer_benchmark.py:162-172) on CPU."""
    x = x.detach().cpu().to(dtype)
    params = {k: v.detach().cpu() for k, v in params.items()}
    m = None if valid_token_mask is None else valid_token_mask.detach().cpu().bool()
    for i in range(num_layers):
        x = block(x, params, i, num_heads, m, causal, dtype, query_chunk)
    x = _layer_norm(x, params, "final_norm", dtype)
    if m is not None:
        x = x.masked_fill(~m[..., None], 0)
    return x


__all__ = ["attention", "block", "forward"]
