"""float16 / bfloat16 I/O: the reference layer's exact arithmetic replayed
from one CUDA graph (techjam2026_b200.exact) is bit-identical to its eager
forward, and the drop-in entry takes that path at those dtypes."""
from __future__ import annotations

import pytest
import torch

from oracle import layer_stack as ls
from techjam2026_b200.configs import TransformerConfig, generate_case, make_state_dict
from techjam2026_b200.exact import ExactGraphForward

pytestmark = pytest.mark.gpu

CFG = TransformerConfig(batch_size=4, seq_len=256, d_model=256, num_heads=4, ffn_dim=1024,
                        num_layers=2, causal=True)


def _eager(params, dtype):
    def fwd(x, m):
        for i in range(CFG.num_layers):
            x = ls.block(x, params, i, CFG.num_heads, m, True, dtype)
        x = ls._layer_norm(x, params, "final_norm", dtype)
        return x.masked_fill(~m[..., None], 0) if m is not None else x
    return fwd


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_exact_graph_is_bit_identical_to_eager(dtype):
    params = {k: v.cuda().to(dtype) for k, v in make_state_dict(CFG, 0).items()}
    fwd = _eager(params, dtype)
    graph = ExactGraphForward(fwd)
    for seed in (0, 1, 2):
        x, m = generate_case(CFG, seed, 0.5)
        x, m = x.cuda().to(dtype), m.cuda()
        with torch.inference_mode():
            ref = fwd(x, m)
        got = graph(x, m)
        assert got.dtype == dtype and torch.equal(got, ref)
        assert torch.count_nonzero(got[~m]) == 0
    assert len(graph._graphs) == 1  # one capture, replayed for every input


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_submission_runs_narrow_dtypes_through_the_exact_graph(dtype, monkeypatch):
    import submission
    params = {k: v.cuda().to(dtype) for k, v in make_state_dict(CFG, 0).items()}
    fwd = _eager(params, dtype)
    monkeypatch.setattr(submission, "HAS_ORGANISER_BASELINE", True)
    monkeypatch.setattr(submission.BaselineTransformer, "forward",
                        lambda self, x, m=None: fwd(x, m), raising=False)
    ours = submission.UserOptimizedTransformer(CFG).cuda().to(dtype).eval()
    x, m = generate_case(CFG, 5, 0.5)
    x, m = x.cuda().to(dtype), m.cuda()
    got = ours(x, m)
    assert ours._plan is not None and ours._plan.exact_reference
    assert isinstance(ours._impl, ExactGraphForward) and not ours._failed
    with torch.inference_mode():
        assert torch.equal(got, fwd(x, m))
