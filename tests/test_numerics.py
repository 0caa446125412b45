"""The accuracy gate restates the organiser's compare_outputs rule
(torch_transformer_benchmark.py:289-356). CPU only."""
from __future__ import annotations

import torch

from techjam2026_b200.numerics import ATOL, RTOL, check, padded_rows_exactly_zero


def test_gate_constants_are_the_scripts_defaults():
    assert (ATOL, RTOL) == (2e-3, 2e-2)


def test_or_rule_not_and():
    ref = torch.tensor([1.0, 0.0, 100.0])
    # 1.5e-2 abs on |ref|=1: fails atol, passes rtol (2e-2)
    # 1.9e-3 abs on 0: passes atol
    # 1.9 abs on 100: passes rtol
    opt = ref + torch.tensor([1.5e-2, 1.9e-3, 1.9])
    assert check(ref, opt).passed


def test_stricter_than_isclose():
    ref = torch.tensor([0.05])
    opt = ref + 2.5e-3           # isclose: 2e-3 + 1e-3 allowed; gate: max(2e-3, 1e-3)
    assert torch.isclose(opt, ref, rtol=RTOL, atol=ATOL).all()
    assert not check(ref, opt).passed


def test_nan_and_inf_fail():
    ref = torch.zeros(4)
    assert not check(ref, torch.tensor([0.0, float("nan"), 0.0, 0.0])).passed
    assert not check(ref, torch.tensor([0.0, 0.0, float("inf"), 0.0])).passed


def test_shape_mismatch_fails():
    r = check(torch.zeros(2, 3), torch.zeros(3, 2))
    assert not r.passed and "shape" in r.note


def test_envelope_utilisation():
    ref = torch.tensor([1.0, 10.0])
    opt = ref + torch.tensor([1e-3, 0.1])   # 1e-3/2e-2 = 0.05 ; 0.1/0.2 = 0.5
    r = check(ref, opt)
    assert abs(r.envelope_utilization - 0.5) < 1e-4 and r.passed


def test_gate_agrees_with_elementwise_rule_on_random_cases():
    g = torch.Generator().manual_seed(0)
    for _ in range(50):
        ref = torch.randn(64, generator=g)
        opt = ref + torch.randn(64, generator=g) * 3e-3
        err = (opt - ref).abs()
        want = bool(((err <= ATOL) | (err <= RTOL * ref.abs())).all())
        assert check(ref, opt).passed == want


def test_padded_rows_exactly_zero_helper():
    out = torch.ones(2, 3, 4)
    mask = torch.tensor([[1, 1, 0], [1, 0, 0]], dtype=torch.bool)
    out[~mask] = 0.0
    assert padded_rows_exactly_zero(out, mask)
    out[1, 2, 0] = 1e-30
    assert not padded_rows_exactly_zero(out, mask)
