"""The CPU oracle, the input generator and the weight convention, pinned
against golden vectors produced by the reference's own code
(tests/golden/make_golden.py). CPU only."""
from __future__ import annotations

import hashlib

import pytest
import torch

import oracle
from golden_cases import CASE_NAMES, load_case, load_inputs
from techjam2026_b200.configs import WORKLOADS, generate_case, make_state_dict


@pytest.mark.parametrize("name", CASE_NAMES)
def test_oracle_matches_reference_output(name):
    case = load_case(name)
    cfg = case["cfg"]
    out = oracle.forward(case["state_dict"], cfg.num_layers, cfg.num_heads, case["x"],
                         case["mask"], causal=cfg.causal)
    # Same fp32 math on the same CPU; differences are BLAS blocking only.
    assert (out - case["out"]).abs().max().item() < 2e-5


@pytest.mark.parametrize("name", CASE_NAMES)
def test_oracle_query_chunking_is_exact(name):
    case = load_case(name)
    cfg = case["cfg"]
    full = oracle.forward(case["state_dict"], cfg.num_layers, cfg.num_heads, case["x"],
                          case["mask"], causal=cfg.causal)
    chunked = oracle.forward(case["state_dict"], cfg.num_layers, cfg.num_heads, case["x"],
                             case["mask"], causal=cfg.causal, query_chunk=17)
    assert (full - chunked).abs().max().item() < 2e-5


@pytest.mark.parametrize("name", CASE_NAMES)
def test_oracle_float64_agrees(name):
    case = load_case(name)
    cfg = case["cfg"]
    o64 = oracle.forward(case["state_dict"], cfg.num_layers, cfg.num_heads, case["x"],
                         case["mask"], causal=cfg.causal, dtype=torch.float64)
    assert (o64.float() - case["out"]).abs().max().item() < 1e-4


@pytest.mark.parametrize("name", CASE_NAMES)
def test_padded_rows_are_exactly_zero_in_reference_and_oracle(name):
    case = load_case(name)
    cfg = case["cfg"]
    dead = ~case["mask"]
    assert torch.count_nonzero(case["out"][dead]) == 0
    out = oracle.forward(case["state_dict"], cfg.num_layers, cfg.num_heads, case["x"],
                         case["mask"], causal=cfg.causal)
    assert torch.count_nonzero(out[dead]) == 0


@pytest.mark.parametrize("name", CASE_NAMES)
def test_generator_reproduces_reference_draws(name):
    case = load_case(name)
    x, mask = generate_case(case["cfg"], case["seed"], case["padding_ratio"])
    assert torch.equal(x, case["x"])
    assert torch.equal(mask, case["mask"])


@pytest.mark.parametrize("name", CASE_NAMES)
def test_weight_convention_reproduces_reference_module(name):
    """Same seeded Xavier procedure on our module tree == on the reference's."""
    case = load_case(name)
    sd = make_state_dict(case["cfg"], case["seed"])
    assert list(sd.keys()) == list(case["state_dict"].keys())
    for k, v in case["state_dict"].items():
        assert torch.equal(sd[k], v), k


def test_generator_at_full_baseline_sizes():
    """Lengths and x checksums of the BASELINE configs match the reference's draws."""
    for key, want in load_inputs().items():
        wname, seed, bpart = key.split("/")
        w = WORKLOADS[wname]
        B = int(bpart[1:])
        x, mask = generate_case(w.cfg, int(seed[4:]), w.padding_ratio, w.input_scale,
                                batch_size=B)
        assert mask.sum(1).tolist() == want["lengths"], key
        assert hashlib.sha256(x.contiguous().numpy().tobytes()).hexdigest() == want["x_sha256"]


def test_length_laws_of_the_configs():
    """U[S/2, S] for padding 0.5 and U[1, S] for c4 (padding 0.9999)."""
    for w in WORKLOADS.values():
        S = w.cfg.seq_len
        lo = max(1, int(round(S * (1.0 - w.padding_ratio))))
        _, mask = generate_case(w.cfg, 0, w.padding_ratio, batch_size=2)
        lens = mask.sum(1)
        assert int(lens.min()) >= lo and int(lens.max()) <= S
    assert max(1, int(round(2048 * (1 - 0.9999)))) == 1


def test_mask_is_a_prefix_and_padded_x_is_zero():
    w = WORKLOADS["c2"]
    x, mask = generate_case(w.cfg, 1, w.padding_ratio)
    for b in range(w.cfg.batch_size):
        n = int(mask[b].sum())
        assert bool(mask[b, :n].all()) and not bool(mask[b, n:].any())
        assert torch.count_nonzero(x[b, n:]) == 0


def test_oracle_matches_reference_at_bfloat16_io():
    """bf16 I/O (the harness's --dtype bfloat16): the reference module cast to
    bf16 on bf16 inputs. The oracle restates the same ops in the same order
    (softmax in fp32, every other result rounded to bf16)."""
    case = load_case("mini_bf16")
    cfg = case["cfg"]
    assert case["dtype"] == "bfloat16" and case["x"].dtype == torch.bfloat16
    out = oracle.forward(case["state_dict"], cfg.num_layers, cfg.num_heads, case["x"],
                         case["mask"], causal=cfg.causal, dtype=torch.bfloat16)
    assert out.dtype == torch.bfloat16
    diff = (out.float() - case["out"].float()).abs().max().item()
    # Same CPU ops in the same order; a bf16 ulp at |x| ~ 4 is 2^-5.
    assert diff <= 2 ** -5, diff
    assert torch.count_nonzero(out[~case["mask"]]) == 0


@pytest.mark.parametrize("name", ["mini_s333", "mini_s4097"])
def test_oracle_on_a_valid_prefix_equals_the_padded_row(name):
    """The full-size parity tests run the oracle on each row's valid prefix
    only (c4, c5): with a prefix mask that reproduces the padded row's valid
    outputs, since no valid output depends on a padded token. Pinned here
    against the reference's own outputs of whole padded rows."""
    case = load_case(name)
    cfg, x, mask = case["cfg"], case["x"], case["mask"]
    for b in range(x.shape[0]):
        n = int(mask[b].sum())
        assert bool(mask[b, :n].all()) and not bool(mask[b, n:].any())
        part = oracle.forward(case["state_dict"], cfg.num_layers, cfg.num_heads,
                              x[b:b + 1, :n], mask[b:b + 1, :n], causal=cfg.causal,
                              query_chunk=256)
        torch.testing.assert_close(part[0], case["out"][b, :n], rtol=2e-5, atol=2e-5)
