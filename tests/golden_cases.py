"""Loader for the golden vectors produced by tests/golden/make_golden.py."""
from __future__ import annotations

import json
import os

import torch

from techjam2026_b200.configs import TransformerConfig

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASE_NAMES = ("c1", "mini_s333", "mini_dh8_noncausal", "mini_nopad", "mini_s4097")


def load_case(name: str) -> dict:
    blob = torch.load(os.path.join(GOLDEN_DIR, f"golden_{name}.pt"), weights_only=True)
    B, S, d, H, F, L, causal = blob["config"]
    blob["cfg"] = TransformerConfig(B, S, d, H, F, L, bool(causal))
    return blob


def load_inputs() -> dict:
    with open(os.path.join(GOLDEN_DIR, "golden_inputs.json"), encoding="utf-8") as f:
        return json.load(f)
