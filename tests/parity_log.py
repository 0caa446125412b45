"""Parity results of the GPU tests, printed in pytest's terminal summary.

Tests call `record(what, result)` with a numerics.CheckResult; conftest's
`pytest_terminal_summary` lists every record (envelope, worst error, the
elements compared), so a quiet `pytest -q -m gpu` run still shows the
envelope of each full-size comparison."""
from __future__ import annotations

RECORDS = []


def record(what: str, result) -> None:
    RECORDS.append((what, result))
