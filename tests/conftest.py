"""Shared pytest configuration.

Tests marked ``gpu`` need a CUDA device (a B200); everything else runs on a
CPU-only machine.  The repository root is put on ``sys.path`` so the tests can
import the package and the CPU oracle; an installed copy of the reference
StrideWeave (``baseline/_ref``) is added when present, for the tests that
drive the CUDA carrier through the reference's own API.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
_REF = ROOT / "baseline" / "_ref"
if _REF.is_dir() and str(_REF) not in sys.path:
    sys.path.append(str(_REF))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
