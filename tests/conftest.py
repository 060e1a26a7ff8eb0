"""Shared test configuration: path setup and the ``gpu`` marker."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PACKAGE = ROOT / "composable-kernel-language_b200" / "python"
for path in (str(ROOT), str(PACKAGE)):
    if path not in sys.path:
        sys.path.insert(0, path)

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
