"""Pytest configuration: the `gpu` marker and shared helpers."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "golden.pt"


def reference_root() -> Path | None:
    """Where the reference package ``tasft`` can be imported from: ``$TASFT_REFERENCE``
    (a checkout), else ``baseline/_ref`` (the reference installed beside this repo, which
    travels with it). None when neither holds it; tests that need it then skip."""
    import os  # noqa: PLC0415

    for cand in (os.environ.get("TASFT_REFERENCE"), ROOT / "baseline" / "_ref"):
        if cand and (Path(cand) / "tasft" / "__init__.py").exists():
            return Path(cand)
    return None


def import_reference() -> Path:
    root = reference_root()
    if root is None:
        pytest.skip("reference package not available (set TASFT_REFERENCE or install baseline/_ref)")
    if str(root) not in sys.path:
        sys.path.insert(0, str(root))
    return root


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    return torch.load(GOLDEN, weights_only=False)
