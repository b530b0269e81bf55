"""Test configuration: import paths and the `gpu` marker.

The package directory is put on sys.path the way the reference configures pytest
(pythonpath = ["src"], pyproject.toml:30-32), so tests import `decode_state`, `paged_kv_ops`, ...
as top-level modules, like the reference's own tests do.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for path in (ROOT / "qwen3.6-2080ti_b200", ROOT, ROOT / "tests" / "golden"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built native library")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
