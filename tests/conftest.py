"""Shared pytest set-up: the `gpu` marker and import paths.

Tests marked `gpu` need a CUDA device (a B200); everything else runs on the
CPU-only build container.
"""

from __future__ import annotations

import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
PKG = ROOT / "magnetar-provider-cpu_b200"
for path in (ROOT, PKG):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def _cuda_available() -> bool:
    try:
        import torch  # noqa: PLC0415

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover - torch missing
        return False


@pytest.fixture(scope="session")
def cuda_device():
    if not _cuda_available():
        pytest.skip("no CUDA device")
    return 0


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o  # noqa: PLC0415

    o.lib()
    return o
