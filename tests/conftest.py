"""Shared pytest setup.

Markers: ``gpu`` -- needs a CUDA device (run with ``-m gpu`` on a B200);
everything else runs on CPU.  The oracle under ``oracle/`` is the checker
only; the GPU tests call the library through its C ABI.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG_DIR = ROOT / "luisacompute-parallelprimitive_b200"
GOLDEN = ROOT / "tests" / "golden"
for p in (str(ROOT), str(PKG_DIR)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


class Golden:
    """Fixture arrays (golden.npz) and digests of large expected outputs (manifest.json)."""

    def __init__(self):
        self.arrays = dict(np.load(GOLDEN / "golden.npz"))
        self.manifest = json.loads((GOLDEN / "manifest.json").read_text())

    def __getitem__(self, name):
        return self.arrays[name]

    def has(self, name):
        return name in self.arrays

    def matches(self, name, actual: np.ndarray) -> bool:
        """True when `actual` equals the expected array (stored or by SHA-256 digest)."""
        import hashlib
        meta = self.manifest[name]
        a = np.ascontiguousarray(actual)
        if a.size != meta["count"]:
            return False
        if name in self.arrays:
            return np.array_equal(a.view(np.uint8), self.arrays[name].view(np.uint8))
        return hashlib.sha256(a.astype(a.dtype.newbyteorder("<")).tobytes()).hexdigest() == meta["sha256"]


@pytest.fixture(scope="session")
def golden():
    return Golden()


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o
    o.build()
    return o


@pytest.fixture(scope="session")
def lcpp():
    import lcpp_b200
    lcpp_b200.lib()
    return lcpp_b200
