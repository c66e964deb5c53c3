"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; everything else runs on CPU."""
import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this container")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def oracle():
    import oracle as O  # oracle/oracle.py (test infrastructure)
    O.lib()
    return O


@pytest.fixture(scope="session")
def golden_chain():
    with open(os.path.join(GOLDEN, "prime_chain_n17_d44_s59_f60_dnum4.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def ntt_kat():
    return dict(np.load(os.path.join(GOLDEN, "ntt_kat_n1024.npz")))


MASK = (1 << 64) - 1


def mix(x: int) -> int:
    """splitmix64 finaliser used by the reference NTT probe's input patterns."""
    x = (x + 0x9E3779B97F4A7C15) & MASK
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & MASK
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & MASK
    return x ^ (x >> 31)


def probe_values(n, q, pattern, salt):
    """Input patterns of the reference NTT probe: zero, q-1, alternating, mixed."""
    if pattern == 0:
        return np.zeros(n, dtype=np.uint64)
    if pattern == 1:
        return np.full(n, q - 1, dtype=np.uint64)
    if pattern == 2:
        v = np.zeros(n, dtype=np.uint64)
        v[1::2] = q - 1
        return v
    rng = np.random.default_rng(salt)
    return (rng.integers(0, 2**63, size=n, dtype=np.uint64) * np.uint64(2)
            + rng.integers(0, 2, size=n, dtype=np.uint64)) % np.uint64(q)
