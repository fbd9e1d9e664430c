import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); parity tests of the CUDA path")


def load_json(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def load_npz(name):
    return np.load(os.path.join(GOLDEN, name))


@pytest.fixture(scope="session")
def trajectories():
    return load_json("trajectories.json")


@pytest.fixture(scope="session")
def cascade_trees():
    return load_json("cascade_trees.json")


def initial_pool(case):
    """Regenerates the trajectory's initial pool: make_golden.py draws it first
    from torch.Generator().manual_seed(seed), one randn per layer."""
    import torch
    g = torch.Generator().manual_seed(case["seed"])
    shape = (case["pages"], 2, case["ps"], 2, 8)
    return np.stack([torch.randn(shape, generator=g).numpy() for _ in range(2)])
