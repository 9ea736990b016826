import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
if GOLDEN not in sys.path:
    sys.path.insert(0, GOLDEN)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def plumbing():
    """(X, Q, expected dists, expected ids) of the plumbing workload, k=10."""
    from gpu_algo_b200 import data
    X, Q = data.workload_arrays("plumbing")
    g = np.load(os.path.join(GOLDEN, "plumbing_k10.npz"))
    return X, Q, g["dists"], g["ids"]


@pytest.fixture(scope="session")
def edges():
    """name -> (Q, X, k, expected dists, expected ids)."""
    from make_golden import edge_cases
    g = np.load(os.path.join(GOLDEN, "edges.npz"))
    return {name: (Q, X, k, g[f"{name}.dists"], g[f"{name}.ids"])
            for name, (Q, X, k) in edge_cases().items()}
