import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "ggml-rocket_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import ggml_b200
    ggml_b200.lib()   # fails loudly if the library is not built
    return torch.device("cuda:0")


def rel_err(got, ref):
    """max |got - ref| / max |ref| -- the north star's 'max relative error' with the
    near-zero guard: the denominator is the tensor's largest reference magnitude."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.max(np.abs(ref))
    return float(np.max(np.abs(got - ref)) / (den if den > 0 else 1.0))


def rk_compare(ref, got):
    """The reference's element rule (test-common.h:102-129): an element is bad only if it misses
    BOTH |d| < 0.5 and rel < 0.05; any non-finite element is bad. Returns (cosine, n_bad)."""
    ref = np.asarray(ref, dtype=np.float64).ravel()
    got = np.asarray(got, dtype=np.float64).ravel()
    fin = np.isfinite(got)
    bad = int(np.sum(~fin))
    r, g = ref[fin], got[fin]
    ad = np.abs(g - r)
    rd = ad / (np.abs(r) + 1e-6)
    bad += int(np.sum((ad >= 0.5) & (rd >= 0.05)))
    na, nb = np.sqrt(np.sum(r * r)), np.sqrt(np.sum(g * g))
    cos = float(np.dot(r, g) / (na * nb)) if na > 0 and nb > 0 else 0.0
    return cos, bad
