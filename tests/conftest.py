import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "golden.npz"
SMALL = dict(n_layer=2, n_tokens=16)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def small_models(tmp_path_factory):
    """Small synthetic Q8_0 / Q4_K models (2 layers, 17 tokens) -- the golden fixtures' models."""
    from edge_maskgit_b200 import synth
    d = tmp_path_factory.mktemp("models")
    out = {}
    for q in ("gq8", "gq4"):
        spec = synth.ModelSpec(quant=q, **SMALL)
        out[q] = (synth.make_model(d / f"{q}.gguf", spec), spec)
    return out


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


# tier tolerances of verification/compare_intermediates.py:77-85 and the logit gate of
# tools/verify-opencl-transformer.cpp:98-101
TIERS = {"f32": (2e-2, 0.99999), "q8": (1.0, 0.9999), "q4": (2.0, 0.99)}
