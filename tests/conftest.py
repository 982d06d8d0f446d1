import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (run on a B200 with `-m gpu`)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(os.path.join(ROOT, "tests", "golden", "hf_qwen35_small.npz"))


@pytest.fixture(scope="session")
def small_model():
    """Seeded 8-layer / 2048-vocab model of the architecture: (state dict, oracle) per norm_init."""
    from oracle import qwen35_oracle as O
    cache = {}

    def get(norm_init="unit", rounding="decode"):
        key = (norm_init, rounding)
        if key not in cache:
            sd = cache.get(("sd", norm_init)) or O.init_weights(0, 8, 2048, norm_init=norm_init)
            cache[("sd", norm_init)] = sd
            cache[key] = (sd, O.Oracle(sd, rounding=rounding))
        return cache[key]
    return get
