import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, GOLDEN):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (runs the sm_100a kernels)")


@pytest.fixture(scope="session")
def tiny_model(tmp_path_factory):
    """The tiny Llama GGUF (seed 0) and its 16-token prompt."""
    import make_tiny_llama
    path = str(tmp_path_factory.mktemp("model") / "tiny.gguf")
    prompt = make_tiny_llama.write_model(path, 0)
    return path, prompt


@pytest.fixture(scope="session")
def golden_e2e():
    import numpy as np
    return dict(np.load(os.path.join(GOLDEN, "tiny_e2e_seed0.npz")))


@pytest.fixture(scope="session")
def golden_kats():
    import numpy as np
    return dict(np.load(os.path.join(GOLDEN, "attn_block_kats.npz")))
