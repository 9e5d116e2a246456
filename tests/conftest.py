"""Test configuration: the ``gpu`` marker (tests that need a B200) and import paths.

The CPU suite (``-m "not gpu"``) covers the oracle against the golden fixtures, the host-side logic of the
Python shim and that the C-ABI library loads and exports every symbol ``include/whisper_attn_b200.h`` declares.
The GPU suite (``-m gpu``) runs the CUDA kernels through the C-ABI against the oracle.
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "whisper-trt_b200", ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def attn_golden():
    import numpy as np

    return np.load(ROOT / "tests" / "golden" / "attn_golden.npz")


@pytest.fixture(scope="session")
def scores_golden():
    import numpy as np

    return np.load(ROOT / "tests" / "golden" / "scores_golden.npz")


@pytest.fixture(scope="session")
def slots_golden():
    import numpy as np

    return np.load(ROOT / "tests" / "golden" / "slots_golden.npz")


@pytest.fixture(scope="session")
def decoder_golden():
    import numpy as np

    return np.load(ROOT / "tests" / "golden" / "decoder_golden.npz")


@pytest.fixture(scope="session")
def mixed_golden():
    import numpy as np

    return np.load(ROOT / "tests" / "golden" / "mixed_golden.npz")
