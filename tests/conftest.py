import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def golden_geometry(z) -> dict:
    """Frame geometry of a golden fixture (``PesqLoss`` keyword arguments);
    empty for the default n_fft 512 / hop 256 / window 512."""

    keys = ("n_fft", "hop_length", "win_length")
    return {k: int(z[k]) for k in keys if k in z.files}


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built extension")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
