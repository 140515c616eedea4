"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; everything else runs on CPU."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libcrispembed.so")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O  # oracle/oracle.py: the CPU checker (test infrastructure)
    O.build()
    return O


@pytest.fixture(scope="session")
def tiny_model(tmp_path_factory):
    """Small NomicBERT-MoE GGUF (Q8_0 linear weights) written from a fixed seed."""
    from crispembed_b200 import synth
    p = tmp_path_factory.mktemp("models") / "tiny_q8.gguf"
    synth.write_model(str(p), synth.tiny_spec())
    return str(p)


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from crispembed_b200 import binding
    binding.load_library()  # raises when the library is missing: no silent fallback
    return torch.device("cuda:0")


def cos_rows(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return (a * b).sum(-1) / (np.linalg.norm(a, axis=-1) * np.linalg.norm(b, axis=-1))
