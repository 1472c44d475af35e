"""Shared fixtures. `gpu` tests need a CUDA device and the built liblfm3attn.so; the rest run on CPU."""
import importlib.util
import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
PKG = ROOT / "lfm3-1.7b-mi50_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built CUDA library")


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle as o

    o.lib()
    return o


@pytest.fixture(scope="session")
def la():
    import lfm3attn

    lfm3attn.lib()
    return lfm3attn


@pytest.fixture(scope="session")
def synth():
    import synth as s

    return s


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
