import os
import sys

import numpy as np
import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")


@pytest.fixture(scope="session")
def oracle():
    import oracle as orc

    return orc.Oracle()


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return dict(np.load(os.path.join(GOLDEN, name + ".npz")))

    return load


@pytest.fixture(scope="session")
def ctx():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    from laguna_raw_halo_strix_b200 import lc

    torch.cuda.init()
    c = lc.Context(0)
    c.set_stream(torch.cuda.current_stream())
    yield c
    c.close()


@pytest.fixture(scope="session")
def dev():
    import torch

    return torch.device("cuda:0")


def to_dev(a, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def check_tol(got, ref, tol=1e-3, what=""):
    """max|err| <= tol * ||ref||_inf (the projection tolerance of the spec)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = max(np.abs(ref).max(), 1e-30)
    err = np.abs(got - ref).max() if ref.size else 0.0
    assert err <= tol * scale, f"{what}: max|err| {err:.3e} > {tol} * {scale:.3e}"
    return err / scale
