"""Shared pytest setup: the gpu marker, import paths and the oracle build."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mpp-4.1-fp4-fp8-block_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    import json
    with open(os.path.join(ROOT, "tests", "golden", "reference_kats.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def ctx():
    """libmpp41 context on cuda:0, launching on torch's current stream."""
    import torch
    import mpp41
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    c = mpp41.Context(0)
    c.set_stream(torch.cuda.current_stream().cuda_stream)
    yield c
    c.close()


def to_dev(a):
    """numpy -> CUDA tensor with the same bytes."""
    import numpy as np
    import torch
    a = np.ascontiguousarray(a)
    t = torch.from_numpy(a.view(np.uint8).reshape(-1).copy()).cuda()
    return t


def from_dev(t, dtype, shape):
    import numpy as np
    import torch
    torch.cuda.synchronize()
    n = int(np.prod(shape))
    return t.cpu().numpy().view(dtype)[:n].reshape(shape)


def empty_dev(nbytes):
    import torch
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device="cuda")
