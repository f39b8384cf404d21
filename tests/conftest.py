import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def load_golden(name):
    with np.load(os.path.join(GOLDEN, name)) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def rb():
    """The product package with its CUDA library built in-tree."""
    from riallm_b200 import build as B
    B.build()
    import riallm_b200
    return riallm_b200


def device_q(rb, g, name, device="cuda"):
    """A device QuantizedTensor from golden-fixture arrays."""
    import torch
    qtype, bs, numel = [int(v) for v in g[f"{name}.qtype"]]
    data = torch.from_numpy(np.ascontiguousarray(g[f"{name}.data"])).to(device)
    return rb.QuantizedTensor(data, (numel,), rb.CompressionType(qtype),
                              torch.from_numpy(g[f"{name}.scales"]).to(device),
                              torch.from_numpy(g[f"{name}.zeros"]).to(device), bs)


def rel_err(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))
