import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT / "fier-2bits_b200", ROOT / "oracle", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(ROOT / "tests" / "golden" / "reference_cpu.npz")


def packed_numpy(packed):
    """Device packed 4-tuple -> numpy (int32, int32, uint16 bits, uint16 bits)."""
    import numpy as np
    s, m, lo, de = (t.detach().cpu() for t in packed)
    return (s.numpy(), m.numpy(), lo.view(__import__("torch").int16).numpy().view(np.uint16),
            de.view(__import__("torch").int16).numpy().view(np.uint16))


def synthetic_keys(kvh, tokens, dim, seed, dtype):
    """N(0,1) keys with x8 outlier channels (seeded), as float32 and device dtype."""
    import torch
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(kvh, tokens, dim, generator=g)
    for h in range(kvh):
        k[h, :, torch.randperm(dim, generator=g)[:4]] *= 8.0
    k = k.to(dtype)
    return k
