import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    cache = {}

    def load(name):
        if name not in cache:
            path = GOLDEN / name
            if name.endswith(".json"):
                import json
                cache[name] = json.loads(path.read_text())
            else:
                cache[name] = dict(np.load(path, allow_pickle=False))
        return cache[name]

    return load


def sha256_tensor(t):
    import hashlib
    import torch

    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def unpack_route(bits, cols):
    import numpy as np

    return np.unpackbits(bits, axis=-1, count=cols).astype(bool)
