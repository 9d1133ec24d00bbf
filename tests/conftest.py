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


DIRECTIONAL_KEYS = ("route", "frontier", "candidates", "exploration", "dropped", "added")


def directional_case(golden):
    """Inputs of ``directional.npz``: the config-3 mass of two heads (plain and
    quantised to multiples of 1/28,800 so that equal scores straddle the
    budget cut), their previous route, the 720p block neighbours and the
    option sets, as ``tests/golden/make_golden.py:directional`` made them."""
    import json

    import numpy as np

    c3 = golden("config3.npz")
    lay = golden("layouts.npz")
    g = golden("directional.npz")
    mass = np.asarray(c3["mass_heads"], np.float32)
    scale = np.float32(450 * 64.0)
    quant = (np.round((mass * scale).astype(np.float32)) / scale).astype(np.float32)
    prev = unpack_route(c3["prev"], 450)[c3["heads"]]
    options = json.loads(str(g["options"]))
    return {"plain": mass, "quant": quant}, prev, lay["720p_neighbors"], options, g
