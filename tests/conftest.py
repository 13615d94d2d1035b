import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "clef-rs_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device (sm_100a)")


@pytest.fixture(scope="session")
def golden():
    import json

    import numpy as np
    z = np.load(ROOT / "tests" / "golden" / "backbone_fixture.npz")
    cfg = json.loads(bytes(z["config_json"]).decode())
    weights = {k[2:]: z[k] for k in z.files if k.startswith("w:")}
    return {"config": cfg, "weights": weights, "expected": z["expected_hidden"], "ids": z["ids"]}
