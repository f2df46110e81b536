import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    d = os.environ.get("PTQ8_MODEL_CACHE")
    if d:
        Path(d).mkdir(parents=True, exist_ok=True)
        return Path(d)
    return tmp_path_factory.mktemp("models")


_MODELS = {}


@pytest.fixture(scope="session")
def make_model(model_dir):
    """Build (once per session) a synthetic calibrated model; returns the paths dict."""
    from ptq_int8_lab_b200 import modelgen as mg

    def get(key, **kw):
        k = (key, tuple(sorted(kw.items())))
        if k not in _MODELS:
            if isinstance(key, int):
                _MODELS[k] = mg.make_config(key, model_dir, **kw)
            else:
                _MODELS[k] = mg.build_calibrated(key, out_dir=model_dir, **kw)
        return _MODELS[k]
    return get
