import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from __graft_entry__ import load_oracle, load_package  # noqa: E402

load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a)")


@pytest.fixture(scope="session")
def pkg():
    return load_package()


@pytest.fixture(scope="session")
def oracle():
    return load_oracle()


@pytest.fixture(scope="session")
def syn():
    import importlib

    return importlib.import_module("bark3_b200.synthetic")


@pytest.fixture(scope="session")
def gpu_encoder_factory(pkg):
    made = []

    def make(weights, n_layers):
        enc = pkg.Encoder(0)
        enc.load(weights)
        enc.finalize(n_layers)
        made.append(enc)
        return enc

    yield make
    for e in made:
        e.close()


def rel_err(got, ref):
    """max |got - ref| / max |ref| (normwise relative error)."""
    import numpy as np

    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30))


def centred_err(got, ref):
    """Frame-centred normwise error: max |(got - mean frame of got) - (ref -
    mean frame of ref)| / max |ref - mean frame of ref|, the mean frame being
    the per-column mean over rows (frames).  Measures the part of a
    (frames, channels) result that differs between frames on its own scale."""
    import numpy as np

    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    g = got - got.mean(axis=0, keepdims=True)
    r = ref - ref.mean(axis=0, keepdims=True)
    return float(np.max(np.abs(g - r)) / max(np.max(np.abs(r)), 1e-30))
