import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the sm_100a kernels)")


def _load_build_module():
    import importlib.util

    spec = importlib.util.spec_from_file_location("bt_build", os.path.join(ROOT, "bigtea_b200", "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def pytest_sessionstart(session):
    # both compiled artefacts are built before any test imports them (the package refuses to
    # import without its library, so the build recipe is loaded by path)
    from oracle import pyoracle

    _load_build_module().build()
    pyoracle.build()


@pytest.fixture(scope="session")
def tiny_cfg():
    import bigtea_b200 as bt

    return bt.config("tiny")


@pytest.fixture(scope="session")
def tiny_weights(tiny_cfg):
    import bigtea_b200 as bt

    return bt.synth_model(tiny_cfg, seed=7)


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(ROOT, "tests", "golden", "kquant_golden.npz"))


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)
