"""Shared pytest setup: the `gpu` marker, import paths, and session-scoped fixtures."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "eahmmf_inference_prototype_v-0.1.0_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return np.load(os.path.join(GOLDEN, name))
    return load


@pytest.fixture(scope="session")
def orc():
    import oracle
    return oracle.Oracle()


@pytest.fixture(scope="session")
def ref():
    import oracle
    if not os.path.exists(oracle.REF_SO):
        pytest.skip("oracle/_ref not built (needs the reference tree at build time)")
    return oracle.Reference(threads=min(8, os.cpu_count() or 1))


@pytest.fixture(scope="session")
def experts_c2():
    import synth
    return synth.expert_set()
