import os
import subprocess
import sys

import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(__file__))

from hypothesis import settings  # noqa: E402

settings.register_profile("default", deadline=None, max_examples=40)
settings.register_profile("thorough", deadline=None, max_examples=400)
settings.load_profile(os.environ.get("HYPOTHESIS_PROFILE", "default"))

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


@pytest.fixture(scope="session")
def probe_lib():
    """Host build of the device numerics (tests/probe/numerics_probe.cpp)."""
    import ctypes

    d = os.path.join(os.path.dirname(__file__), "probe")
    so = os.path.join(d, "libnumerics_probe.so")
    src = os.path.join(d, "numerics_probe.cpp")
    hdr = os.path.join(ROOT, "exactattention_b200", "csrc", "ea_numerics.h")
    if not os.path.exists(so) or os.path.getmtime(so) < max(os.path.getmtime(src), os.path.getmtime(hdr)):
        subprocess.run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-o", so, src], check=True)
    return ctypes.CDLL(so)


@pytest.fixture(scope="session")
def cuda_lib():
    from exactattention_b200 import _lib, build

    build.build()
    return _lib.load()
