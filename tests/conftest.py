"""pytest setup: the `gpu` marker, import paths for the package
(mormot2-qwen-tts_b200/qtts.py, synth.py), the oracle (test infrastructure)
and the golden helpers."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mormot2-qwen-tts_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def device():
    import qtts
    d = qtts.QwenDevice(0)
    yield d
    d.close()
