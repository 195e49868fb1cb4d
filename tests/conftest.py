"""pytest set-up: the `gpu` marker (tests that need a B200) and import paths for the engine's
ctypes binding (animejanai-inference_b200/ajib.py) and the test helpers."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "animejanai-inference_b200"))
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
