import importlib.util
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")
PKG_ROOT = os.path.join(REPO, "pi05-infer_b200")
if PKG_ROOT not in sys.path:
    sys.path.insert(0, PKG_ROOT)
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


def load_oracle():
    """Import ``oracle/pi05_oracle.py`` (test infrastructure; the checker only)."""
    name = "pi05_oracle"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(REPO, "oracle", "pi05_oracle.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def has_gpu():
    try:
        import torch

        return torch.cuda.is_available() and torch.cuda.get_device_capability(0)[0] == 10
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if has_gpu():
        return
    skip = pytest.mark.skip(reason="no sm_100 GPU in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_ref_loader():
    """Import ``baseline/ref_loader.py`` (loads files of the reference installed under
    ``baseline/_ref``); None when the reference is not installed there."""
    name = "pi05_ref_loader"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(name, os.path.join(REPO, "baseline", "ref_loader.py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    mod = sys.modules[name]
    return mod if mod.available() else None
