"""Shared pytest setup.

* Registers the ``gpu`` marker (tests that need a B200 and the built library).
* Loads the ComfyUI pack directory ``comfyui-applesilicon-optimized_b200`` as the
  package ``b200q`` (ComfyUI imports custom-node packs by directory path, so the
  directory name is not a Python identifier), without running its install-time
  bootstrap, so each test decides which seams are patched.
"""
import importlib.util
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PACK_DIR = ROOT / "comfyui-applesilicon-optimized_b200"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

os.environ.setdefault("B200Q_NO_BOOTSTRAP", "1")


def load_pack():
    mod = sys.modules.get("b200q")
    if mod is not None:
        return mod
    spec = importlib.util.spec_from_file_location(
        "b200q", PACK_DIR / "__init__.py", submodule_search_locations=[str(PACK_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["b200q"] = mod
    spec.loader.exec_module(mod)
    return mod


load_pack()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built b200q library")


@pytest.fixture(scope="session")
def native():
    """The native binding; GPU tests fail loudly if the library cannot run."""
    from b200q._patches import _native
    import torch
    assert torch.cuda.is_available(), "gpu test without a CUDA device"
    assert _native.available(), "b200q library missing or device is not sm_100"
    _native.lib()
    return _native
