import pathlib
import sys

import pytest
import torch

REPO = pathlib.Path(__file__).resolve().parent.parent
for path in (REPO, REPO / "refinekv-release_b200"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))

GOLDEN = REPO / "tests" / "golden" / "golden_refinekv_v0_1_2.pt"


def native_build_module():
    """The in-tree build script (refinekv-release_b200/build.py) as a module."""
    import importlib.util

    spec = importlib.util.spec_from_file_location(
        "refinekv_b200_build", REPO / "refinekv-release_b200" / "build.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU and the built native library")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    return torch.load(GOLDEN, weights_only=False)
