"""Test configuration: the ``gpu`` marker and import paths.

``metal-kans_b200/`` holds the drop-in Python package ``metal_kans``; the repository root holds
``oracle`` (CPU checker, test infrastructure only).
"""
import os
import sys

import pytest

REPO = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
PKG_ROOT = os.path.join(REPO, "metal-kans_b200")
for p in (PKG_ROOT, REPO):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built library")


def cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this container")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_npz(name):
    import numpy as np

    with np.load(os.path.join(GOLDEN, name)) as z:
        return {k: z[k] for k in z.files}


def group(d, prefix):
    """Sub-dict of a flattened golden archive: keys 'prefix/<name>' -> '<name>'."""
    n = len(prefix) + 1
    return {k[n:]: v for k, v in d.items() if k.startswith(prefix + "/")}
