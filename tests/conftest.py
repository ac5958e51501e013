"""Shared pytest setup: the plugin directory is put on sys.path (it is bind-mounted into site-packages in a
vLLM deployment, so its modules import as top-level `fp4x_kernels` / `fp4patch`), and the `gpu` marker is
registered."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PLUGIN_DIR = os.path.join(ROOT, "qwen3.8-flash-next-fp4-local-spark_b200")
for p in (ROOT, PLUGIN_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)
