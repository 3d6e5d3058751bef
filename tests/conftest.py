"""Shared pytest setup: the `gpu` marker, repo paths and package loading."""
import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "omeinsum-rs_b200")
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def load_pkg():
    """Import the host package (directory omeinsum-rs_b200/) as `omeinsum_b200`."""
    if "omeinsum_b200" in sys.modules:
        return sys.modules["omeinsum_b200"]
    spec = importlib.util.spec_from_file_location(
        "omeinsum_b200", os.path.join(PKG_DIR, "__init__.py"),
        submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["omeinsum_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
