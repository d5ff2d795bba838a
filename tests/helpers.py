"""Shared helpers for the test-suite."""

import importlib.util
import sys

from tests.conftest import ROOT


def load_workloads():
    """Load the input generator without importing the CUDA package."""
    name = "_i8moe_workloads"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(
        name, ROOT / "int8blockwisegemm_b200" / "workloads.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod
