"""Every module of the package imports on a CPU-only host (catches syntax
errors and broken imports in modules that only GPU or multi-rank tests use)."""

import importlib
import pkgutil

import pytest

import deltaserve_vllm_b200 as pkg

MODULES = sorted(m.name for m in pkgutil.walk_packages(pkg.__path__, pkg.__name__ + "."))


@pytest.mark.parametrize("name", MODULES)
def test_module_imports(name):
    importlib.import_module(name)
