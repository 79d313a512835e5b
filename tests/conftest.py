"""Test configuration: the `gpu` marker, the package loader and fixtures.

The product package lives in the directory ``jero-arch-llama_b200`` (not a
valid Python identifier); it is loaded here under the module name
``jero_arch_llama_b200``.
"""
import importlib.util
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(REPO, "jero-arch-llama_b200")
ORACLE_DIR = os.path.join(REPO, "oracle")
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def _ensure_built():
    if not os.path.exists(os.path.join(PKG_DIR, "libjal.so")):
        subprocess.run(["make", "-C", PKG_DIR, "-j8"], check=True)
    if not os.path.exists(os.path.join(ORACLE_DIR, "liboracle.so")):
        subprocess.run(["make", "-C", ORACLE_DIR], check=True)


def load_package():
    name = "jero_arch_llama_b200"
    if name in sys.modules:
        return sys.modules[name]
    _ensure_built()
    spec = importlib.util.spec_from_file_location(name, os.path.join(PKG_DIR, "__init__.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def jal():
    return load_package()


@pytest.fixture(scope="session")
def oracle():
    _ensure_built()
    import oracle_py
    return oracle_py


@pytest.fixture(scope="session")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("CUDA device not available")
    torch.cuda.init()
    return torch
