"""Shared fixtures.

* ``pkg``     -- the product package (loaded from minicpm-o-uya_b200/, whose
                 directory name is not an identifier)
* ``O``       -- the CPU oracle (oracle/oracle.py); tests are its only users
* ``gpu_ctx`` -- a helper context on cuda:0 (GPU tests only)
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the sm_100a helper)")


def load_pkg():
    if "minicpmo_b200" in sys.modules:
        return sys.modules["minicpmo_b200"]
    pkg_dir = ROOT / "minicpm-o-uya_b200"
    spec = importlib.util.spec_from_file_location("minicpmo_b200", pkg_dir / "__init__.py",
                                                  submodule_search_locations=[str(pkg_dir)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["minicpmo_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def pkg():
    return load_pkg()


@pytest.fixture(scope="session")
def O():
    from oracle import oracle

    oracle.orc()
    return oracle


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(ROOT / "tests" / "golden" / "reference_vectors.npz"))


@pytest.fixture(scope="module")
def gpu_ctx(pkg):
    from minicpmo_b200.gpu import GpuContext

    ctx = GpuContext(0)
    yield ctx
    ctx.close()


def rel_row_err(y, ref) -> float:
    """max_i |y_i - ref_i| / ||ref||_2 (the matvec tolerance metric)."""
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(np.asarray(y, np.float64) - ref)) / max(np.linalg.norm(ref), 1e-30))
