"""Test configuration.

Marker `gpu`: needs a CUDA device (B200).  Everything else runs on CPU:
    python -m pytest tests -m "not gpu"      # oracle, golden vectors, C-ABI surface, host logic, gloo ranks
    python -m pytest tests -m gpu            # parity of the CUDA kernels against the oracle
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "dflash-swift_b200"
for p in (str(ROOT), str(ROOT / "oracle"), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on the B200 box)")
    config.addinivalue_line(
        "markers", "unconfirmed: code whose GPU run has not yet been seen to pass on a B200; such tests are "
                   "collected after all others, so a run stopping at its first failure has run every confirmed test")


def pytest_collection_modifyitems(session, config, items):
    # stable sort, order kept otherwise: unconfirmed tests after the confirmed ones, and the
    # allocation-free entry point's file after everything
    items.sort(key=lambda item: (item.fspath.basename == "test_zz_no_alloc.py",
                                 item.get_closest_marker("unconfirmed") is not None))


def _ensure_built():
    so = PKG / "libdflashcuda.so"
    oracle_so = ROOT / "oracle" / "liboracle.so"
    if not so.exists() or not oracle_so.exists():
        spec = importlib.util.spec_from_file_location("graft_entry", ROOT / "__graft_entry__.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()


_ensure_built()


@pytest.fixture(scope="session")
def dc():
    import dflashcuda
    return dflashcuda


@pytest.fixture(scope="session")
def O():
    import oracle
    return oracle


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    return torch.device("cuda:0")
