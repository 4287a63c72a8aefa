"""pytest configuration: the `gpu` marker and loaders for the package and the oracle.

The package directory is ``moe-680m_b200`` (not an importable name); it is loaded under the
module name ``moe680m_b200``.  The oracle (``oracle/``) is test infrastructure.
"""
import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG_DIR = ROOT / "moe-680m_b200"


def load_pkg():
    if "moe680m_b200" in sys.modules:
        return sys.modules["moe680m_b200"]
    spec = importlib.util.spec_from_file_location("moe680m_b200", PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["moe680m_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


if str(ROOT / "oracle") not in sys.path:
    sys.path.insert(0, str(ROOT / "oracle"))
if str(ROOT / "tests") not in sys.path:
    sys.path.insert(0, str(ROOT / "tests"))
load_pkg()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


@pytest.fixture(scope="session")
def pkg():
    return load_pkg()
