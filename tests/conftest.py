"""Shared test set-up.

- registers the ``gpu`` marker (tests that need a B200; the CPU suite runs with
  ``-m "not gpu"``);
- loads the product package from ``hopper-lab_b200/`` (hyphenated directory) as
  ``hopper_lab_b200`` and the CPU oracle from ``oracle/``.
"""
import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def _load_pkg():
    if "hopper_lab_b200" in sys.modules:
        return sys.modules["hopper_lab_b200"]
    spec = importlib.util.spec_from_file_location(
        "hopper_lab_b200", ROOT / "hopper-lab_b200" / "__init__.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["hopper_lab_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


_load_pkg()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a)")


@pytest.fixture(scope="session")
def b200():
    return _load_pkg()


@pytest.fixture(scope="session")
def oracle():
    import oracle as O

    O.lib()
    return O
