"""Test configuration: the `gpu` marker, import paths and the checker builds.

`-m "not gpu"` runs everywhere (oracle against golden vectors, host logic, the C-ABI library
loading and exporting its symbols).  `-m gpu` tests are the parity tests proper; they call the
B200 engine through its C ABI and need an sm_100 device.
"""
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / 'neurogen-2.5_b200'
for p in (ROOT, PKG):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs an sm_100 (B200) GPU')


def _ensure_built():
    oracle = ROOT / 'oracle' / 'liboracle.so'
    if not oracle.is_file():
        subprocess.run(['make', '-C', str(ROOT / 'oracle'), 'oracle'], check=True,
                       stdout=subprocess.DEVNULL)
    lib = PKG / 'lib' / 'libneurogen_native.so'
    if not lib.is_file():
        subprocess.run(['make', '-C', str(PKG), '-j8'], check=True, stdout=subprocess.DEVNULL)


_ensure_built()


def gpu_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


@pytest.fixture(scope='session')
def golden_lang():
    import numpy as np
    return np.load(ROOT / 'tests' / 'golden' / 'lang_golden.npz')


@pytest.fixture(scope='session')
def ref_available():
    return (ROOT / 'oracle' / '_ref' / 'libneurogen_ref.so').is_file()
