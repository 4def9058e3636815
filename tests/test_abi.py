"""The C-ABI library: loads, exports every declared symbol, validates like the reference.

Runs without a GPU.  No compute call is made here; creation on a machine without an sm_100
device must fail loudly (no CPU fallback).
"""
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import gpu_available
from neurogen_b200 import EXPORTS, library, library_path
from neurogen_b200.language import LanguageConfig, parameter_count, init_packed_weights

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for header in (ROOT / 'include').glob('*.h'):
        text = re.sub(r'/\*.*?\*/', '', header.read_text(), flags=re.S)
        names |= set(re.findall(r'\b(ng_[a-z_]+)\s*\(', text))
    return names


def test_every_declared_symbol_is_exported():
    lib = library()
    declared = declared_symbols()
    assert declared == set(EXPORTS)
    out = subprocess.run(['nm', '-D', '--defined-only', str(library_path())], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r' T (ng_\w+)', out))
    assert declared <= exported, declared - exported
    for name in declared:
        getattr(lib, name)


def test_library_is_sm100a_only():
    out = subprocess.run(['cuobjdump', '--list-elf', str(library_path())], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip('cuobjdump unavailable')
    arches = set(re.findall(r'sm_(\d+a?)', out.stdout))
    assert arches == {'100a'}, arches


@pytest.mark.parametrize('cfg', [LanguageConfig(), LanguageConfig(columns=3, width=17, regions=2),
                                 LanguageConfig(columns=1, width=1, regions=1)])
def test_parameter_count_matches_packed_stream(cfg):
    lib = library()
    n = lib.ng_parameter_count(cfg.columns, cfg.width, cfg.regions)
    assert n == parameter_count(cfg) == init_packed_weights(cfg, seed=1).size


def create(cfg, w, backend=b'cuda'):
    lib = library()
    return lib.ng_create(cfg.columns, cfg.width, cfg.regions, cfg.ticks, cfg.idle_steps, w, w.size, backend)


def test_validation_errors_match_reference_messages():
    lib = library()
    cfg = LanguageConfig(columns=2, width=8, regions=2, ticks=3, idle_steps=1)
    w = init_packed_weights(cfg, seed=0)
    bad = LanguageConfig(columns=2, width=8, regions=2, ticks=3, idle_steps=1)
    assert not lib.ng_create(0, 8, 2, 3, 1, w, w.size, b'cuda')
    assert lib.ng_error().decode() == 'Invalid native model dimensions'
    assert not lib.ng_create(2, 8, 2, 3, 17, w, w.size, b'cuda')
    assert lib.ng_error().decode() == 'Invalid native model dimensions'
    assert not create(bad, w[:-1].copy())
    assert lib.ng_error().decode() == 'Native weight count does not match architecture'
    wn = w.copy()
    wn[5] = np.nan
    assert not create(bad, wn)
    assert lib.ng_error().decode() == 'Non-finite weights'
    assert not create(bad, w, b'cpu')
    assert 'unavailable' in lib.ng_error().decode() and 'no silent fallback' in lib.ng_error().decode()
    assert lib.ng_backend(None) == b'invalid'


def test_null_handles_are_rejected():
    lib = library()
    s = np.zeros(4, np.float32)
    assert lib.ng_step(None, 1, s, 4, s, s, s, s) == -1
    assert lib.ng_error().decode() == 'Null native engine'
    assert lib.ng_advance(None, s, s, 4, 0, s, s, s) == -1
    assert lib.ng_error().decode() == 'Null native engine'


@pytest.mark.skipif(gpu_available(), reason='checks the no-GPU failure path')
def test_no_gpu_fails_loudly():
    lib = library()
    cfg = LanguageConfig(columns=1, width=4, regions=1)
    w = init_packed_weights(cfg, seed=0)
    assert not create(cfg, w)
    msg = lib.ng_error().decode()
    assert 'CUDA' in msg or 'sm_100' in msg


@pytest.mark.skipif(gpu_available(), reason='checks the no-GPU failure path')
def test_no_gpu_network_fails_loudly():
    """The network engine has no CPU path either: creating a network, or one from an edge list,
    without an sm_100 device fails with a message and no handle."""
    from neurogen_b200.network import Network, default_config
    cfg = default_config(n=64, n_exc=51)
    with pytest.raises(ValueError, match='CUDA|sm_100'):
        Network(cfg)
    edges = (np.array([0, 1]), np.array([1, 2]), np.array([1, 2]), np.array([0.5, 0.25]))
    with pytest.raises(ValueError, match='CUDA|sm_100'):
        Network(cfg, edges)
