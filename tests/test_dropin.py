"""Checkpoint loading against the reference package (CPU; no engine is created).

`neurogen_b200.language.load_checkpoint` must read a `neurogen-language-v2` file written by the
reference's own `training.atomic_save` (training.py:31-45) into exactly the packed weight
stream of the reference adapter's `packed_weights` (native.py:46-52), refuse other formats, and
refuse models whose architecture buffers were edited (native.py:73-80).  Skipped when
baseline/_ref holds no reference package.
"""
import sys
from dataclasses import asdict
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
REF_PKG = ROOT / 'baseline' / '_ref'

pytestmark = pytest.mark.skipif(not (REF_PKG / 'neurogen' / 'language' / 'training.py').is_file(),
                                reason='reference package not installed in baseline/_ref')


@pytest.fixture(scope='module')
def ref():
    if str(REF_PKG) not in sys.path:
        sys.path.append(str(REF_PKG))
    from neurogen.language import config, model, native, training
    return dict(config=config, model=model, native=native, training=training)


def small_model(ref, seed=3):
    import torch
    torch.manual_seed(seed)
    cfg = ref['config'].LanguageConfig(columns=2, width=24, regions=3, ticks=2, idle_steps=1)
    return ref['model'].LanguageModel(cfg).eval()


def test_checkpoint_weights_equal_reference_packing(ref, tmp_path):
    import torch
    from neurogen_b200.language import load_checkpoint, parameter_count
    m = small_model(ref)
    path = tmp_path / 'checkpoint.pt'
    ref['training'].atomic_save({'format': ref['training'].FORMAT, 'config': asdict(m.config),
                                 'model': m.state_dict(), 'step': 3, 'history': []}, path)
    cfg, weights, payload = load_checkpoint(path)
    assert (cfg.columns, cfg.width, cfg.regions, cfg.ticks, cfg.idle_steps) == (2, 24, 3, 2, 1)
    expected = ref['native'].packed_weights(m)
    assert weights.dtype == np.float32 and np.array_equal(weights, expected)
    assert weights.size == parameter_count(cfg)
    assert payload['step'] == 3
    # The reference's own loader accepts the same file.
    m2, _ = ref['training'].load_checkpoint(path, torch.device('cpu'))
    assert np.array_equal(ref['native'].packed_weights(m2), expected)


def test_checkpoint_format_and_architecture_checks(ref, tmp_path):
    import torch
    from neurogen_b200.language import load_checkpoint
    m = small_model(ref)
    path = tmp_path / 'bio.pt'
    ref['training'].atomic_save({'format': 'neurogen-biology-v1', 'config': asdict(m.config),
                                 'model': m.state_dict()}, path)
    with pytest.raises(ValueError, match='Unsupported language checkpoint'):
        load_checkpoint(path)
    sd = m.state_dict()
    key = next(k for k in sd if k.startswith('regions.1.') and k.split('.')[-1] not in
               ('raw_weight', 'weight', 'bias', 'memory_decay'))
    sd[key] = sd[key] + 1
    path = tmp_path / 'edited.pt'
    ref['training'].atomic_save({'format': ref['training'].FORMAT, 'config': asdict(m.config), 'model': sd}, path)
    with pytest.raises(ValueError, match='architecture buffer'):
        load_checkpoint(path)
