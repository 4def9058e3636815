"""Drop-in proof: the reference's own Python adapter and checkpoint format drive this library.

The reference package (installed offline into baseline/_ref by
`pip install --no-index --no-deps --target baseline/_ref <reference checkout>`) is imported
unchanged.  Its ctypes adapter `neurogen.language.native` loads whatever
NEUROGEN_NATIVE_LIBRARY names, so pointing that variable at libneurogen_native.so and asking
for the `native-cuda` device runs the reference's `NativeLanguageModel` -- its own argtypes, its
per-item `ng_step`/`ng_advance` loop and its state packing -- on the B200 engine.  The
assertions restate those of the reference's parity test (tests/test_native.py:49-69, 71-90,
92-113): outputs and every state field within atol = rtol = 3e-5 of the independent PyTorch
model, caller-owned states never mutated, sessions saved by one backend resumed on the other,
the sequence and audio front ends, and two threads sharing one handle.

The checkpoint test writes a `neurogen-language-v2` file with the reference's own
`training.atomic_save` (training.py:31-45, the payload keys of training.py:215-221) and loads it
with this package's `NativeLanguageModel.from_checkpoint`; the result is compared with the
reference's native CPU library on the same weights.

Skipped when baseline/_ref holds no reference package.
"""
import copy
import sys
from concurrent.futures import ThreadPoolExecutor
from dataclasses import asdict
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
REF_PKG = ROOT / 'baseline' / '_ref'
LIB = ROOT / 'neurogen-2.5_b200' / 'lib' / 'libneurogen_native.so'

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not (REF_PKG / 'neurogen' / 'language' / 'native.py').is_file(),
                                 reason='reference package not installed in baseline/_ref')]


@pytest.fixture(scope='module')
def ref(tmp_path_factory):
    """The reference package's language modules, with its adapter pointed at this library."""
    import os
    os.environ['NEUROGEN_NATIVE_LIBRARY'] = str(LIB)
    if str(REF_PKG) not in sys.path:
        sys.path.append(str(REF_PKG))
    import torch
    from neurogen.language import config, model, native, runtime, training
    torch.set_num_threads(1)
    return dict(config=config, model=model, native=native, runtime=runtime, training=training)


def pair(ref, seed=7, columns=3, width=17):
    """(PyTorch model, the same model on native-cuda), with non-uniform recurrent weights."""
    import torch
    torch.manual_seed(seed)
    cfg = ref['config'].LanguageConfig(columns=columns, width=width, regions=2, ticks=3, idle_steps=1,
                                       speech_width=16, mel_bins=8)
    torch_model = ref['model'].LanguageModel(cfg).eval()
    with torch.no_grad():
        for region in torch_model.regions:
            region.raw_weight.add_(torch.randn_like(region.raw_weight) * .3)
    native = ref['native'].NativeLanguageModel.from_model(copy.deepcopy(torch_model), 'native-cuda')
    return torch_model, native


def same(a, b, atol=3e-5):
    import torch
    if isinstance(a, (tuple, list)):
        assert len(a) == len(b)
        for x, y in zip(a, b):
            same(x, y, atol)
    else:
        torch.testing.assert_close(a, b, atol=atol, rtol=3e-5)


def test_reference_adapter_runs_on_this_library(ref):
    _, native = pair(ref)
    assert native.native_backend.startswith('cuda')
    assert Path(native._native_lib._name).resolve() == LIB.resolve()


@pytest.mark.parametrize('seed,columns,width', [(7, 3, 17), (11, 1, 1)])
def test_tokens_idle_batch_and_full_state(ref, seed, columns, width):
    """Batch 2: 24 tokens then 8 idle advances; every output and state field within 3e-5 of the
    PyTorch model; the caller's previous state is left untouched."""
    import torch
    torch_model, native = pair(ref, seed, columns, width)
    with torch.no_grad():
        a = b = None
        for i in range(24):
            token = torch.tensor([257 if i == 0 else i, 100 + i])
            ra, rb = torch_model.step(token, a), native.step(token, b)
            same(ra, rb)
            a, b = ra[1], rb[1]
        previous = b
        original = tuple(tuple(x.clone() for x in r) for r in b)
        for _ in range(8):
            ra = torch_model.advance(torch.zeros(2, width), a, idle=True)
            rb = native.advance(torch.zeros(2, width), b, idle=True)
            same(ra, rb)
            a, b = ra[1], rb[1]
        same(previous, original)
        assert any(bool(x.any()) for region in b for x in region)


def test_session_cross_backend_resume(ref, tmp_path):
    """A reference Session on the PyTorch model and one on native-cuda hear the same text, save
    and resume each other's session files, and stay within 3e-5; a third session on the same
    handle does not disturb the second."""
    Session = ref['runtime'].Session
    torch_model, native = pair(ref)
    a, b = Session(torch_model), Session(native)
    a.hear_text('hello')
    b.hear_text('hello')
    same(a.state, b.state)
    path = tmp_path / 'session.pt'
    a.save(path, 'same-weights')
    b.load(path, 'same-weights')
    a.idle(4)
    b.idle(4)
    same(a.state, b.state)
    b.save(path, 'same-weights')
    a.load(path, 'same-weights')
    same(a.feed([42]), b.feed([42]))
    other = Session(native)
    before = tuple(tuple(x.clone() for x in r) for r in b.state)
    other.feed([10, 11, 12])
    same(b.state, before)


def test_sequence_and_audio_front_ends(ref):
    import torch
    torch_model, native = pair(ref)
    with torch.no_grad():
        tokens = torch.tensor([[257, 65, 66]])
        same(torch_model(tokens), native(tokens))
        features = torch.rand(1, 3, 8)
        same(torch_model.listen(features), native.listen(features))
        ha, hb = torch_model(tokens)[3], native(tokens)[3]
        same(torch_model.acoustic_decode(features, ha), native.acoustic_decode(features, hb))


def test_shared_handle_threads(ref):
    import torch
    _, native = pair(ref)

    def run(token):
        with torch.no_grad():
            return native(torch.tensor([[257, token, token]]))

    expected = [run(10), run(20)]
    with ThreadPoolExecutor(max_workers=2) as ex:
        actual = list(ex.map(run, [10, 20]))
    same(expected, actual)


def test_inference_only_and_invalid_tokens(ref):
    import torch
    _, native = pair(ref)
    with pytest.raises(ValueError, match='inference-only'):
        native.train()
    with pytest.raises(ValueError):
        native.step(torch.tensor([-1]))


def test_checkpoint_written_by_reference_training(ref, tmp_path):
    """neurogen-language-v2 file from the reference's atomic_save -> this package's
    NativeLanguageModel.from_checkpoint -> token steps equal to the reference native CPU library
    on the same weights (state 1e-5, logits 1e-4 relative, spikes exact)."""
    import torch
    from neurogen_b200.language import NativeLanguageModel, load_checkpoint
    from oracle.lang import RefEngine
    torch_model, _ = pair(ref, seed=3, columns=4, width=32)
    path = tmp_path / 'checkpoint.pt'
    opt = torch.optim.Adam(torch_model.parameters(), lr=1e-3)
    ref['training'].atomic_save({'format': ref['training'].FORMAT, 'config': asdict(torch_model.config),
                                 'model': torch_model.state_dict(), 'optimizer': opt.state_dict(), 'step': 0,
                                 'settings': {}, 'data_hashes': {}, 'data_source': 'synthetic',
                                 'sampler_rng': torch.get_rng_state(), 'torch_rng': torch.get_rng_state(),
                                 'gpu_rng': [], 'history': [], 'speech_trained': False, 'source_sha256': ''},
                                path)
    cfg, weights, _ = load_checkpoint(path)
    assert np.array_equal(weights, ref['native'].packed_weights(torch_model))
    model = NativeLanguageModel.from_checkpoint(path)
    engine = RefEngine(cfg, weights)
    s = np.zeros(engine.S, np.float32)
    state = None
    with torch.no_grad():
        for tok in (257, 72, 101, 108, 108, 111, 33, 10):
            logits, state, act, hidden = model.step(torch.tensor([tok]), state)
            lr, s, ar, hr = engine.step(tok, s)
            got = model.pack_state(state, 1)[0]
            np.testing.assert_allclose(logits[0].numpy(), lr, rtol=1e-4, atol=1e-6)
            np.testing.assert_allclose(got, s, rtol=1e-5, atol=1e-6)
            n = cfg.columns * 64
            rs = 5 * n + cfg.width
            for r in range(cfg.regions):
                assert np.array_equal(got[r * rs + 3 * n:r * rs + 4 * n], s[r * rs + 3 * n:r * rs + 4 * n])


def test_from_model_with_the_reference_torch_model(ref):
    """This package's NativeLanguageModel.from_model on the reference's own LanguageModel: same
    outputs as the PyTorch model within 3e-5; a model whose architecture buffers were edited is
    refused (reference native.py:73-80)."""
    import torch
    from neurogen_b200.language import NativeLanguageModel
    torch_model, _ = pair(ref, seed=5)
    mine = NativeLanguageModel.from_model(copy.deepcopy(torch_model))
    with torch.no_grad():
        a = b = None
        for i in range(12):
            token = torch.tensor([257 if i == 0 else 40 + i, 7 * i])
            ra, rb = torch_model.step(token, a), mine.step(token, b)
            same(ra, rb)
            a, b = ra[1], rb[1]
    bad = copy.deepcopy(torch_model)
    name, buf = next(iter(bad.regions[0].named_buffers()))
    with torch.no_grad():
        buf.add_(1)
    with pytest.raises(ValueError, match='architecture buffer'):
        NativeLanguageModel.from_model(bad)
