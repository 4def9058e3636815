"""The language-core oracle, pinned to the reference (CPU only).

The C restatement (oracle/lang_oracle.c) must reproduce the reference native CPU library's
outputs bit for bit (SHA-256 recorded from oracle/_ref by tests/golden/make_lang_golden.py) and
agree with the reference PyTorch model within the reference's own parity tolerance
(atol = rtol = 3e-5, tests/test_native.py:41-47).
"""
import hashlib

import numpy as np
import pytest

from neurogen_b200.language import LanguageConfig, init_packed_weights
from oracle.lang import OracleEngine, RefEngine

SMALL = LanguageConfig(columns=3, width=17, regions=2, ticks=3, idle_steps=1, speech_width=16, mel_bins=8)


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a, np.float32).tobytes())
    return h.hexdigest()


def test_small_restatement_reproduces_reference_native_bits(golden_lang):
    g = golden_lang
    orc = OracleEngine(SMALL, g['small_weights'])
    st = np.zeros(orc.S, np.float32)
    shas = list(g['small_native_sha'])
    k = 0
    for tok in g['small_tokens']:
        lg, st, act, h = orc.step(int(tok), st)
        assert digest(lg, st, h, np.array([act], np.float32)) == shas[k], f'token step {k}'
        k += 1
    for _ in range(8):
        h, st, act = orc.advance(np.zeros(SMALL.width, np.float32), st, True)
        assert digest(st, h, np.array([act], np.float32)) == shas[k], f'idle advance {k}'
        k += 1


def test_small_restatement_matches_reference_torch_model(golden_lang):
    g = golden_lang
    orc = OracleEngine(SMALL, g['small_weights'])
    st = np.zeros(orc.S, np.float32)
    for i, tok in enumerate(g['small_tokens']):
        lg, st, act, h = orc.step(int(tok), st)
        np.testing.assert_allclose(lg, g['small_torch_logits'][i], atol=3e-5, rtol=3e-5)
        np.testing.assert_allclose(st, g['small_torch_state'][i], atol=3e-5, rtol=3e-5)
        np.testing.assert_allclose(h, g['small_torch_hidden'][i], atol=3e-5, rtol=3e-5)
        np.testing.assert_allclose(act, g['small_torch_activity'][i], atol=3e-5, rtol=3e-5)


def test_bc250_seeded_init_is_the_reference_init(golden_lang):
    w = init_packed_weights(LanguageConfig(), seed=0)
    assert w.size == 14_804_744
    assert hashlib.sha256(w.tobytes()).hexdigest() == str(golden_lang['bc250_weights_sha'])


def test_bc250_restatement_first_tokens(golden_lang):
    g = golden_lang
    cfg = LanguageConfig()
    orc = OracleEngine(cfg, init_packed_weights(cfg, seed=0))
    st = np.zeros(orc.S, np.float32)
    for i, tok in enumerate(g['bc250_tokens'][:len(g['bc250_native_sha'])]):
        lg, st, act, h = orc.step(int(tok), st)
        assert digest(lg, st, h, np.array([act], np.float32)) == str(g['bc250_native_sha'][i])


@pytest.mark.parametrize('columns,width,regions,ticks,idle', [
    (1, 1, 1, 1, 0), (2, 8, 2, 3, 1), (3, 33, 3, 2, 2), (5, 40, 2, 4, 0)])
def test_restatement_bit_identical_to_reference_library(ref_available, columns, width, regions, ticks, idle):
    if not ref_available:
        pytest.skip('reference library not built (oracle/_ref)')
    cfg = LanguageConfig(columns=columns, width=width, regions=regions, ticks=ticks, idle_steps=idle)
    rng = np.random.default_rng(columns * 1000 + width)
    w = init_packed_weights(cfg, seed=columns + width)
    w = (w + rng.normal(0, .05, w.size)).astype(np.float32)
    ref, orc = RefEngine(cfg, w), OracleEngine(cfg, w)
    sa = np.zeros(ref.S, np.float32)
    sb = sa.copy()
    for i in range(10):
        tok = int(rng.integers(0, 264))
        a, b = ref.step(tok, sa), orc.step(tok, sb)
        for x, y in zip(a, b):
            assert np.array_equal(np.asarray(x), np.asarray(y))
        sa, sb = a[1], b[1]
    x = rng.normal(0, 1, width).astype(np.float32)
    for idle_flag in (0, 1):
        a, b = ref.advance(x, sa, idle_flag), orc.advance(x, sb, idle_flag)
        for u, v in zip(a, b):
            assert np.array_equal(np.asarray(u), np.asarray(v))
        sa, sb = a[1], b[1]


def test_spike_recording_agrees_with_state(golden_lang):
    g = golden_lang
    orc = OracleEngine(SMALL, g['small_weights'])
    st = np.zeros(orc.S, np.float32)
    n = orc.n
    rs = 5 * n + SMALL.width
    for tok in g['small_tokens'][:6]:
        lg, nxt, act, h, spikes = orc.step(int(tok), st, record=True)
        per = spikes.reshape(1 + SMALL.idle_steps, SMALL.regions, SMALL.ticks, n)
        for r in range(SMALL.regions):
            last = nxt[r * rs + 3 * n: r * rs + 4 * n]
            assert np.array_equal(per[-1, r, -1], last.astype(np.uint8))
            counts = nxt[r * rs + 4 * n + SMALL.width: r * rs + 5 * n + SMALL.width]
            before = st[r * rs + 4 * n + SMALL.width: r * rs + 5 * n + SMALL.width]
            assert np.array_equal(counts - before, per[:, r].sum((0, 1)).astype(np.float32))
        assert act == pytest.approx(per.mean(), abs=1e-7)
        st = nxt


def test_oracle_seeded_weights_equal_the_packages(golden_lang):
    """The CPU legs' seeded weights (oracle/lang.py) are the reference model's seed-0 stream."""
    import hashlib
    from oracle.lang import seeded_weights
    w = seeded_weights()
    assert hashlib.sha256(w.tobytes()).hexdigest() == str(golden_lang['bc250_weights_sha'])
    small = LanguageConfig(columns=3, width=17, regions=2, ticks=3, idle_steps=1)
    assert np.array_equal(seeded_weights(3, 17, 2, 7), init_packed_weights(small, seed=7))
