"""GPU parity of the language core against the reference's own native CPU library.

Bars: spike indices identical for the first 100 ticks; state within 1e-5
relative; logits within 1e-4 relative.  The engine reproduces the reference's fp32 operation
order, so most outputs are bit-identical; the measured counts are printed for the record.
The exception is the token readout of two or more sessions, which runs on the tensor cores
(split-tf32): its logits are held to 1e-4 relative elementwise with an absolute floor of 1e-4
of the logit vector's largest magnitude (a logit near zero is a difference of much larger
terms, so no fp32 method other than the reference's own operation order gets it to 1e-4 of
itself).  The readout does not feed the state, which stays exact.
"""
import threading

import numpy as np
import pytest

from neurogen_b200.language import LanguageConfig, NativeEngine, init_packed_weights
from oracle.lang import OracleEngine, RefEngine

pytestmark = pytest.mark.gpu

SMALL = LanguageConfig(columns=3, width=17, regions=2, ticks=3, idle_steps=1, speech_width=16, mel_bins=8)
STATE_RTOL, STATE_ATOL = 1e-5, 1e-6
LOGIT_RTOL, LOGIT_ATOL = 1e-4, 1e-6


def assert_logits_close(got, want):
    """Tensor-core readout bar: 1e-4 relative, floor 1e-4 of the vector's largest logit."""
    np.testing.assert_allclose(got, want, rtol=LOGIT_RTOL, atol=LOGIT_RTOL * float(np.abs(want).max()))


def fields(cfg, state):
    n, w = cfg.columns * 64, cfg.width
    rs = 5 * n + w
    out = {}
    for r in range(cfg.regions):
        b = state[..., r * rs:(r + 1) * rs]
        out[r] = dict(v=b[..., :n], trace=b[..., n:2 * n], adapt=b[..., 2 * n:3 * n],
                      last=b[..., 3 * n:4 * n], mem=b[..., 4 * n:4 * n + w], counts=b[..., 4 * n + w:])
    return out


def assert_state_close(cfg, got, want):
    fg, fw = fields(cfg, got), fields(cfg, want)
    for r in fg:
        np.testing.assert_array_equal(fg[r]['last'], fw[r]['last'])     # spikes: exact
        np.testing.assert_array_equal(fg[r]['counts'], fw[r]['counts'])
        for k in ('v', 'trace', 'adapt', 'mem'):
            np.testing.assert_allclose(fg[r][k], fw[r][k], rtol=STATE_RTOL, atol=STATE_ATOL, err_msg=k)


def test_small_config_tokens_and_idle_vs_reference(golden_lang):
    g = golden_lang
    w = g['small_weights']
    eng, ref = NativeEngine(SMALL, w), RefEngine(SMALL, w)
    sa = np.zeros((1, ref.S), np.float32)
    sb = sa[0].copy()
    exact = total = 0
    for tok in g['small_tokens']:
        la, sa, aa, ha = eng.step_batch(np.array([tok]), sa)
        lb, sb, ab, hb = ref.step(int(tok), sb)
        np.testing.assert_allclose(la[0], lb, rtol=LOGIT_RTOL, atol=LOGIT_ATOL)
        assert_state_close(SMALL, sa[0], sb)
        np.testing.assert_allclose(ha[0], hb, rtol=1e-4, atol=1e-6)
        assert abs(aa[0] - ab) < 1e-7
        exact += int(np.array_equal(sa[0], sb) and np.array_equal(la[0], lb))
        total += 1
    x = np.zeros((1, SMALL.width), np.float32)
    for _ in range(8):
        ha, sa, aa = eng.advance_batch(x, sa, idle=True)
        hb, sb, ab = ref.advance(x[0], sb, True)
        assert_state_close(SMALL, sa[0], sb)
    print(f'bit-identical token steps: {exact}/{total}')


def test_batch_rows_equal_single_session_runs(monkeypatch):
    """With the SIMT readout every output of a batched step has the bits of a batch-1 step."""
    monkeypatch.setenv('NEUROGEN_READOUT', 'simt')
    cfg = LanguageConfig(columns=4, width=40, regions=2, ticks=2, idle_steps=1)
    w = init_packed_weights(cfg, seed=3)
    eng = NativeEngine(cfg, w)
    B = 37  # exercises the tiled projection with a ragged session tile
    rng = np.random.default_rng(0)
    toks = rng.integers(0, 264, (6, B))
    sb = np.zeros((B, eng.state_size), np.float32)
    singles = [np.zeros((1, eng.state_size), np.float32) for _ in range(B)]
    for t in range(6):
        lb, sb, ab, hb = eng.step_batch(toks[t], sb)
        for b in (0, 1, 17, 36):
            l1, singles[b], a1, h1 = eng.step_batch(toks[t, b:b + 1], singles[b])
            assert np.array_equal(l1[0], lb[b]) and np.array_equal(singles[b][0], sb[b])


def recover_tick_spikes(cfg, before, after):
    """Per-tick spikes of one advance with ticks=2: tick 1 is last_spikes, tick 0 follows from
    the exact integer spike counters (counts_after - counts_before - tick1)."""
    fb, fa = fields(cfg, before), fields(cfg, after)
    out = []
    for r in range(cfg.regions):
        t1 = fa[r]['last']
        t0 = fa[r]['counts'] - fb[r]['counts'] - t1
        out.append(np.stack([t0, t1]))
    return np.stack(out)  # [R, 2, n]


def test_bc250_every_spike_of_first_128_ticks(golden_lang):
    """Seed-0 BC-250 profile, free-running on the tokens of the benchmark stream: the spikes of
    every unit at every tick of the first 32 tokens (64 advances x 2 ticks = 128 ticks per
    region, 4 regions) equal the reference's."""
    cfg = LanguageConfig()
    w = init_packed_weights(cfg, seed=0)
    eng, orc = NativeEngine(cfg, w), OracleEngine(cfg, w)
    emb = w[:264 * cfg.width].reshape(264, cfg.width)
    zero = np.zeros((1, cfg.width), np.float32)
    sg = np.zeros((1, orc.S), np.float32)
    so = sg[0].copy()
    for tok in golden_lang['bc250_tokens'][:32]:
        lo, nxt, ao, ho, spikes = orc.step(int(tok), so, record=True)
        per = spikes.reshape(2, cfg.regions, cfg.ticks, orc.n)
        h0, s1, _ = eng.advance_batch(emb[tok][None], sg, idle=False)
        np.testing.assert_array_equal(recover_tick_spikes(cfg, sg[0], s1[0]), per[0])
        h1, s2, _ = eng.advance_batch(zero, s1, idle=True)
        np.testing.assert_array_equal(recover_tick_spikes(cfg, s1[0], s2[0]), per[1])
        assert_state_close(cfg, s2[0], nxt)
        sg, so = s2, nxt


def test_bc250_token_step_teacher_forced_512_tokens(golden_lang):
    """All 512 tokens of the seed-0 stream, each step started from the reference's own state:
    logits 1e-4 relative, state 1e-5 relative, spikes exact (any spike decision within the fp32
    noise of its threshold would be reported here)."""
    cfg = LanguageConfig()
    w = init_packed_weights(cfg, seed=0)
    eng, ref = NativeEngine(cfg, w), RefEngine(cfg, w)
    s = np.zeros(ref.S, np.float32)
    identical = 0
    toks = golden_lang['bc250_tokens']
    for i, tok in enumerate(toks):
        lg, sg, ag, hg = eng.step_batch(np.array([tok]), s[None])
        lr, sr, ar, hr = ref.step(int(tok), s)
        if i < len(golden_lang['bc250_native_logits']):
            assert np.array_equal(lr, golden_lang['bc250_native_logits'][i])
        np.testing.assert_allclose(lg[0], lr, rtol=LOGIT_RTOL, atol=LOGIT_ATOL)
        assert_state_close(cfg, sg[0], sr)
        identical += int(np.array_equal(sg[0], sr) and np.array_equal(lg[0], lr))
        s = sr
    print(f'bit-identical BC-250 token steps: {identical}/{len(toks)}')


def test_batched_sessions_vs_reference():
    cfg = LanguageConfig()
    w = init_packed_weights(cfg, seed=0)
    eng, ref = NativeEngine(cfg, w), RefEngine(cfg, w)
    B = 6
    rng = np.random.default_rng(5)
    toks = rng.integers(0, 264, (4, B))
    sb = np.zeros((B, ref.S), np.float32)
    sr = [np.zeros(ref.S, np.float32) for _ in range(B)]
    for t in range(4):
        lb, sb, ab, hb = eng.step_batch(toks[t], sb)
        for b in range(B):
            lr, sr[b], ar, hr = ref.step(int(toks[t, b]), sr[b])
            assert_logits_close(lb[b], lr)
            assert_state_close(cfg, sb[b], sr[b])


def test_errors_and_caller_state_immutability():
    cfg = LanguageConfig(columns=2, width=8, regions=2, ticks=3, idle_steps=1)
    eng = NativeEngine(cfg, init_packed_weights(cfg, seed=1))
    s = np.zeros((1, eng.state_size), np.float32)
    s[0, 3] = np.nan
    with pytest.raises(ValueError, match='Non-finite native state'):
        eng.step_batch(np.array([1]), s)
    s[0, 3] = 0
    with pytest.raises(ValueError, match='Token must be in 0..263'):
        eng.step_batch(np.array([264]), s)
    before = s.copy()
    eng.step_batch(np.array([5]), s)
    assert np.array_equal(before, s)
    lib = eng.lib
    bad = np.zeros(eng.state_size + 1, np.float32)
    out = np.zeros(eng.state_size + 1, np.float32)
    l = np.zeros(264, np.float32)
    h = np.zeros(cfg.width, np.float32)
    a = np.zeros(1, np.float32)
    assert lib.ng_step(eng.handle, 1, bad, bad.size, out, l, h, a) == -1
    assert lib.ng_error().decode() == 'Invalid native state size'


def test_shared_handle_from_two_threads():
    cfg = LanguageConfig(columns=2, width=16, regions=2, ticks=2, idle_steps=1)
    eng = NativeEngine(cfg, init_packed_weights(cfg, seed=4))

    def run(token):
        s = np.zeros((1, eng.state_size), np.float32)
        outs = []
        for t in (257, token, token):
            lg, s, _, _ = eng.step_batch(np.array([t]), s)
            outs.append(lg.copy())
        return outs

    expected = [run(10), run(20)]
    results = [None, None]

    def worker(k, tok):
        results[k] = run(tok)

    threads = [threading.Thread(target=worker, args=(k, t)) for k, t in enumerate((10, 20))]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    for e, r in zip(expected, results):
        for x, y in zip(e, r):
            assert np.array_equal(x, y)


def test_pool_matches_host_batch():
    cfg = LanguageConfig(columns=3, width=24, regions=2, ticks=2, idle_steps=1)
    w = init_packed_weights(cfg, seed=6)
    eng = NativeEngine(cfg, w)
    lib = eng.lib
    B = 5
    pool = lib.ng_pool_create(eng.handle, B)
    assert pool
    try:
        toks = np.array([1, 2, 3, 4, 5], np.int32)
        logits = np.zeros((B, 264), np.float32)
        assert lib.ng_pool_step(pool, toks, logits.ctypes.data, None, None) == 0
        st = np.zeros((B, eng.state_size), np.float32)
        assert lib.ng_pool_store(pool, st) == 0
        lb, sb, _, _ = eng.step_batch(toks, np.zeros((B, eng.state_size), np.float32))
        assert np.array_equal(lb, logits) and np.array_equal(sb, st)
    finally:
        lib.ng_pool_destroy(pool)


@pytest.mark.parametrize('var,tile', [('NEUROGEN_PROJ_TILE', t) for t in ('8', '16', '32', '64')] +
                         [('NEUROGEN_PROJ_SMALL', t) for t in ('8', '16', '32')] +
                         [('NEUROGEN_PROJ_ROWMAJOR', t) for t in ('16', '32')] +
                         [('NEUROGEN_PROJ_REG', t) for t in ('22', '42', '24', '44', '43', '23')])
def test_every_projection_tile_is_bit_identical(var, tile):
    """Each session tile of the batched projection kernels (wide tiles and the small-batch
    kernel) gives the same bits as the batch-1 kernel (one sequential chain per output in every
    case).  Runs in a child process because the tile override is read once per process."""
    import os
    import subprocess
    import sys
    code = f"""
import sys, numpy as np
sys.path[:0] = {[str(p) for p in sys.path[:3]]!r}
from neurogen_b200.language import LanguageConfig, NativeEngine, init_packed_weights
cfg = LanguageConfig(columns=6, width=96, regions=3, ticks=2, idle_steps=1)
eng = NativeEngine(cfg, init_packed_weights(cfg, seed=11))
B = 45
rng = np.random.default_rng(1)
toks = rng.integers(0, 264, (3, B))
sb = np.zeros((B, eng.state_size), np.float32)
single = np.zeros((B, eng.state_size), np.float32)
for t in range(3):
    lb, sb, _, _ = eng.step_batch(toks[t], sb)
    for b in (0, 7, 44):
        l1, s1, _, _ = eng.step_batch(toks[t, b:b + 1], single[b:b + 1])
        single[b] = s1[0]
        assert np.array_equal(l1[0], lb[b]) and np.array_equal(s1[0], sb[b]), (t, b)
print('ok')
"""
    env = dict(os.environ, **{var: tile, 'NEUROGEN_READOUT': 'simt'})
    out = subprocess.run([sys.executable, '-c', code], env=env, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and 'ok' in out.stdout, out.stderr[-2000:]


@pytest.mark.parametrize('columns,ticks,batch', [
    (3, 3, 1),    # cluster of 3 CTAs, one column each
    (8, 2, 2),    # cluster of 2 CTAs, four columns each, two sessions per CTA
    (6, 3, 5),    # cluster of 3, two columns each, ragged session tile
    (9, 3, 3),    # no cluster shape: one launch per tick
    (1, 1, 1),    # single column, single tick
    (4, 2, 3),    # one CTA of four columns
    (8, 2, 70),   # cluster of 2 CTAs, many sessions
    (2, 3, 9),    # one CTA of two columns
])
def test_tick_paths_match_reference(columns, ticks, batch):
    """Every tick-kernel shape (cluster widths, columns per CTA, the per-tick fallback) against
    the reference library, several sessions at once."""
    cfg = LanguageConfig(columns=columns, width=24, regions=2, ticks=ticks, idle_steps=1)
    w = init_packed_weights(cfg, seed=columns * 10 + ticks)
    rng = np.random.default_rng(columns)
    w = (w + rng.normal(0, 0.2, w.size)).astype(np.float32)  # non-uniform recurrent weights
    eng, ref = NativeEngine(cfg, w), RefEngine(cfg, w)
    sb = np.zeros((batch, ref.S), np.float32)
    sr = [np.zeros(ref.S, np.float32) for _ in range(batch)]
    for t in range(8):
        toks = rng.integers(0, 264, batch)
        lb, sb, ab, hb = eng.step_batch(toks, sb)
        for b in range(batch):
            lr, sr[b], ar, hr = ref.step(int(toks[b]), sr[b])
            if batch > 1:
                assert_logits_close(lb[b], lr)
            else:
                np.testing.assert_allclose(lb[b], lr, rtol=LOGIT_RTOL, atol=LOGIT_ATOL)
            assert_state_close(cfg, sb[b], sr[b])


def test_session_pool_save_load_roundtrip(tmp_path):
    """A session saved from a device pool in the reference's session layout and loaded into
    another pool (any slot) continues exactly as the original."""
    from neurogen_b200.language import (LanguageConfig, NativeLanguageModel, SessionPool, init_packed_weights,
                                        load_session)
    cfg = LanguageConfig(columns=4, width=32, regions=2, ticks=2, idle_steps=1)
    model = NativeLanguageModel(cfg, init_packed_weights(cfg, seed=3))
    a = SessionPool(model, 4)
    rng = np.random.default_rng(0)
    for _ in range(5):
        a.step(rng.integers(0, 264, 4))
    a.save(tmp_path / 's.pt', 2, 'ckpt-1')
    payload = load_session(tmp_path / 's.pt', 'ckpt-1')
    assert payload['format'] == 'neurogen-session-v2' and len(payload['state']) == cfg.regions
    assert tuple(payload['state'][0][4].shape) == (1, cfg.width)
    with pytest.raises(ValueError, match='different model checkpoint'):
        load_session(tmp_path / 's.pt', 'ckpt-2')
    b = SessionPool(model, 3)
    b.load(tmp_path / 's.pt', 0, 'ckpt-1')
    assert np.array_equal(b.logits[0], a.logits[2])
    for _ in range(4):
        toks = rng.integers(0, 264, 4)
        la = a.step(toks)
        lb = b.step(np.array([toks[2], 7, 9]))
        assert np.array_equal(la[2], lb[0])
    assert np.array_equal(a.states()[2], b.states()[0])


def head_weights(cfg, w):
    """Head Linear(width, 264) at the end of the packed weight vector: weight [264][w], bias."""
    n = 264 * cfg.width + 264
    tail = w[-n:]
    return tail[:264 * cfg.width].reshape(264, cfg.width).astype(np.float64), tail[264 * cfg.width:].astype(np.float64)


@pytest.mark.parametrize('B', [2, 37, 128, 130, 256])
def test_tensor_core_readout_bc250(B, monkeypatch):
    """The tcgen05 readout of B sessions (BC-250, K=768: 24 k chunks in 4 segments) against the
    float64 product of the same hidden states, against the sequential SIMT readout, and the
    state bit-identical between the two readouts (the readout feeds nothing back)."""
    cfg = LanguageConfig()
    w = init_packed_weights(cfg, seed=0)
    eng = NativeEngine(cfg, w)
    W, bias = head_weights(cfg, w)
    rng = np.random.default_rng(B)
    s0 = np.zeros((B, eng.state_size), np.float32)
    for _ in range(2):   # move off the zero state
        _, s0, _, _ = eng.step_batch(rng.integers(0, 264, B), s0)
    toks = rng.integers(0, 264, B)
    lt, st, at, ht = eng.step_batch(toks, s0)
    exact = ht.astype(np.float64) @ W.T + bias
    scale = np.abs(exact).max(axis=1, keepdims=True)
    err = np.abs(lt - exact) / scale
    print(f'B={B}: max |tc - f64| / row scale = {err.max():.2e}')
    assert err.max() < 2e-5
    monkeypatch.setenv('NEUROGEN_READOUT', 'simt')
    ls, ss, as_, hs = eng.step_batch(toks, s0)
    assert np.array_equal(ss, st) and np.array_equal(hs, ht) and np.array_equal(as_, at)
    assert_logits_close(lt, ls)
    assert not np.array_equal(lt, ls)   # the tensor-core path did run


def test_tensor_core_readout_ragged_k_and_fallback(monkeypatch):
    """K=40 (a partial k chunk, fewer chunks than segments) on the tensor cores; K=17 (rows not
    16-byte aligned) falls back to the SIMT readout, bit-identical to batch 1."""
    for width, tc in ((40, True), (17, False)):
        cfg = LanguageConfig(columns=2, width=width, regions=2, ticks=2, idle_steps=1)
        w = init_packed_weights(cfg, seed=width)
        eng = NativeEngine(cfg, w)
        W, bias = head_weights(cfg, w)
        B = 9
        rng = np.random.default_rng(0)
        sb = np.zeros((B, eng.state_size), np.float32)
        for _ in range(3):
            lb, sb, _, hb = eng.step_batch(rng.integers(0, 264, B), sb)
        exact = hb.astype(np.float64) @ W.T + bias
        err = np.abs(lb - exact) / np.abs(exact).max(axis=1, keepdims=True)
        assert err.max() < 2e-5
        l1, _, _, _ = eng.step_batch(np.array([5]), sb[:1])
        monkeypatch.setenv('NEUROGEN_READOUT', 'simt')
        l1s, _, _, _ = eng.step_batch(np.array([5]), sb[:1])
        lbs, _, _, _ = eng.step_batch(np.full(B, 5), sb)
        monkeypatch.delenv('NEUROGEN_READOUT')
        lbt, _, _, _ = eng.step_batch(np.full(B, 5), sb)
        assert np.array_equal(l1, l1s) and np.array_equal(lbs[0], l1s[0])
        assert np.array_equal(lbt, lbs) != tc


@pytest.mark.parametrize('sb', ['2', '4', '8'])
def test_tick_sessions_per_thread_bit_identical(sb, monkeypatch):
    """The recurrent tick kernel with 2, 4 or 8 sessions a thread (ragged last CTA) gives the bits
    of one session a thread, for 4-, 2- and 1-column CTAs."""
    for columns in (8, 6, 3):
        cfg = LanguageConfig(columns=columns, width=24, regions=2, ticks=3, idle_steps=1)
        w = init_packed_weights(cfg, seed=columns)
        rng = np.random.default_rng(columns)
        w = (w + rng.normal(0, 0.2, w.size)).astype(np.float32)
        eng = NativeEngine(cfg, w)
        B = 13
        toks = rng.integers(0, 264, (4, B))
        out = {}
        for mode in ('1', sb):
            monkeypatch.setenv('NEUROGEN_TICK_SB', mode)
            st = np.zeros((B, eng.state_size), np.float32)
            for t in range(4):
                lg, st, _, _ = eng.step_batch(toks[t], st)
            out[mode] = (lg, st)
        assert np.array_equal(out['1'][0], out[sb][0]) and np.array_equal(out['1'][1], out[sb][1])


def test_listen_matches_reference_advance_and_head():
    """listen (reference model.py:152-158): each mel frame through the audio projection, one
    non-idle advance on the GPU engine, logits from the head; against the reference library's
    advance with the same projections."""
    import torch
    from neurogen_b200.language import NativeLanguageModel
    cfg = LanguageConfig(columns=3, width=24, regions=2, ticks=2, idle_steps=1, mel_bins=8)
    w = init_packed_weights(cfg, seed=5)
    torch.manual_seed(1)
    audio = torch.nn.Linear(cfg.mel_bins, cfg.width)
    W, bias = head_weights(cfg, w)
    sd = {'audio_input.weight': audio.weight.detach().clone(), 'audio_input.bias': audio.bias.detach().clone(),
          'head.weight': torch.from_numpy(W.astype(np.float32)), 'head.bias': torch.from_numpy(bias.astype(np.float32))}
    model = NativeLanguageModel(cfg, w, state_dict=sd)
    feats = torch.randn(2, 5, cfg.mel_bins)
    logits, state, act = model.listen(feats)
    assert tuple(logits.shape) == (2, 5, 264)
    ref = RefEngine(cfg, w)
    with torch.no_grad():
        for b in range(2):
            s = np.zeros(ref.S, np.float32)
            for t in range(5):
                x = audio(feats[b, t]).numpy()
                h, s, _ = ref.advance(x, s, False)
                want = (torch.from_numpy(h) @ sd['head.weight'].T + sd['head.bias']).numpy()
                np.testing.assert_allclose(logits[b, t].numpy(), want, rtol=1e-4, atol=1e-5)
    with pytest.raises(ValueError, match='mel_bins'):
        model.listen(torch.zeros(2, 3, cfg.mel_bins + 1))


READOUT_STALL_CHILD = r'''
import sys
sys.path[:0] = {paths!r}
import numpy as np
from neurogen_b200.language import LanguageConfig, NativeEngine, init_packed_weights
cfg = LanguageConfig(columns=2, width=32, regions=2, ticks=2, idle_steps=1)
eng = NativeEngine(cfg, init_packed_weights(cfg, seed=2))
s = np.zeros((4, eng.state_size), np.float32)
try:
    eng.step_batch(np.array([1, 2, 3, 4]), s)
    print('no error')
except ValueError as e:
    print('raised:', e)
l1, s1, _, _ = eng.step_batch(np.array([1, 2, 3, 4]), s)     # same engine, the next step
fresh = NativeEngine(cfg, init_packed_weights(cfg, seed=2))
l2, s2, _, _ = fresh.step_batch(np.array([1, 2, 3, 4]), s)
print('after:', bool(np.array_equal(l1, l2) and np.array_equal(s1, s2)))
'''


def test_readout_wait_runs_out_cleanly(tmp_path):
    """The tensor-core readout's waits are bounded.  A test switch makes the first readout launch
    take the timeout path before it issues any copy or MMA: the batched step reports
    'Readout kernel timed out', and the next step on the same engine runs normally and equals a
    fresh engine's."""
    import os
    import subprocess
    import sys
    script = tmp_path / 'stall.py'
    script.write_text(READOUT_STALL_CHILD.format(paths=[str(p) for p in sys.path[:3]]))
    env = dict(os.environ, NEUROGEN_TEST_READOUT_STALL='1')
    env.pop('NEUROGEN_READOUT', None)
    out = subprocess.run([sys.executable, str(script)], env=env, capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr[-3000:]
    assert 'raised: Readout kernel timed out' in out.stdout, out.stdout
    assert 'after: True' in out.stdout, out.stdout


def libm_inputs():
    """Every float of the binades where the host library and a correctly rounded evaluation
    differ most ([2^-3, 2^-2), [2^-1, 1), [1, 2)), both signs, plus 4 M random floats of
    magnitude 2^-30 .. 2^7 and the range edges."""
    dense = np.concatenate([np.arange(np.float32(lo).view(np.uint32), np.float32(2 * lo).view(np.uint32),
                                      dtype=np.uint32) for lo in (0.125, 0.5, 1.0)]).view(np.float32)
    rng = np.random.default_rng(0)
    rand = (rng.uniform(-30, 7, 4_000_000).astype(np.float32))
    rand = (np.exp2(rand) * rng.choice([-1, 1], rand.size)).astype(np.float32)
    edges = np.array([0.0, 2.0 ** -40, 2.0 ** -22, 16.75, 16.7501, 22.0, 21.999998, 88.8, 100.0, 1e30],
                     np.float32)
    x = np.concatenate([dense, -dense, rand, edges, -edges]).astype(np.float32)
    return np.ascontiguousarray(x)


def test_device_tanh_and_sigmoid_equal_the_host_library():
    """The tick kernels' feedback tanh and input sigmoid return the host C library's tanhf and
    1 / (1 + expf(-x)) bit for bit (the reference engine's functions; neither is correctly
    rounded, so this needs the correction tables of libm_match.cuh)."""
    import ctypes as ct
    from neurogen_b200 import library
    from oracle.lang import ORACLE_LIB
    x = libm_inputs()
    dt, ds = np.empty_like(x), np.empty_like(x)
    lib = library()
    assert lib.ng_math_eval(x, x.size, dt, ds) == 0, lib.ng_error().decode()
    orc = ct.CDLL(str(ORACLE_LIB))
    orc.om_libm_eval.argtypes = [ct.c_void_p, ct.c_size_t, ct.c_void_p, ct.c_void_p]
    ht, hs = np.empty_like(x), np.empty_like(x)
    orc.om_libm_eval(x.ctypes.data, x.size, ht.ctypes.data, hs.ctypes.data)
    bad_t = int((dt.view(np.uint32) != ht.view(np.uint32)).sum())
    bad_s = int((ds.view(np.uint32) != hs.view(np.uint32)).sum())
    cr = np.tanh(x.astype(np.float64)).astype(np.float32)
    not_cr = int((cr.view(np.uint32) != ht.view(np.uint32)).sum())
    print(f'{x.size:,} inputs: tanh mismatches {bad_t}, sigmoid mismatches {bad_s} '
          f'(host tanhf differs from correct rounding on {not_cr:,} of them)')
    assert bad_t == 0 and bad_s == 0
