"""Session files in the reference's ``neurogen-session-v2`` layout (CPU; no GPU needed).

tests/golden/session_ref_small.pt was written by the reference runtime's own Session.save
(tests/golden/make_session_golden.py).  Our loader must read it, and the payloads our pools write
must carry the same fields with the same types, so sessions move both ways.
"""
import numpy as np
import pytest
import torch

from neurogen_b200.language import SESSION_FORMAT, load_session, save_session, session_payload

GOLDEN = __import__('pathlib').Path(__file__).resolve().parent / 'golden' / 'session_ref_small.pt'


def test_reference_session_file_loads():
    payload = load_session(GOLDEN, 'golden-checkpoint')
    assert payload['format'] == SESSION_FORMAT
    state = payload['state']
    assert len(state) == 2 and all(len(r) == 6 for r in state)
    assert tuple(state[0][0].shape) == (1, 4, 64) and tuple(state[0][4].shape) == (1, 32)
    assert tuple(payload['logits'].shape) == (264,)
    with pytest.raises(ValueError, match='different model checkpoint'):
        load_session(GOLDEN, 'another-checkpoint')


def test_our_payload_has_the_reference_fields(tmp_path):
    ref = torch.load(GOLDEN, map_location='cpu', weights_only=True)
    state = tuple(tuple(t.clone() for t in r) for r in ref['state'])
    ours = session_payload(state, ref['logits'].numpy(), 'golden-checkpoint')
    assert set(ours) == set(ref)
    for key in ref:
        assert type(ours[key]) is type(ref[key]), key
    assert ours['random'].dtype == ref['random'].dtype and ours['random'].shape == ref['random'].shape
    path = tmp_path / 'x.pt'
    save_session(path, ours)
    back = load_session(path, 'golden-checkpoint')
    for r1, r2 in zip(back['state'], ref['state']):
        for a, b in zip(r1, r2):
            assert torch.equal(a, b)
    assert np.array_equal(back['logits'].numpy(), ref['logits'].numpy())


def test_bench_counts_the_engines_launches_per_token():
    """bench.py's gpu_launches claim for a BC-250 token step equals the kernels the engine enqueues:
    2 advances x (1 batched feedback + 4 regions x (input, cluster ticks, output, LayerNorm)) less
    region 0's idle input, plus readout and activity = 35 (the ncu launch list of two pool token steps
    holds 70 kernels)."""
    import importlib.util
    from pathlib import Path
    from neurogen_b200.language import LanguageConfig
    spec = importlib.util.spec_from_file_location('bench', Path(__file__).resolve().parents[1] / 'bench.py')
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    assert bench.lang_launches_per_token(LanguageConfig()) == 35
    # No cluster shape for 9 columns: one launch per tick plus a copy for an odd tick count.
    # Advance 0: feedback + 2 x (input, 3 ticks + copy, output, norm); idle advance: feedback, region 0
    # without input, region 1 with; readout, activity.
    assert bench.lang_launches_per_token(LanguageConfig(columns=9, width=24, regions=2, ticks=3, idle_steps=1)) == \
        (1 + 2 * 7) + (1 + 6 + 7) + 2


def test_bench_algorithmic_bytes_per_tick():
    """The roofline numerator for the scaled tick: CSR events x (4 B index + 2 B fp16 weight + 1 B
    delay) + N x 48 B of state and ring slot + N/8 spike bits; block storage: per spiking neuron and
    block of its block-column a 32-byte tile column and a 4-byte block word.  At a 3% rate these are
    the 40.8 MB and 48.9 MB a tick the roofline fractions are quoted on."""
    import importlib.util
    from pathlib import Path
    from neurogen_b200.network import scaled_262k
    spec = importlib.util.spec_from_file_location('bench', Path(__file__).resolve().parents[1] / 'bench.py')
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    n = 262144
    spikes = 0.03 * n
    csr, bsr = scaled_262k('csr'), scaled_262k('bsr')
    assert bench.tick_bytes(csr, spikes, spikes * 512) == n * 48 + n / 8 + spikes * 512 * 7
    assert bench.tick_bytes(bsr, spikes, spikes * 512) == n * 48 + n / 8 + spikes * 128 * 36
    assert abs(bench.tick_bytes(csr, spikes, spikes * 512) / 1e6 - 40.8) < 0.1
    assert abs(bench.tick_bytes(bsr, spikes, spikes * 512) / 1e6 - 48.9) < 0.1


def test_bench_learning_bytes_per_tick():
    """The learning workload's roofline numerator adds, per contact, the index read and the weight
    and three traces read and written (36 B: a stored contact's potential trace is its pre trace), and
    per neuron the post trace and rate read and written (16 B) and its history bit; the network part
    is the isolated tick's (fp32 weights: 9 B an event)."""
    import importlib.util
    from pathlib import Path
    spec = importlib.util.spec_from_file_location('bench', Path(__file__).resolve().parents[1] / 'bench.py')
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    cfg = bench.engine_config(bench.oracle_tick_config('learn8k', 0.0))
    assert cfg.plasticity and cfg.weight_kind != 1
    n = cfg.n
    spikes, events, contacts = 0.02 * n, 0.02 * n * 164, 1_342_177
    base = bench.tick_bytes(cfg, spikes, events)
    assert base == n * 48 + n / 8 + events * 9
    assert bench.tick_bytes(cfg, spikes, events, contacts=contacts) - base == contacts * 36 + n * 16 + n / 8
