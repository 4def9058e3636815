"""The network oracle pinned to the reference simulator, and the seeded generators (CPU only).

* fp64 mode reproduces neurogen/biology.py (frozen synapses, no background) on its own
  anatomy: every spike of 200 ticks and the membrane voltage to 1e-9 mV
  (tests/golden/make_net_golden.py).
* the known-answer tests of tests/test_biology.py:34-56 (a delay-d emission arrives exactly d
  ticks later, E->g_E and I->g_I, with g == w exactly) and :177-190 (passive membrane
  V = -55 - 10 exp(-10/20) at 1e-12 for dt in {0.25, 0.5, 1}).
* generator properties: fan-in, block structure, delays, Dale signs, fixed-point grid,
  determinism.
"""
import numpy as np
import pytest

from conftest import ROOT
from neurogen_b200.network import Topology, default_config, isolated_8k, scaled_262k
from oracle.net import NetOracle, unpack_spikes


@pytest.fixture(scope='module')
def golden():
    return np.load(ROOT / 'tests' / 'golden' / 'net_golden.npz')


def golden_cfg(g, **kw):
    return default_config(n=int(g['n']), n_exc=int(g['n_exc']), drive_p=0.0, **kw)


def test_fp64_restatement_reproduces_biology_py(golden):
    g = golden
    o = NetOracle(golden_cfg(g), g['pre'], g['post'], g['delay'], g['weight'])
    o.set_state64(v=g['v0'])
    spikes, v, ge, gi = o.run64(len(g['spikes']), current=g['current'])
    got = unpack_spikes(spikes, int(g['n']))
    assert got.sum() > 100
    np.testing.assert_array_equal(got, g['spikes'])
    np.testing.assert_allclose(v[:len(g['voltage'])], g['voltage'], atol=1e-9, rtol=0)
    np.testing.assert_allclose(ge[:len(g['ge'])], g['ge'], atol=1e-12, rtol=1e-12)


def test_fp32_contract_tracks_biology_py(golden):
    g = golden
    w = (np.round(g['weight'] * 2.0 ** 24) / 2.0 ** 24).astype(np.float32)
    cfg = golden_cfg(g, bias_pa=0.0)
    o = NetOracle(cfg, g['pre'], g['post'], g['delay'], w)
    # fp32 mode has a scalar bias; use the cells without injected current as a check of the
    # passive + synaptic path by injecting nothing and comparing the first silent ticks.
    o.set_state(v=g['v0'].astype(np.float32))
    spikes, _ = o.run(5)
    ref = NetOracle(cfg, g['pre'], g['post'], g['delay'], g['weight'])
    ref.set_state64(v=g['v0'])
    s64, v64, _, _ = ref.run64(5)
    st = o.get_state()
    np.testing.assert_array_equal(unpack_spikes(spikes, int(g['n'])), unpack_spikes(s64, int(g['n'])))
    np.testing.assert_allclose(st['v'], v64[-1], atol=2e-4)


def single_synapse(excitatory, fp64):
    cfg = default_config(n=4, n_exc=2, drive_p=0.0)
    pre = 0 if excitatory else 2
    w = 2.0 if excitatory else -2.0
    o = NetOracle(cfg, [pre], [1], [3], [w])
    v = np.full(4, -65.0)
    v[pre] = 0.0  # induces one emission at tick 0 with no external drive
    return o, v, pre


@pytest.mark.parametrize('excitatory', [True, False])
@pytest.mark.parametrize('fp64', [True, False])
def test_delayed_transmission_and_dale_sign(excitatory, fp64):
    o, v, pre = single_synapse(excitatory, fp64)
    if fp64:
        o.set_state64(v=v)
        spikes, vv, ge, gi = o.run64(4)
        fired = unpack_spikes(spikes, 4)
        assert fired[0, pre]
        assert ge[1:3].sum() == 0 and gi[1:3].sum() == 0
        assert (ge[3, 1] if excitatory else gi[3, 1]) == 2.0
        assert (vv[3, 1] > -65) if excitatory else (vv[3, 1] < -65)
    else:
        o.set_state(v=v.astype(np.float32))
        spikes, counts = o.run(3)
        assert unpack_spikes(spikes, 4)[0, pre]
        assert counts[0, 1] == 1
        st = o.get_state()
        assert st['ge'].sum() == 0 and st['gi'].sum() == 0
        o.run(1)
        st = o.get_state()
        assert (st['ge'][1] if excitatory else st['gi'][1]) == 2.0
        assert (st['v'][1] > -65) if excitatory else (st['v'][1] < -65)


@pytest.mark.parametrize('dt', [.25, .5, 1.])
def test_passive_membrane_solution_across_timesteps(dt):
    cfg = default_config(n=8, n_exc=6, drive_p=0.0, dt_ms=dt, bias_pa=100.0)
    o = NetOracle(cfg, [], [], [], [])
    o.set_state64(v=np.full(8, -65.0))
    steps = round(10 / dt)
    _, v, _, _ = o.run64(steps)
    expected = -55 - 10 * np.exp(-10 / 20)
    np.testing.assert_allclose(v[-1, :6], expected, atol=1e-12)
    o.set_state(v=np.full(8, -65.0, np.float32))
    o.run(steps)
    np.testing.assert_allclose(o.get_state()['v'][:6], expected, atol=2e-4)


def test_fixed_fanin_generator_properties():
    cfg = default_config(n=4096, n_exc=3276, topology='fixed_fanin', fanin=64, weight_kind='halfnormal_f16',
                         w_mu=0.0, w_sigma=0.05, seed=5)
    pre, post, delay, w = Topology(cfg).export()
    assert len(pre) == 4096 * 64
    assert (np.bincount(post, minlength=4096) == 64).all()
    assert (pre != post).all()
    assert delay.min() == 1 and delay.max() == 8
    assert ((w > 0) == (pre < cfg.n_exc)).all()
    assert np.array_equal(w.astype(np.float16).astype(np.float32), w)
    assert abs(np.abs(w).mean() - 0.05 * np.sqrt(2 / np.pi)) < 1e-3
    assert (np.diff(pre) >= 0).all()
    again = Topology(cfg).export()
    for x, y in zip((pre, post, delay, w), again):
        assert np.array_equal(x, y)
    cfg.seed = 6
    assert not np.array_equal(Topology(cfg).export()[0], pre)


def test_erdos_renyi_generator_properties():
    cfg = isolated_8k()
    pre, post, delay, w = Topology(cfg).export()
    m = len(pre)
    assert abs(m / (8192 * 8191) - 0.02) < 5e-4
    assert (pre != post).all()
    assert np.array_equal(np.round(np.abs(w).astype(np.float64) * 2 ** 24), np.abs(w).astype(np.float64) * 2 ** 24)
    assert ((w > 0) == (pre < cfg.n_exc)).all()
    logw = np.log(np.abs(w))
    assert abs(logw.mean() + 2.0) < 0.01 and abs(logw.std() - 0.5) < 0.01


@pytest.mark.parametrize('storage', ['csr', 'bsr'])
def test_block_generator_properties(storage):
    cfg = default_config(n=2048, n_exc=1638, topology='bsr16', bsr_blocks=16, bsr_fill=64,
                         weight_kind='halfnormal_f16', w_mu=0.0, w_sigma=0.05, storage=storage, seed=2)
    pre, post, delay, w = Topology(cfg).export()
    assert len(pre) == (2048 // 16) * 16 * 64
    blocks = {}
    for p, q, d in zip(pre // 16, post // 16, delay):
        blocks.setdefault((q, p), set()).add(d)
    assert all(len(v) == 1 for v in blocks.values())          # one delay per block
    per_row = np.bincount([q for q, _ in blocks], minlength=128)
    assert (per_row == 16).all()
    fill = np.bincount([q * 128 + p for p, q in zip(pre // 16, post // 16)])
    assert set(fill[fill > 0]) == {64}


def test_block_storage_matches_its_csr_copy():
    base = dict(n=1024, n_exc=819, topology='bsr16', bsr_blocks=8, bsr_fill=40, weight_kind='halfnormal_f16',
                w_mu=0.0, w_sigma=0.05, seed=9)
    a = Topology(default_config(storage='csr', **base)).export()
    b = Topology(default_config(storage='bsr', **base)).export()
    for x, y in zip(a, b):
        assert np.array_equal(x, y)


def test_invalid_network_configs_are_rejected():
    from neurogen_b200 import library
    lib = library()
    for kw in (dict(n=0), dict(n_exc=5000), dict(delay_max=16), dict(delay_min=0),
               dict(topology='bsr16', n=1000), dict(storage='bsr'), dict(drive_p=1.5),
               dict(tau_exc_ms=0.0)):
        with pytest.raises(ValueError):
            Topology(default_config(**kw))
    assert lib.ng_error().decode()


def test_fixed_point_range_is_enforced():
    cfg = default_config(n=64, n_exc=64, topology='fixed_fanin', fanin=60, w_mu=4.0, w_sigma=0.1)
    with pytest.raises(ValueError, match='fixed-point'):
        Topology(cfg)


def test_scaled_configs_describe_the_benchmark():
    c = scaled_262k('csr')
    assert (c.n, c.fanin, c.delay_min, c.delay_max, c.drive_kind) == (262144, 512, 1, 8, 1)
    b = scaled_262k('bsr')
    assert (b.topology, b.bsr_blocks, b.bsr_fill, b.storage) == (2, 128, 64, 1)
    assert 128 * 64 // 16 == 512  # same mean fan-in as the CSR matrix


def test_fp32_contract_raster_equals_fp64_unrounded_at_8k():
    """The isolated 8,192-neuron benchmark network for its full 1,000 ticks: the engine's fp32
    contract (weights rounded once onto the 2^-24 nS grid, fixed-point ring, polynomial exp)
    against the fp64 equations with the unrounded lognormal weights and libm exp.  Every spike
    decision of every tick agrees; the voltages stay within a few 1e-4 mV."""
    from oracle import net as on
    cfg = on.isolated_8k()
    pre, post, delay, w, w64 = on.generate(cfg, exact=True)
    # Half a grid step, plus fp32 rounding for weights above 0.5 nS.
    assert (np.abs(w.astype(np.float64) - w64) <= 2.0 ** -25 + np.abs(w64) * 2.0 ** -24).all()
    assert not np.array_equal(w.astype(np.float64), w64)   # the rounding did change weights
    f32 = NetOracle(cfg, pre, post, delay, w)
    f64 = NetOracle(cfg, pre, post, delay, w, w64)
    T = 1000
    s32, c32 = f32.run(T)
    s64, v64, _, _ = f64.run64(T)
    a, b = unpack_spikes(s32, cfg['n']), unpack_spikes(s64, cfg['n'])
    mismatches = int((a != b).sum())
    dv = float(np.abs(f32.get_state()['v'].astype(np.float64) - v64[-1]).max())
    print(f'N=8,192, {T} ticks, {int(a.sum())} spikes: {mismatches} differing spike decisions; '
          f'max |V32 - V64| after {T} ticks {dv:.2e} mV')
    assert a.sum() > 100000 and mismatches == 0
    assert dv < 1e-2


@pytest.mark.parametrize('name', ['er', 'fanin', 'bsr'])
def test_oracle_generator_equals_engine_generator(name):
    """oracle/net_topo.c restates the engine's seeded generator: the same synapses (pre, post,
    delay, weight bits), so the CPU legs build their networks without the CUDA library."""
    from oracle import net as on
    if name == 'er':
        pc, oc = isolated_8k(seed=3), on.isolated_8k(seed=3)
    elif name == 'fanin':
        kw = dict(n=20000, n_exc=16000, topology=1, fanin=64, weight_kind=1, w_mu=0.0, w_sigma=0.05, seed=5,
                  delay_min=2, delay_max=7)
        pc, oc = default_config(**kw), on.config(**kw)
    else:
        kw = dict(n=4096, n_exc=3277, topology=2, bsr_blocks=32, bsr_fill=64, weight_kind=1, w_mu=0.0,
                  w_sigma=0.05, seed=4)
        pc, oc = default_config(**kw), on.config(**kw)

    def canon(e):
        pre, post, delay, w = e[:4]
        o = np.lexsort((w.view(np.uint32), delay, post, pre))
        return [x[o] for x in (pre, post, delay, w)]

    for x, y in zip(canon(Topology(pc).export()), canon(on.generate(oc))):
        assert np.array_equal(x, y)


def test_oracle_workload_configs_equal_the_engines():
    """The oracle-side workload definitions (used by the CPU legs) equal the engine's."""
    from oracle import net as on
    from neurogen_b200 import network as nw
    pairs = [(nw.isolated_8k(seed=2), on.isolated_8k(seed=2)), (nw.scaled_262k('csr', 0.02), on.scaled_262k('csr', 0.02)),
             (nw.scaled_262k('bsr', 0.03), on.scaled_262k('bsr', 0.03)), (nw.partitioned_4m(), on.partitioned_4m()),
             (nw.default_config(), on.config())]
    for eng, orc in pairs:
        for k, v in orc.items():
            assert getattr(eng, k) == (float(np.float32(v)) if isinstance(v, float) else v), k
