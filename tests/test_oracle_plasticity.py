"""The network oracle's plasticity pinned to the reference simulator (CPU only).

* fp64 mode with learning reproduces neurogen/biology.py with plasticity on (structural rewiring
  and background off; tests/golden/make_net_plastic_golden.py): every spike of 300 ticks, traces
  and rates exactly, weights to 1e-8 relative and voltages to 1e-7 mV after 100 and 300 ticks.
* the reference's known-answer tests of its rule, restated on the oracle's one-step probe:
  tests/test_biology.py:58-75 (causal pairing strengthens, anticausal weakens, simultaneous
  events leave the weight, a distant pair changes it far less) and :77-95 (the inhibitory rule
  weakens an I->E contact without postsynaptic activity and strengthens it with it; scaling raises
  E weights below the target rate and lowers them above it), in fp64 and in the fp32 contract.
* the fp32 contract (the CUDA engine's) follows the fp64 equations on a driven network.
"""
import numpy as np
import pytest

from conftest import ROOT
from neurogen_b200.network import default_config
from oracle.net import NetOracle, unpack_spikes

STATE = ('pre_trace', 'potential_trace', 'coactivity', 'usage')


@pytest.fixture(scope='module')
def golden():
    return np.load(ROOT / 'tests' / 'golden' / 'net_plastic_golden.npz')


def test_fp64_learning_reproduces_biology_py(golden):
    g = golden
    n = int(g['n'])
    o = NetOracle(default_config(n=n, n_exc=int(g['n_exc']), drive_p=0.0), g['pre'], g['post'], g['delay'],
                  g['weight'])
    o.set_plasticity(True)
    o.set_state64(v=g['v0'])
    done = 0
    for snap in (100, 300):
        spikes, v, _, _ = o.run64(snap - done, current=g['current'])
        np.testing.assert_array_equal(unpack_spikes(spikes, n), g['spikes'][done:snap])
        done = snap
        st = o.plasticity_state(fp64=True)
        # Weights to 1e-8 relative (the scaling factor's exp: NumPy's vector exp against the C
        # library's, a few ulps); traces and rates are exact; voltages to 1e-7 mV.
        np.testing.assert_allclose(st['weight'], g[f'weight_{snap}'], rtol=1e-8, atol=0)
        for k in STATE:
            np.testing.assert_array_equal(st[k], g[f'{k}_{snap}'], err_msg=k)
        np.testing.assert_array_equal(st['post_trace'], g[f'post_trace_{snap}'])
        np.testing.assert_array_equal(st['rate'], g[f'rate_{snap}'])
        np.testing.assert_allclose(v[-1], g[f'voltage_{snap}'], rtol=0, atol=1e-7)
    assert g['spikes'].sum() > 300 and (g['weight_300'] != g['weight']).sum() > 1000


def contact_net(excitatory_pre, excitatory_post=True, weight=1.5, **plastic):
    """Two cells and one contact (E->E, I->E or I->I)."""
    cfg = default_config(n=4, n_exc=2, drive_p=0.0)
    pre = 0 if excitatory_pre else 2
    post = 1 if excitatory_post else 3
    w = weight if excitatory_pre else -weight
    o = NetOracle(cfg, [pre], [post], [1], np.float32([w]), np.float64([w]))
    o.set_plasticity(True, **plastic)
    return o, pre, post


@pytest.mark.parametrize('fp64', [True, False])
def test_stdp_causal_anticausal_simultaneous(fp64):
    """tests/test_biology.py:58-75: pre then post strengthens, post then pre weakens, a
    simultaneous pair leaves the weight unchanged, and a pair 100 ticks apart changes it far
    less than one 10 ticks apart."""
    changes = []
    for offset in (10, -10, 0, 100):
        o, pre, post = contact_net(True, scaling_tau_ms=1e30)
        pre_time, post_time = (0, offset) if offset >= 0 else (-offset, 0)
        for t in range(abs(offset) + 1):
            spikes = np.zeros(4, bool)
            spikes[post] = t == post_time
            o.learn_probe([t == pre_time], spikes, fp64=fp64)
        changes.append(float(o.plasticity_state(fp64=fp64)['weight'][0]) - 1.5)
    assert changes[0] > 0
    assert changes[1] < 0
    assert changes[2] == 0
    assert changes[3] < changes[0] / 10


@pytest.mark.parametrize('fp64', [True, False])
def test_inhibitory_homeostasis_and_scaling_direction(fp64):
    """tests/test_biology.py:77-95."""
    o, pre, post = contact_net(False, weight=5.0, stdp_rate=0.0, scaling_tau_ms=1000)
    w = lambda: abs(float(o.plasticity_state(fp64=fp64)['weight'][0]))  # noqa: E731
    initial = w()
    o.learn_probe([True], np.zeros(4, bool), fp64=fp64)
    assert w() < initial            # an arrival without postsynaptic activity weakens I->E
    # with a postsynaptic trace above the target, the arrival strengthens it
    spikes = np.zeros(4, bool)
    spikes[post] = True
    o.learn_probe([False], spikes, fp64=fp64)
    initial = w()
    o.learn_probe([True], np.zeros(4, bool), fp64=fp64)
    assert w() > initial
    # scaling: no activity, rate 0 (below target) raises an E weight; I->I contacts do not learn
    e, _, _ = contact_net(True, stdp_rate=0.0, scaling_tau_ms=1000)
    before = float(e.plasticity_state(fp64=fp64)['weight'][0])
    e.learn_probe([False], np.zeros(4, bool), fp64=fp64)
    assert float(e.plasticity_state(fp64=fp64)['weight'][0]) > before
    ii, _, _ = contact_net(False, excitatory_post=False, weight=5.0)
    ii.learn_probe([True], np.zeros(4, bool), fp64=fp64)
    assert abs(float(ii.plasticity_state(fp64=fp64)['weight'][0])) == 5.0


def test_scaling_lowers_weights_above_the_target_rate():
    """tests/test_biology.py:91-95, the other direction: a postsynaptic cell driven by current to a
    rate above the 5 Hz target lowers its E contact's weight through scaling alone (no STDP)."""
    o = NetOracle(default_config(n=4, n_exc=2, drive_p=0.0), [0], [1], [1], np.float32([1.5]), np.float64([1.5]))
    o.set_plasticity(True, stdp_rate=0.0, scaling_tau_ms=1000)
    o.set_state64(v=np.array([-65.0] * 4))
    o.run64(400, current=np.array([0.0, 600.0, 0.0, 0.0]))
    st = o.plasticity_state(fp64=True)
    assert st['rate'][1] > 5.0 and st['weight'][0] < 1.5


def test_fp32_contract_follows_fp64_with_learning():
    """A driven 512-cell Erdos-Renyi network with learning: the fp32 contract and the fp64
    equations agree on every spike of the first 150 ticks and on the weights to 1e-5."""
    rng = np.random.default_rng(4)
    n, n_exc = 512, 410
    m = 16000
    pre = rng.integers(0, n, m).astype(np.int32)
    post = rng.integers(0, n, m).astype(np.int32)
    keep = pre != post
    pre, post = pre[keep], post[keep]
    delay = rng.integers(1, 9, len(pre)).astype(np.int32)
    w = np.where(pre < n_exc, rng.uniform(1.2, 2.0, len(pre)), -rng.uniform(4, 6, len(pre)))
    w = (np.round(w * 2.0 ** 24) / 2.0 ** 24)
    cfg = default_config(n=n, n_exc=n_exc, drive_kind='conductance', drive_p=0.02, drive_ns=16.0, seed=3)
    a = NetOracle(cfg, pre, post, delay, w.astype(np.float32), w)
    a.set_plasticity(True, scaling_tau_ms=1000.0)
    b = NetOracle(cfg, pre, post, delay, w.astype(np.float32), w)
    b.set_plasticity(True, scaling_tau_ms=1000.0)
    s32, c32 = a.run(150)
    s64, _, _, _ = b.run64(150)
    assert c32[:, 0].sum() > 500
    np.testing.assert_array_equal(s32, s64)
    w32, w64 = a.plasticity_state()['weight'], b.plasticity_state(fp64=True)['weight']
    assert (w32 != w).sum() > 1000
    np.testing.assert_allclose(w32, w64, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize('bad', [dict(weight_kind=1), dict(storage=1, topology=2, weight_kind=1),
                                 dict(launch='resident'), dict(launch='fused'), dict(target_hz=0.0),
                                 dict(stdp_rate=-1.0), dict(plasticity=2)])
def test_learning_configuration_is_checked(bad):
    """The engine refuses learning where its arithmetic contract does not hold (fp16 weights,
    block storage, the fused and resident launch shapes) and invalid rates, on the host."""
    from neurogen_b200.network import Topology
    cfg = default_config(**dict(dict(n=256, n_exc=200, plasticity=1), **bad))
    with pytest.raises(ValueError):
        Topology(cfg)
