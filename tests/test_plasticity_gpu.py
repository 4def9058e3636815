"""GPU learning (biology.py:182-218) against the oracle's fp32 contract, bit for bit.

The network engine with cfg.plasticity = 1 learns every tick between the membrane update and the
tick's emissions (k_net_learn, k_net_post): STDP on E contacts, the inhibitory rule on I->E
contacts, synaptic scaling, weight clipping and the traces.  Every spike, the neuron state and
delay ring, every learned weight and every trace must equal oracle/net_oracle.c's (which is
pinned to the reference simulator in tests/test_oracle_plasticity.py).
"""
import numpy as np
import pytest

from conftest import ROOT
from neurogen_b200.network import Network, Topology, default_config
from oracle.net import NetOracle

pytestmark = pytest.mark.gpu

STATE_KEYS = ('v', 'a', 'ge', 'gi', 'ref', 'ring')
TRACES = ('pre_trace', 'potential_trace', 'coactivity', 'usage')


def plastic_config(**kw):
    base = dict(n=2048, n_exc=1638, p_connect=0.03, w_mu=0.4, w_sigma=0.2, drive_kind='conductance',
                drive_p=0.03, drive_ns=12.0, seed=6, plasticity=1, scaling_tau_ms=2000.0)
    base.update(kw)
    return default_config(**base)


def oracle_for(cfg, edges):
    orc = NetOracle(cfg, *edges)
    orc.set_plasticity(True, stdp_rate=cfg.stdp_rate, inhibitory_rate=cfg.inhibitory_rate,
                       target_hz=cfg.target_hz, scaling_tau_ms=cfg.scaling_tau_ms)
    return orc


def assert_same_learning(net, orc, edges):
    """State, learned weights and traces equal; contacts matched by (pre, post, delay), since
    the engine stores a row's delay-1 contacts first.  Returns the learned weights in input order."""
    a, b = net.get_state(), orc.get_state()
    for k in STATE_KEYS:
        assert np.array_equal(a[k], b[k]), k
    ex = net.export()
    k_gpu = np.lexsort((ex[2], ex[1], ex[0]))
    k_in = np.lexsort((edges[2], edges[1], edges[0]))
    got, want = net.plasticity_state(), orc.plasticity_state()
    np.testing.assert_array_equal(ex[3][k_gpu], want['weight'][k_in])
    for k in TRACES:
        np.testing.assert_array_equal(got[k][k_gpu], want[k][k_in], err_msg=k)
    for k in ('post_trace', 'rate'):
        np.testing.assert_array_equal(got[k], want[k], err_msg=k)
    w = np.empty_like(want['weight'])
    w[k_in] = ex[3][k_gpu]
    return w


def test_learning_bit_exact_200_ticks():
    cfg = plastic_config()
    topo = Topology(cfg)
    edges = topo.export()
    net = topo.network()
    assert net.launch == 'split'
    orc = oracle_for(cfg, edges)
    for _ in range(2):
        gs, gc = net.run(100)
        os_, oc = orc.run(100)
        np.testing.assert_array_equal(gs, os_)   # every spike of every tick
        np.testing.assert_array_equal(gc, oc)    # spikes and delivered events per tick
    w = assert_same_learning(net, orc, edges)
    assert gc[:, 0].sum() > 1000
    changed = (w != edges[3]).sum()
    assert changed > 0.5 * len(w), changed      # most contacts learned
    assert np.abs(w[edges[0] < cfg.n_exc]).max() <= 4.0 and np.abs(w).min() >= 0.01


def test_learning_graph_replay_equals_recorded_run():
    """The graph path (no per-tick outputs) gives the learning state of the recorded path,
    including a run length that is not a multiple of the graph and an odd start tick."""
    cfg = plastic_config(seed=8)
    topo = Topology(cfg)
    a, b = topo.network(), topo.network()
    a.run(1 + 2 * 64 + 7)
    b.run_device(1)
    b.run_device(2 * 64 + 7)
    sa, sb = a.get_state(), b.get_state()
    for k in STATE_KEYS:
        assert np.array_equal(sa[k], sb[k]), k
    assert np.array_equal(a.export()[3], b.export()[3])
    pa, pb = a.plasticity_state(), b.plasticity_state()
    for k in pa:
        assert np.array_equal(pa[k], pb[k]), k


def test_learning_on_the_reference_anatomy():
    """The reference simulator's own 384-cell anatomy and initial weights (the golden network of
    tests/golden/make_net_plastic_golden.py, Bernoulli conductance drive in place of its
    current): 300 ticks bit-exact with the oracle, weights and traces included."""
    g = np.load(ROOT / 'tests' / 'golden' / 'net_plastic_golden.npz')
    cfg = default_config(n=int(g['n']), n_exc=int(g['n_exc']), drive_kind='conductance', drive_p=0.05,
                         drive_ns=20.0, seed=2, plasticity=1, launch='split')
    edges = (g['pre'], g['post'], g['delay'], g['weight'].astype(np.float32))
    net = Network(cfg, edges=edges)
    orc = oracle_for(cfg, edges)
    v0 = g['v0'].astype(np.float32)
    net.set_state(v=v0)
    orc.set_state(v=v0)
    gs, gc = net.run(300)
    os_, oc = orc.run(300)
    np.testing.assert_array_equal(gs, os_)
    np.testing.assert_array_equal(gc, oc)
    assert gc[:, 0].sum() > 300
    assert_same_learning(net, orc, edges)
