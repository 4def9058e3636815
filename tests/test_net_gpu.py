"""GPU parity of the isolated-tick network engine against the fp32 oracle.

The engine's contract is bit-exactness with oracle/net_oracle.c in its fp32 mode: every spike
of every tick, and the full state (V, adaptation, g_E, g_I, refractory, delay ring) after the
run.  Covered: Erdos-Renyi 8,192 (conductance drive, self-generated spikes), fixed fan-in and
16x16 block matrices with fp16 weights (imposed spikes), CSR and block storage of the same
block matrix, empty networks, explicit edge lists, the biology.py known-answer tests, and the
full N=262,144 configuration through size-independent properties.
"""
import numpy as np
import pytest

from neurogen_b200.network import Network, Topology, default_config, isolated_8k, scaled_262k
from oracle.net import NetOracle, unpack_spikes

pytestmark = pytest.mark.gpu

# 'resident' is the resident launch with its default tick; 'resident_pipe' and 'resident_serial'
# select the pipelined and the serial tick explicitly.
LAUNCH = {'fused': 1, 'split': 2, 'resident': 3, 'resident_pipe': 3, 'resident_serial': 3}
LAUNCHES = list(LAUNCH)


@pytest.fixture(autouse=True)
def resident_mode(request, monkeypatch):
    """Selects the resident tick (read at network creation) for tests parametrized by launch
    shape ('resident_pipe', 'resident_serial') or by mode ('pipe', 'serial')."""
    params = getattr(getattr(request.node, 'callspec', None), 'params', {})
    mode = {'resident_pipe': 'pipe', 'resident_serial': 'serial'}.get(params.get('launch'), params.get('mode'))
    if mode:
        monkeypatch.setenv('NEUROGEN_RESIDENT_MODE', mode)
    else:
        monkeypatch.delenv('NEUROGEN_RESIDENT_MODE', raising=False)


def run_both(cfg, ticks, state=None):
    topo = Topology(cfg)
    edges = topo.export()
    net = topo.network()
    orc = NetOracle(cfg, *edges)
    if state:
        net.set_state(**state)
        orc.set_state(**state)
    gs, gc = net.run(ticks)
    os_, oc = orc.run(ticks)
    return net, orc, (gs, gc), (os_, oc)


def assert_same_state(net, orc):
    a, b = net.get_state(), orc.get_state()
    for k in ('v', 'a', 'ge', 'gi', 'ref', 'ring'):
        assert np.array_equal(a[k], b[k]), k
    assert a['tick'] == b['tick']


@pytest.mark.parametrize('launch', LAUNCHES)
def test_isolated_8k_bit_exact_200_ticks(launch):
    cfg = isolated_8k()
    cfg.launch = LAUNCH[launch]
    net, orc, (gs, gc), (os_, oc) = run_both(cfg, 200)
    assert oc[:, 0].sum() > 1000
    np.testing.assert_array_equal(gs, os_)  # every spike of every tick
    np.testing.assert_array_equal(gc, oc)   # spikes and synaptic events per tick
    assert_same_state(net, orc)


@pytest.mark.parametrize('storage', ['csr', 'bsr'])
@pytest.mark.parametrize('launch', LAUNCHES)
def test_block_matrix_both_storages_bit_exact(storage, launch):
    cfg = default_config(n=4096, n_exc=3277, topology='bsr16', bsr_blocks=32, bsr_fill=64,
                         weight_kind='halfnormal_f16', w_mu=0.0, w_sigma=0.05, storage=storage,
                         drive_kind='imposed', drive_p=0.03, seed=4, launch=LAUNCH[launch])
    net, orc, (gs, gc), (os_, oc) = run_both(cfg, 60)
    np.testing.assert_array_equal(gs, os_)
    np.testing.assert_array_equal(gc, oc)
    assert_same_state(net, orc)


@pytest.mark.parametrize('launch', LAUNCHES)
def test_fixed_fanin_fp16_imposed_bit_exact(launch):
    cfg = default_config(n=16384, n_exc=13107, topology='fixed_fanin', fanin=128, weight_kind='halfnormal_f16',
                         w_mu=0.0, w_sigma=0.05, drive_kind='imposed', drive_p=0.05, seed=8,
                         launch=LAUNCH[launch])
    net, orc, (gs, gc), (os_, oc) = run_both(cfg, 40)
    np.testing.assert_array_equal(gs, os_)
    np.testing.assert_array_equal(gc, oc)
    assert_same_state(net, orc)


@pytest.mark.parametrize('launch', LAUNCHES)
def test_ragged_sizes_and_empty_network(launch):
    # n not a multiple of 32 (partial last warp) and an empty synapse set.
    cfg = default_config(n=1000, n_exc=777, p_connect=0.05, drive_ns=16.0, drive_p=0.05, seed=3,
                         launch=LAUNCH[launch])
    net, orc, (gs, gc), (os_, oc) = run_both(cfg, 50)
    np.testing.assert_array_equal(gs, os_)
    assert_same_state(net, orc)
    cfg0 = default_config(n=37, n_exc=30, p_connect=0.0, drive_ns=30.0, drive_p=0.2, seed=1, launch=LAUNCH[launch])
    net, orc, (gs, gc), (os_, oc) = run_both(cfg0, 20)
    assert Topology(cfg0).synapses == 0
    np.testing.assert_array_equal(gs, os_)
    assert_same_state(net, orc)


@pytest.mark.parametrize('excitatory', [True, False])
def test_delayed_transmission_known_answer(excitatory):
    cfg = default_config(n=4, n_exc=2, drive_p=0.0)
    pre = 0 if excitatory else 2
    w = 2.0 if excitatory else -2.0
    net = Network(cfg, edges=([pre], [1], [3], [w]))
    v = np.full(4, -65.0, np.float32)
    v[pre] = 0.0
    net.set_state(v=v)
    spikes, counts = net.run(3)
    assert unpack_spikes(spikes, 4)[0, pre] and counts[0, 1] == 1
    st = net.get_state()
    assert st['ge'].sum() == 0 and st['gi'].sum() == 0
    net.run(1)
    st = net.get_state()
    assert (st['ge'][1] if excitatory else st['gi'][1]) == 2.0


def test_passive_membrane_known_answer():
    for dt in (.25, .5, 1.):
        cfg = default_config(n=8, n_exc=6, drive_p=0.0, dt_ms=dt, bias_pa=100.0)
        net = Network(cfg, edges=([], [], [], []))
        net.run(round(10 / dt), record=False)
        np.testing.assert_allclose(net.get_state()['v'][:6], -55 - 10 * np.exp(-10 / 20), atol=2e-4)


def test_state_roundtrip_and_resume():
    cfg = isolated_8k(seed=2)
    topo = Topology(cfg)
    a, b = topo.network(), topo.network()
    a.run(30)
    st = a.get_state()
    b.set_state(**{k: st[k] for k in ('v', 'a', 'ge', 'gi', 'ref', 'ring')}, tick=st['tick'])
    sa, _ = a.run(40)
    sb, _ = b.run(40)
    np.testing.assert_array_equal(sa, sb)


def test_scaled_262k_csr_properties():
    """Full-size configuration: spike counts follow Bernoulli(p), every synaptic event is
    delivered (ring mass conservation), and the first ticks are bit-exact with the oracle."""
    cfg = scaled_262k('csr', rate=0.03)
    topo = Topology(cfg)
    edges = topo.export()
    net = topo.network()
    orc = NetOracle(cfg, *edges)
    gs, gc = net.run(6)
    os_, oc = orc.run(6)
    np.testing.assert_array_equal(gs, os_)
    np.testing.assert_array_equal(gc, oc)
    assert_same_state(net, orc)
    p = gc[:, 0] / cfg.n
    assert np.all(np.abs(p - 0.03) < 5 * np.sqrt(0.03 * 0.97 / cfg.n))
    # Mass conservation: after a run, the ring holds exactly the fixed-point sum of every
    # weight emitted and not yet delivered.
    fired = unpack_spikes(gs, cfg.n)
    pre, post, delay, w = edges
    q = np.round(np.abs(w.astype(np.float64)) * 2 ** 24).astype(np.int64)
    pending = 0
    for k in range(6):
        sel = fired[k][pre] & (k + delay >= 6)
        pending += q[sel].sum()
    assert net.get_state()['ring'].astype(np.int64).sum() == pending


@pytest.mark.parametrize('launch', LAUNCHES)
def test_graph_replay_equals_recorded_run(launch):
    """The graph path (no per-tick outputs, device tick counter) and the recorded path give the
    same state, totals and trajectory, including a run length that is not a multiple of the
    graph length and a resume from an arbitrary tick."""
    cfg = isolated_8k(seed=5)
    cfg.launch = LAUNCH[launch]
    topo = Topology(cfg)
    a, b = topo.network(), topo.network()
    _, ca = a.run(150)
    b.run_device(150)
    sa, sb = a.get_state(), b.get_state()
    for k in ('v', 'a', 'ge', 'gi', 'ref', 'ring'):
        assert np.array_equal(sa[k], sb[k]), k
    assert sa['tick'] == sb['tick'] == 150
    assert b.stats() == (int(ca[:, 0].sum()), int(ca[:, 1].sum()))
    b.run_device(70)
    _, _ = a.run(70)
    sa, sb = a.get_state(), b.get_state()
    assert all(np.array_equal(sa[k], sb[k]) for k in ('v', 'a', 'ge', 'gi', 'ref', 'ring'))
    # Resume from an odd tick: graph replays start on even ticks, so one tick runs before them.
    b.run_device(131)
    _, _ = a.run(131)
    sa, sb = a.get_state(), b.get_state()
    assert sa['tick'] == sb['tick'] == 351
    assert all(np.array_equal(sa[k], sb[k]) for k in ('v', 'a', 'ge', 'gi', 'ref', 'ring'))


def test_pipelined_graph_full_size():
    """N=262,144 fixed fan-in: the graph path (delay>=2 pushes on a second stream beside the next
    tick) ends in the same state and totals as the recorded path, which runs every push whole and
    in order on one stream."""
    cfg = scaled_262k('csr', rate=0.05)
    cfg.launch = LAUNCH['split']
    topo = Topology(cfg)
    a, b = topo.network(), topo.network()
    assert a.launch == 'split'
    _, ca = a.run(3 + 1 + 2 * 64)
    b.run_device(3)
    b.run_device(1 + 2 * 64)  # from tick 3: one direct tick, then two graph replays
    sa, sb = a.get_state(), b.get_state()
    for k in ('v', 'a', 'ge', 'gi', 'ref', 'ring'):
        assert np.array_equal(sa[k], sb[k]), k
    assert b.stats() == (int(ca[:, 0].sum()), int(ca[:, 1].sum()))


@pytest.mark.parametrize('mode', ['pipe', 'serial'])
@pytest.mark.parametrize('storage', ['csr', 'bsr'])
def test_resident_full_size_equals_split(storage, mode):
    """N=262,144 at 5%, fixed fan-in CSR or 16x16 blocks: the resident launch (state and ring in
    shared memory, owner blocks with overflow chains, built from either storage) gives every spike,
    count and state bit of the split launch, across launch boundaries (2,048 ticks a launch) and a
    resume from an odd tick."""
    cfg = scaled_262k(storage, rate=0.05)
    topo = Topology(cfg)
    cfg_split = scaled_262k(storage, rate=0.05)
    cfg_split.launch = LAUNCH['split']
    res, ref = topo.network(), Topology(cfg_split).network()
    assert res.launch == 'resident' and ref.launch == 'split'
    gs, gc = res.run(37)
    rs, rc = ref.run(37)
    np.testing.assert_array_equal(gs, rs)
    np.testing.assert_array_equal(gc, rc)
    res.run_device(2100)
    ref.run_device(2100)
    sa, sb = res.get_state(), ref.get_state()
    for k in ('v', 'a', 'ge', 'gi', 'ref', 'ring'):
        assert np.array_equal(sa[k], sb[k]), k
    assert sa['tick'] == sb['tick'] == 2137
    assert res.stats() == ref.stats()


def test_auto_launch_choice():
    assert Topology(isolated_8k()).network().launch == 'resident'
    assert Topology(scaled_262k('bsr', rate=0.03)).network().launch == 'resident'
    small = default_config(n=1000, launch='split')
    assert Topology(small).network().launch == 'split'


def edges_sorted(edges):
    pre, post, delay, w = edges
    order = np.lexsort((w.view(np.uint32), delay, post, pre))
    return pre[order], post[order], delay[order], w[order]


def test_device_generated_fanin_equals_host_generated():
    """ng_net_create draws fixed fan-in fp16 networks on the device: the same synapses as the host
    generator (ng_topology_create) and, run side by side, every spike and state bit."""
    cfg = default_config(n=16384, n_exc=13107, topology='fixed_fanin', fanin=128, weight_kind='halfnormal_f16',
                         w_mu=0.0, w_sigma=0.05, drive_kind='imposed', drive_p=0.05, seed=8)
    dev, host = Network(cfg), Topology(cfg).network()
    assert dev.synapses == host.synapses == 16384 * 128
    for a, b in zip(edges_sorted(dev.export()), edges_sorted(host.export())):
        assert np.array_equal(a, b)
    ds, dc = dev.run(40)
    hs, hc = host.run(40)
    np.testing.assert_array_equal(ds, hs)
    np.testing.assert_array_equal(dc, hc)
    a, b = dev.get_state(), host.get_state()
    for k in ('v', 'a', 'ge', 'gi', 'ref', 'ring'):
        assert np.array_equal(a[k], b[k]), k


def test_device_generation_checks_the_ring_range():
    cfg = default_config(n=4096, n_exc=3276, topology='fixed_fanin', fanin=512, weight_kind='halfnormal_f16',
                         w_mu=0.0, w_sigma=2.0, seed=3)
    with pytest.raises(ValueError, match='fixed-point range'):
        Topology(cfg)
    with pytest.raises(ValueError, match='fixed-point range'):
        Network(cfg)


STALL_CHILD = r'''
import os, sys
sys.path[:0] = [{root!r}, {pkg!r}]
from neurogen_b200.network import Network, Topology, isolated_8k
os.environ['NEUROGEN_TEST_RESIDENT_STALL'] = '1'
net = Topology(isolated_8k()).network()
assert net.launch == 'resident'
try:
    net.run(10)
except ValueError as e:
    print('raised:', e)
del os.environ['NEUROGEN_TEST_RESIDENT_STALL']
ok = Topology(isolated_8k()).network()   # the context is still usable
s, c = ok.run(20)
print('after:', int(c[:, 0].sum()))
'''


@pytest.mark.parametrize('mode', ['pipe', 'serial'])
def test_resident_barrier_wait_runs_out_cleanly(tmp_path, mode):
    """The grid barrier's wait is bounded: with an unreachable target every CTA gives up after its
    limit, the host raises, and the same process creates and runs a new network afterwards."""
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    script = tmp_path / 'stall.py'
    script.write_text(STALL_CHILD.format(root=str(root), pkg=str(root / 'neurogen-2.5_b200')))
    out = subprocess.run([sys.executable, str(script)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr[-3000:]
    assert 'raised:' in out.stdout and 'timed out' in out.stdout
    assert 'after:' in out.stdout and int(out.stdout.split('after:')[1]) > 0


def test_split_push_shapes_agree_at_one_million_neurons(monkeypatch):
    """The split push's CTA span (8 or 64 bitmask words) and per-lane chunk (8 or 16 synapses)
    change only the work layout: a 1,048,576-neuron network gives the same spikes, counts and
    state for every combination."""
    cfg = default_config(n=1048576, n_exc=838860, topology='fixed_fanin', fanin=24, weight_kind='halfnormal_f16',
                         w_mu=0.0, w_sigma=0.05, drive_kind='imposed', drive_p=0.02, seed=9, launch='split')
    results = []
    for span in ('8', '64'):
        for chunk in ('8', '16'):
            monkeypatch.setenv('NEUROGEN_PUSH_SPAN', span)
            monkeypatch.setenv('NEUROGEN_PUSH_CHUNK', chunk)
            net = Network(cfg)
            s, c = net.run(12)
            net.run_device(70)
            results.append((s, c, net.get_state(), net.stats()))
            del net
    s0, c0, st0, t0 = results[0]
    assert c0[:, 1].sum() > 0
    for s, c, st, tot in results[1:]:
        np.testing.assert_array_equal(s, s0)
        np.testing.assert_array_equal(c, c0)
        for k in ('v', 'a', 'ge', 'gi', 'ref', 'ring'):
            assert np.array_equal(st[k], st0[k]), k
        assert tot == t0
