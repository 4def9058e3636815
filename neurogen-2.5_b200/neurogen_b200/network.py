"""Isolated-tick spiking network on the B200 engine (include/neurogen_b200.h part 4).

A conductance-based adaptive LIF network with per-synapse integer delays: the equations of
the reference's NumPy simulator step (neurogen/biology.py:132-180) with frozen synapses, run as
one fused CUDA launch per tick (ALIF update, warp-ballot spike bitmask, spike-driven push of
CSR or 16x16-block synapses into an E/I delay ring).
"""
import ctypes as ct

import numpy as np

from ._lib import library, NetConfig, ptr

RING = 16
TOPO = {'erdos_renyi': 0, 'fixed_fanin': 1, 'bsr16': 2}
WEIGHTS = {'lognormal_f32': 0, 'halfnormal_f16': 1}
DRIVE = {'conductance': 0, 'imposed': 1}


def default_config(**overrides):
    """ng_net_default_config() with keyword overrides (string enums accepted)."""
    cfg = NetConfig()
    library().ng_net_default_config(ct.byref(cfg))
    for key, value in overrides.items():
        if key == 'topology' and isinstance(value, str):
            value = TOPO[value]
        elif key == 'weight_kind' and isinstance(value, str):
            value = WEIGHTS[value]
        elif key == 'drive_kind' and isinstance(value, str):
            value = DRIVE[value]
        elif key == 'storage' and isinstance(value, str):
            value = {'csr': 0, 'bsr': 1}[value]
        elif key == 'launch' and isinstance(value, str):
            value = {'auto': 0, 'fused': 1, 'split': 2, 'resident': 3}[value]
        if not hasattr(cfg, key):
            raise KeyError(key)
        setattr(cfg, key, value)
    return cfg


# Workloads quoted by the benchmark configuration (sizes, distributions, drive).
def isolated_8k(seed=0):
    """N=8,192 (80% E), Erdos-Renyi 2%, lognormal(-2, 0.5) fp32 weights, delays 1-8,
    Bernoulli(0.02) conductance drive of 16 nS per event (puts the rate at ~2%); tau_m =
    C/gL = 20 ms, tau_a = 200 ms, dt = 1 ms."""
    return default_config(n=8192, n_exc=6553, topology='erdos_renyi', p_connect=0.02,
                          weight_kind='lognormal_f32', w_mu=-2.0, w_sigma=0.5, delay_min=1,
                          delay_max=8, seed=seed, drive_kind='conductance', drive_p=0.02,
                          drive_ns=16.0)


def scaled_262k(storage='csr', rate=0.03, seed=0):
    """N=262,144, fan-in 512 uniform (CSR) or 16x16 blocks with 128 block-columns per
    block-row at 25% fill (BSR), fp16 |N(0, 0.05)| weights with E/I sign, delays 1-8, spikes
    imposed Bernoulli(rate) per neuron per tick."""
    n = 262144
    common = dict(n=n, n_exc=int(n * 0.8), weight_kind='halfnormal_f16', w_mu=0.0, w_sigma=0.05,
                  delay_min=1, delay_max=8, seed=seed, drive_kind='imposed', drive_p=rate)
    if storage == 'csr':
        return default_config(topology='fixed_fanin', fanin=512, storage='csr', **common)
    return default_config(topology='bsr16', bsr_blocks=128, bsr_fill=64,
                          storage='bsr' if storage == 'bsr' else 'csr', **common)


def partitioned_4m(rank=0, world=1, rate=0.01, seed=0):
    """N=4,194,304 neurons, fan-in 1,000 uniform (fp16 |N(0, 0.05)| with E/I sign), delays 1-8,
    imposed Bernoulli(rate) spikes; rows partitioned over `world` GPUs."""
    n = 4194304
    return default_config(n=n, n_exc=int(n * 0.8), topology='fixed_fanin', fanin=1000,
                          weight_kind='halfnormal_f16', w_mu=0.0, w_sigma=0.05, delay_min=1, delay_max=8,
                          seed=seed, drive_kind='imposed', drive_p=rate, part_rank=rank,
                          part_world=world if world > 1 else 0)


def nccl_unique_id():
    """A fresh 128-byte NCCL unique id (make it on one rank, share it with the others)."""
    buf = ct.create_string_buffer(128)
    if library().ng_nccl_unique_id(buf):
        raise ValueError(library().ng_error().decode())
    return bytes(buf.raw)


class Network:
    """One network on the current CUDA device (owns its synapses, state and stream)."""

    def __init__(self, cfg, edges=None):
        self.lib = library()
        self.cfg = cfg
        if edges is None:
            self.h = self.lib.ng_net_create(ct.byref(cfg))
        else:
            pre, post, delay, weight = (np.ascontiguousarray(x, dt) for x, dt in zip(
                edges, (np.int32, np.int32, np.int32, np.float32)))
            self.h = self.lib.ng_net_create_edges(ct.byref(cfg), len(pre), pre, post, delay, weight)
        if not self.h:
            raise ValueError(self.lib.ng_error().decode())
        self.n = cfg.n
        self.words = (self.n + 31) // 32

    @classmethod
    def partitioned(cls, cfg, nccl_id):
        """This rank's partition (cfg.part_rank of cfg.part_world); collective over the ranks."""
        net = cls.__new__(cls)
        net.lib = library()
        net.cfg = cfg
        idbuf = ct.create_string_buffer(bytes(nccl_id), 128)
        net.h = net.lib.ng_net_create_partitioned(ct.byref(cfg), idbuf)
        if not net.h:
            raise ValueError(net.lib.ng_error().decode())
        net.n = cfg.n // cfg.part_world
        net.words = (cfg.n + 31) // 32
        return net

    def close(self):
        if getattr(self, 'h', None):
            self.lib.ng_net_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def _check(self, code):
        if code:
            raise ValueError(self.lib.ng_error().decode())

    @property
    def synapses(self):
        return self.lib.ng_net_synapses(self.h)

    @property
    def launch(self):
        """Launch shape in use: 'fused', 'split' or 'resident'."""
        return {1: 'fused', 2: 'split', 3: 'resident', 4: 'resident'}[self.lib.ng_net_launch_kind(self.h)]

    @property
    def exchange(self):
        """How a partitioned network's ranks exchange spikes: None, 'nccl' or 'peer'."""
        return {0: None, 1: 'nccl', 2: 'peer'}[self.lib.ng_net_exchange_kind(self.h)]

    @property
    def resident_tick(self):
        """The resident launch's tick: 'pipelined' or 'serial' (None for the other launch shapes)."""
        return {3: 'serial', 4: 'pipelined'}.get(self.lib.ng_net_launch_kind(self.h))

    def plasticity_state(self):
        """Learning state (plasticity networks): per contact in export() order the pre trace,
        potential trace, coactivity and usage; per neuron the post trace and the rate (Hz)."""
        m, n = self.synapses, self.n
        per_edge = {k: np.empty(m, np.float32) for k in ('pre_trace', 'potential_trace', 'coactivity', 'usage')}
        post_tr, rate = np.empty(n, np.float32), np.empty(n, np.float32)
        self._check(self.lib.ng_net_plasticity_state(self.h, *[x.ctypes.data for x in per_edge.values()],
                                                     post_tr.ctypes.data, rate.ctypes.data))
        return dict(per_edge, post_trace=post_tr, rate=rate)

    def export(self):
        m = self.synapses
        pre, post, delay = (np.empty(m, np.int32) for _ in range(3))
        weight = np.empty(m, np.float32)
        self._check(self.lib.ng_net_export(self.h, pre, post, delay, weight))
        return pre, post, delay, weight

    def set_state(self, v=None, a=None, ge=None, gi=None, ref=None, ring=None, tick=0):
        arrs = [None if x is None else np.ascontiguousarray(x, dt) for x, dt in
                ((v, np.float32), (a, np.float32), (ge, np.float32), (gi, np.float32),
                 (ref, np.int32), (ring, np.int32))]
        self._check(self.lib.ng_net_set_state(self.h, *[ptr(x) for x in arrs], tick))

    def get_state(self):
        n = self.n
        v, a, ge, gi = (np.zeros(n, np.float32) for _ in range(4))
        ref = np.zeros(n, np.int32)
        ring = np.zeros((RING, n, 2), np.int32)
        tick = np.zeros(1, np.int64)
        self._check(self.lib.ng_net_get_state(self.h, ptr(v), ptr(a), ptr(ge), ptr(gi), ptr(ref),
                                              ptr(ring), ptr(tick)))
        return dict(v=v, a=a, ge=ge, gi=gi, ref=ref, ring=ring, tick=int(tick[0]))

    def stats(self):
        """(spikes, synaptic events) delivered since creation."""
        out = np.zeros(2, np.int64)
        self._check(self.lib.ng_net_stats(self.h, out))
        return int(out[0]), int(out[1])

    def run_device(self, ticks, stream=0):
        """Enqueue ticks on a CUDA stream handle (graph replay; no host copies)."""
        self._check(self.lib.ng_net_run_device(self.h, ticks, None, None, stream or None))

    def run(self, ticks, record=True):
        """-> (spike words uint32 [ticks, words] or None, counts int64 [ticks, 2])."""
        spikes = np.zeros((ticks, self.words), np.uint32) if record else None
        counts = np.zeros((ticks, 2), np.int64)
        self._check(self.lib.ng_net_run(self.h, ticks, ptr(spikes), ptr(counts)))
        return spikes, counts


class Topology:
    """Host-only generated synapses (no GPU): the exact synapses ``Network(cfg)`` builds."""

    def __init__(self, cfg):
        self.lib = library()
        self.cfg = cfg
        self.h = self.lib.ng_topology_create(ct.byref(cfg))
        if not self.h:
            raise ValueError(self.lib.ng_error().decode())

    def __del__(self):
        if getattr(self, 'h', None):
            self.lib.ng_topology_destroy(self.h)
            self.h = None

    @property
    def synapses(self):
        return self.lib.ng_topology_synapses(self.h)

    def export(self):
        m = self.synapses
        pre, post, delay = (np.empty(m, np.int32) for _ in range(3))
        weight = np.empty(m, np.float32)
        if self.lib.ng_topology_export(self.h, pre, post, delay, weight):
            raise ValueError(self.lib.ng_error().decode())
        return pre, post, delay, weight

    def network(self):
        """Upload these synapses to the current CUDA device."""
        net = Network.__new__(Network)
        net.lib = self.lib
        net.cfg = self.cfg
        net.h = self.lib.ng_net_create_topology(self.h)
        if not net.h:
            raise ValueError(self.lib.ng_error().decode())
        net.n = self.cfg.n
        net.words = (net.n + 31) // 32
        return net
