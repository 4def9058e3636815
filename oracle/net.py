"""ORACLE (test infrastructure only): ctypes access to oracle/net_oracle.c.

``NetOracle`` runs the conductance ALIF network with per-synapse delays on the CPU, in the
fp32 arithmetic contract of the CUDA engine (bit-exact target) or in fp64 (pinned to the
reference's neurogen/biology.py).  Only tests/, ``__graft_entry__.smoke()`` and bench.py's
CPU-baseline leg use this module.
"""
import ctypes as ct
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
RING = 16


class Params(ct.Structure):
    _fields_ = [('n', ct.c_int32), ('n_exc', ct.c_int32), ('dt', ct.c_float), ('cap_e', ct.c_float),
                ('cap_i', ct.c_float), ('g_leak', ct.c_float), ('e_leak', ct.c_float),
                ('e_inh', ct.c_float), ('v_th', ct.c_float), ('v_reset', ct.c_float),
                ('t_ref', ct.c_float), ('tau_e', ct.c_float), ('tau_i', ct.c_float),
                ('tau_a', ct.c_float), ('adapt_inc', ct.c_float), ('bias', ct.c_float),
                ('drive_kind', ct.c_int32), ('drive_p', ct.c_float), ('drive_ns', ct.c_float),
                ('seed', ct.c_uint64)]


def params_from(cfg):
    """Oracle parameters from an ng_net_config (ctypes struct) or a dict of the same names."""
    g = (lambda k: getattr(cfg, k)) if not isinstance(cfg, dict) else cfg.__getitem__
    return Params(g('n'), g('n_exc'), g('dt_ms'), g('cap_exc_pf'), g('cap_inh_pf'), g('g_leak_ns'),
                  g('e_leak_mv'), g('e_inh_mv'), g('v_thresh_mv'), g('v_reset_mv'), g('t_ref_ms'),
                  g('tau_exc_ms'), g('tau_inh_ms'), g('tau_adapt_ms'), g('adapt_inc_pa'),
                  g('bias_pa'), g('drive_kind'), g('drive_p'), g('drive_ns'), g('seed'))


def _p(a):
    return None if a is None else a.ctypes.data_as(ct.c_void_p)


# Defaults of the engine's network configuration (biology.py's BiologyConfig and membrane
# constants, biology.py:19-77, 153-170), restated here so that the CPU legs need no CUDA library.
DEFAULTS = dict(n=1024, n_exc=819, topology=0, p_connect=0.02, fanin=512, bsr_blocks=128, bsr_fill=64,
                weight_kind=0, w_mu=-2.0, w_sigma=0.5, delay_min=1, delay_max=8, seed=0, dt_ms=1.0,
                cap_exc_pf=200.0, cap_inh_pf=100.0, g_leak_ns=10.0, e_leak_mv=-65.0, e_inh_mv=-80.0,
                v_thresh_mv=-50.0, v_reset_mv=-65.0, t_ref_ms=2.0, tau_exc_ms=5.0, tau_inh_ms=10.0,
                tau_adapt_ms=200.0, adapt_inc_pa=15.0, bias_pa=0.0, drive_kind=0, drive_p=0.02, drive_ns=4.0,
                storage=0, launch=0, part_rank=0, part_world=0, plasticity=0, stdp_rate=.005,
                inhibitory_rate=.002, target_hz=5.0, scaling_tau_ms=1e5)


def config(**overrides):
    """A network configuration as a dict of the engine's field names."""
    unknown = set(overrides) - set(DEFAULTS)
    if unknown:
        raise KeyError(sorted(unknown))
    return dict(DEFAULTS, **overrides)


# The benchmark workloads (sizes, distributions and drive of the benchmark configurations).
def isolated_8k(seed=0):
    return config(n=8192, n_exc=6553, topology=0, p_connect=0.02, weight_kind=0, w_mu=-2.0, w_sigma=0.5,
                  seed=seed, drive_kind=0, drive_p=0.02, drive_ns=16.0)


def scaled_262k(storage='csr', rate=0.03, seed=0):
    n = 262144
    common = dict(n=n, n_exc=int(n * 0.8), weight_kind=1, w_mu=0.0, w_sigma=0.05, seed=seed, drive_kind=1,
                  drive_p=rate)
    if storage == 'csr':
        return config(topology=1, fanin=512, storage=0, **common)
    return config(topology=2, bsr_blocks=128, bsr_fill=64, storage=1 if storage == 'bsr' else 0, **common)


def partitioned_4m(rate=0.01, seed=0, scale=1):
    n = 4194304 // scale
    return config(n=n, n_exc=int(n * 0.8), topology=1, fanin=1000, weight_kind=1, w_mu=0.0, w_sigma=0.05,
                  seed=seed, drive_kind=1, drive_p=rate)


class TopoConfig(ct.Structure):
    _fields_ = [('n', ct.c_int32), ('n_exc', ct.c_int32), ('topology', ct.c_int32), ('p_connect', ct.c_float),
                ('fanin', ct.c_int32), ('bsr_blocks', ct.c_int32), ('bsr_fill', ct.c_int32),
                ('weight_kind', ct.c_int32), ('w_mu', ct.c_float), ('w_sigma', ct.c_float),
                ('delay_min', ct.c_int32), ('delay_max', ct.c_int32), ('seed', ct.c_uint64)]


def _get(cfg, k):
    return cfg[k] if isinstance(cfg, dict) else getattr(cfg, k)


def generate(cfg, exact=False):
    """Synapses of a generated network (oracle/net_topo.c, the engine's draws restated) ->
    (pre, post, delay, weight fp32[, unrounded weight fp64]) in some fixed order."""
    lib = ct.CDLL(str(HERE / 'liboracle.so'))
    lib.ot_count.restype = ct.c_int64
    lib.ot_count.argtypes = [ct.POINTER(TopoConfig)]
    lib.ot_fill.argtypes = [ct.POINTER(TopoConfig)] + [ct.c_void_p] * 5
    tc = TopoConfig(*[_get(cfg, k) for k, _ in TopoConfig._fields_])
    m = lib.ot_count(ct.byref(tc))
    pre, post, delay = (np.empty(m, np.int32) for _ in range(3))
    w = np.empty(m, np.float32)
    w64 = np.empty(m, np.float64) if exact else None
    lib.ot_fill(ct.byref(tc), _p(pre), _p(post), _p(delay), _p(w), _p(w64))
    return (pre, post, delay, w, w64) if exact else (pre, post, delay, w)


class NetOracle:
    def __init__(self, cfg, pre, post, delay, weight, weight64=None):
        """weight: the fp32-contract weights; weight64 (optional): the fp64 mode's weights
        (default: the same values)."""
        lib = self.lib = ct.CDLL(str(HERE / 'liboracle.so'))
        lib.on_create.restype = ct.c_void_p
        lib.on_create.argtypes = [ct.POINTER(Params), ct.c_int64] + [ct.c_void_p] * 4
        lib.on_create_w.restype = ct.c_void_p
        lib.on_create_w.argtypes = [ct.POINTER(Params), ct.c_int64] + [ct.c_void_p] * 5
        lib.on_destroy.argtypes = [ct.c_void_p]
        lib.on_run.argtypes = [ct.c_void_p, ct.c_int, ct.c_void_p, ct.c_void_p]
        lib.on_run_mt.argtypes = [ct.c_void_p, ct.c_int, ct.c_void_p]
        lib.on_run64.argtypes = [ct.c_void_p, ct.c_int] + [ct.c_void_p] * 5
        lib.on_set_state.argtypes = [ct.c_void_p] + [ct.c_void_p] * 6 + [ct.c_int64]
        lib.on_get_state.argtypes = [ct.c_void_p] + [ct.c_void_p] * 7
        lib.on_set_state64.argtypes = [ct.c_void_p] + [ct.c_void_p] * 5
        lib.on_set_plasticity.argtypes = [ct.c_void_p, ct.POINTER(Plastic)]
        lib.on_learn_probe.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_void_p, ct.c_int]
        lib.on_get_plasticity.argtypes = [ct.c_void_p] + [ct.c_void_p] * 7
        lib.on_get_plasticity64.argtypes = [ct.c_void_p] + [ct.c_void_p] * 7
        self.params = params_from(cfg)
        self.n = self.params.n
        self.words = (self.n + 31) // 32
        self._keep = [np.ascontiguousarray(x, dt) for x, dt in
                      ((pre, np.int32), (post, np.int32), (delay, np.int32), (weight, np.float32),
                       (weight if weight64 is None else weight64, np.float64))]
        self.h = lib.on_create_w(ct.byref(self.params), len(self._keep[0]), *[_p(x) for x in self._keep])
        # Contacts are stored by presynaptic cell, stable in input order.
        self.order = np.argsort(self._keep[0], kind='stable')

    def __del__(self):
        if getattr(self, 'h', None):
            self.lib.on_destroy(self.h)

    def run(self, ticks):
        """fp32 contract -> (spike words uint32 [ticks, words], counts int64 [ticks, 2])."""
        spikes = np.zeros((ticks, self.words), np.uint32)
        counts = np.zeros((ticks, 2), np.int64)
        self.lib.on_run(self.h, ticks, _p(spikes), _p(counts))
        return spikes, counts

    def run_mt(self, ticks):
        """on_run on all OpenMP threads (identical results) -> counts int64 [ticks, 2]."""
        counts = np.zeros((ticks, 2), np.int64)
        self.lib.on_run_mt(self.h, ticks, _p(counts))
        return counts

    def run64(self, ticks, current=None):
        """fp64 equations -> (spike words, v [ticks, n], ge, gi)."""
        spikes = np.zeros((ticks, self.words), np.uint32)
        v = np.zeros((ticks, self.n))
        ge = np.zeros((ticks, self.n))
        gi = np.zeros((ticks, self.n))
        cur = None if current is None else np.ascontiguousarray(current, np.float64)
        self.lib.on_run64(self.h, ticks, _p(cur), _p(spikes), _p(v), _p(ge), _p(gi))
        return spikes, v, ge, gi

    def set_state(self, v=None, a=None, ge=None, gi=None, ref=None, ring=None, tick=0):
        arrs = [None if x is None else np.ascontiguousarray(x, dt) for x, dt in
                ((v, np.float32), (a, np.float32), (ge, np.float32), (gi, np.float32),
                 (ref, np.int32), (ring, np.int32))]
        self.lib.on_set_state(self.h, *[_p(x) for x in arrs], tick)

    def set_state64(self, v=None, a=None, ge=None, gi=None, ref=None):
        arrs = [None if x is None else np.ascontiguousarray(x, np.float64) for x in (v, a, ge, gi, ref)]
        self.lib.on_set_state64(self.h, *[_p(x) for x in arrs])

    def get_state(self):
        n = self.n
        v, a, ge, gi = (np.zeros(n, np.float32) for _ in range(4))
        ref = np.zeros(n, np.int32)
        ring = np.zeros((RING, n, 2), np.int32)
        tick = np.zeros(1, np.int64)
        self.lib.on_get_state(self.h, _p(v), _p(a), _p(ge), _p(gi), _p(ref), _p(ring), _p(tick))
        return dict(v=v, a=a, ge=ge, gi=gi, ref=ref, ring=ring, tick=int(tick[0]))


    # ---- plasticity (oracle/net_oracle.c: biology.py:182-218 learn) ----
    def set_plasticity(self, on=True, stdp_rate=.005, inhibitory_rate=.002, target_hz=5.0, scaling_tau_ms=1e5):
        """Learning every tick from now on (traces start at zero); on=False keeps the weights and
        still updates the traces, as biology.py does with plasticity off."""
        self.lib.on_set_plasticity(self.h, ct.byref(Plastic(int(on), stdp_rate, inhibitory_rate, target_hz,
                                                            scaling_tau_ms)))

    def learn_probe(self, arrivals, spikes, fp64=False):
        """One learn() step with given arrival flags (per contact, input order) and spikes (per
        cell), the reference's probe of its rule."""
        arr = np.zeros(len(self.order), np.uint8)
        arr[:] = np.asarray(arrivals, bool)[self.order]
        spk = np.ascontiguousarray(spikes, np.uint8)
        self.lib.on_learn_probe(self.h, _p(arr), _p(spk), int(fp64))

    def plasticity_state(self, fp64=False):
        """Weights and traces per contact in input order, post trace and rate per cell."""
        m, n = len(self.order), self.n
        dt = np.float64 if fp64 else np.float32
        per_edge = [np.zeros(m, dt) for _ in range(5)]
        post_tr, rate = np.zeros(n, dt), np.zeros(n, dt)
        fn = self.lib.on_get_plasticity64 if fp64 else self.lib.on_get_plasticity
        fn(self.h, *[_p(x) for x in per_edge], _p(post_tr), _p(rate))
        out = {}
        for k, x in zip(('weight', 'pre_trace', 'potential_trace', 'coactivity', 'usage'), per_edge):
            y = np.empty_like(x)
            y[self.order] = x
            out[k] = y
        out.update(post_trace=post_tr, rate=rate)
        return out


class Plastic(ct.Structure):
    _fields_ = [('on', ct.c_int32), ('stdp_rate', ct.c_float), ('inh_rate', ct.c_float),
                ('target_hz', ct.c_float), ('scaling_tau_ms', ct.c_float)]


def unpack_spikes(words, n):
    """uint32 words [..., ceil(n/32)] -> bool [..., n] (bit i%32 of word i/32)."""
    bits = np.unpackbits(words.view(np.uint8), axis=-1, bitorder='little')
    return bits[..., :n].astype(bool)
