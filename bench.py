"""Benchmark of the B200 engine (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Workloads (seeded synthetic inputs of the benchmark configurations):
  tick262k  (headline) scaled single-GPU tick: N=262,144, fan-in 512 CSR, fp16 weights, delays
            1-8, imposed Bernoulli(0.03) spikes; one step = 10,000 ticks.  metric ticks/s.
  bsr262k   the same with the 16x16 block matrix (128 block-columns per block-row, 25% fill).
  tick8k    isolated tick: N=8,192 Erdos-Renyi 2%, lognormal fp32 weights, Bernoulli(0.02)
            conductance drive; one step = 1,000 ticks.  metric ticks/s.
  learn8k   the same network learning every tick (biology.py's STDP, inhibitory rule, synaptic
            scaling and traces on every contact; split launch shape).
  partitioned4m  N=4,194,304, fan-in 1,000, fp16, imposed Bernoulli(0.01), 1,000 ticks a step;
            under torchrun the neurons are row-partitioned over the ranks, which exchange the
            tick's spike bitmask slices by one-sided peer stores over NVLink (NCCL all-gather when
            a rank cannot map its peers; one network: strong scaling).
  bc250     BC-250 language core, seed-0 weights, batch 1, one step = 512 tokens.  tokens/s.
  sessions  BC-250, 256 independent sessions (split over the ranks: strong scaling), one step =
            64 tokens per session.  tokens/s.
The line's top-level fields are the --workload (default tick262k); the other workloads follow
under "workloads", each with its own value, roofline, e2e and (N=1) cpu_baseline.  Tick
workloads other than partitioned4m do not shard (replicas: each rank runs its own seed).  With
N>1 the line also carries "partition_parity": a 65,536-neuron network partitioned over the
ranks, 100 ticks, compared on rank 0 with the same network run whole on one GPU.

--impl reference times the reference's own CPU implementation of each workload on this host's
cores, with no CUDA library loaded: the reference native library (oracle/_ref) for the language
core, the C restatement of the reference simulator (oracle/net_oracle.c, networks from
oracle/net_topo.c) for the tick networks, which have no native implementation in the reference.
"""
import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / 'neurogen-2.5_b200'))
sys.path.insert(0, str(ROOT))

PEAKS_FALLBACK = {'hbm_gbs': 6650.0, 'bf16_tflops': 1590.0}
METRIC_TICKS = 'ticks/sec (synaptic events/sec alongside)'
METRIC_TOKENS = 'tokens/sec at BC-250 profile'
TICK_WORKLOADS = ('tick262k', 'bsr262k', 'tick8k', 'learn8k', 'partitioned4m')
LANG_WORKLOADS = ('bc250', 'sessions')
WORKLOAD_NAMES = {'tick262k': 'scaled_tick_262144_csr', 'bsr262k': 'scaled_tick_262144_bsr16',
                  'tick8k': 'isolated_tick_8192', 'learn8k': 'isolated_tick_8192_learning',
                  'partitioned4m': 'partitioned_4194304_fanin1000',
                  'bc250': 'bc250_batch1', 'sessions': 'bc250_sessions256'}
TICKS_PER_STEP = {'tick262k': 10000, 'bsr262k': 10000, 'tick8k': 1000, 'learn8k': 1000, 'partitioned4m': 1000}
TOKENS_PER_STEP = {'bc250': 512, 'sessions': 64}
SESSIONS = 256
# Steps and warm-up steps of the workloads that follow the headline (bounded run time).
EXTRA_STEPS = {'tick262k': 3, 'bsr262k': 3, 'tick8k': 10, 'learn8k': 5, 'partitioned4m': 3, 'bc250': 3,
               'sessions': 5}
L2_BYTES = 126e6


def parse():
    p = argparse.ArgumentParser()
    p.add_argument('--gpus', type=int, default=1)
    p.add_argument('--steps', type=int, default=5)
    p.add_argument('--warmup', type=int, default=3)
    p.add_argument('--workload', default='tick262k', choices=list(TICK_WORKLOADS + LANG_WORKLOADS))
    p.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    p.add_argument('--rate', type=float, default=0.03)
    p.add_argument('--no-cpu-baseline', action='store_true')
    p.add_argument('--no-e2e', action='store_true')
    p.add_argument('--no-extras', action='store_true', help='time the --workload only')
    p.add_argument('--ticks', type=int, default=0, help='override ticks per step (profiling runs)')
    p.add_argument('--tokens', type=int, default=0, help='override tokens per step (profiling runs)')
    p.add_argument('--neurons', type=int, default=0,
                   help='partitioned4m: override the 4,194,304 neurons (profiling runs, e.g. one rank\'s share)')
    p.add_argument('--sessions', type=int, default=0,
                   help='sessions workload: override the 256 sessions (profiling runs, e.g. one rank\'s share)')
    return p.parse_args()


def peaks():
    path = ROOT / 'MEASURED_PEAKS.json'
    if path.is_file():
        return json.loads(path.read_text()), 'measured'
    return dict(PEAKS_FALLBACK), 'fallback'


class Dist:
    def __init__(self):
        self.world = int(os.environ.get('WORLD_SIZE', '1'))
        self.rank = int(os.environ.get('RANK', '0'))
        self.local = int(os.environ.get('LOCAL_RANK', '0'))
        self.pg = None

    def init(self):
        import torch
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=180),
                                    device_id=torch.device('cuda', self.local))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def _reduce(self, x, op):
        if not self.pg:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64, device='cuda')
        self.pg.all_reduce(t, op=op)
        return float(t.item())

    def max(self, x):
        return self._reduce(x, self.pg.ReduceOp.MAX) if self.pg else x

    def sum(self, x):
        return self._reduce(x, self.pg.ReduceOp.SUM) if self.pg else x

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


class Clocks:
    """nvidia-smi sampling during a timed region."""
    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile('w+', suffix='.csv', delete=False)
            self.proc = subprocess.Popen(['nvidia-smi', f'--id={self.index}', f'--query-gpu={self.FIELDS}',
                                          '--format=csv,noheader,nounits', '-lms', '200'],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            self.proc.wait(timeout=10)

    def summary(self):
        if not self.proc:
            return None
        rows = []
        with open(self.file.name) as f:
            for line in f:
                parts = [x.strip() for x in line.split(',')]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace('.', '', 1).isdigit()]
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        reasons = sorted({names[k] for r in rows for k in range(4) if r[5 + k].lower() == 'active'})
        return {'sm_mhz': float(np.median(sm)) if sm else None,
                'sm_max_mhz': float(rows[0][2]) if rows[0][2].replace('.', '', 1).isdigit() else None,
                'reasons': reasons, 'samples': len(rows)}


class L2Flush:
    """Writes a buffer twice the size of L2 between timed steps (outside the timed region)."""

    def __init__(self):
        import torch
        self.buf = torch.empty(int(2 * L2_BYTES) // 4, dtype=torch.int32, device='cuda')

    def __call__(self):
        self.buf.fill_(1)


def time_steps(step, stream, steps, flush=None):
    """CUDA-event time of `steps` calls of step() on `stream`, each bracketed by a device
    synchronisation; the L2 flush (if any) runs between steps, outside the timed region."""
    import torch
    total = 0.0
    for _ in range(steps):
        if flush:
            flush()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        step()
        end.record(stream)
        torch.cuda.synchronize()
        total += start.elapsed_time(end) / 1e3
    return total


# ---------------------------------------------------------------------------
# Workload definitions shared by both arms.
# ---------------------------------------------------------------------------
def oracle_tick_config(name, rate, n_override=0):
    """The workload's network configuration as the oracle's dict (no CUDA library)."""
    from oracle import net as on
    if name == 'partitioned4m':
        c = on.partitioned_4m(rate=0.01)
        if n_override:
            c.update(n=n_override, n_exc=int(n_override * 0.8))
        return c
    if name == 'tick262k':
        return on.scaled_262k('csr', rate=rate)
    if name == 'bsr262k':
        return on.scaled_262k('bsr', rate=rate)
    if name == 'learn8k':
        return dict(on.isolated_8k(), plasticity=1, launch=2)
    return on.isolated_8k()


def tick_config_dict(name, c, world, ticks):
    """The `config` object of a tick workload: what the workload is, identical in both arms."""
    fanin, topo = c['fanin'], c['topology']
    synapses = (c['n'] * fanin if topo == 1 else
                (c['n'] // 16) * c['bsr_blocks'] * c['bsr_fill'] if topo == 2 else
                round(c['n'] * (c['n'] - 1) * c['p_connect']))
    part = name == 'partitioned4m'
    return {'workload': WORKLOAD_NAMES[name], 'n': c['n'], 'ticks_per_step': ticks,
            'fanin': fanin if topo == 1 else None,
            'bsr': [c['bsr_blocks'], c['bsr_fill']] if topo == 2 else None,
            'drive': ('imposed Bernoulli(%g) spikes' % c['drive_p'] if c['drive_kind'] == 1 else
                      'Bernoulli(%g) conductance drive of %g nS' % (c['drive_p'], c['drive_ns'])),
            'weights': 'fp16' if c['weight_kind'] == 1 else 'fp32', 'delays': [c['delay_min'], c['delay_max']],
            'synapses': synapses if topo != 0 else f'~{synapses}',
            'learning': ('STDP + inhibitory rule + synaptic scaling + traces every tick'
                         if c.get('plasticity') else None),
            'l2': 'inputs larger than L2' if synapses * 6 > L2_BYTES else 'network fits in L2; L2 flushed between steps',
            'parallelism': (f'rows{world} + spike bitmask exchange (one-sided peer stores over NVLink, '
                            'NCCL all-gather fall-back)' if part and world > 1 else
                            'one GPU' if part else f'replicas{world}')}


def lang_config_dict(name, world, sessions=SESSIONS):
    return {'workload': WORKLOAD_NAMES[name], 'sessions': 1 if name == 'bc250' else sessions,
            'tokens_per_step': TOKENS_PER_STEP[name], 'weights': 'seed-0 random init (packed 14,804,744 fp32)',
            'l2': 'weights (59 MB) L2-resident by design; L2 flushed between steps',
            'parallelism': f'replicas{world}' if name == 'bc250' else f'dp{world} over sessions'}


def engine_config(c):
    """The engine's NetConfig from an oracle config dict."""
    from neurogen_b200.network import default_config
    return default_config(**{k: v for k, v in c.items()})


# ---------------------------------------------------------------------------
# Tick-network workloads (our arm).
# ---------------------------------------------------------------------------
def tick_bytes(cfg, spikes, events, held=None, contacts=0):
    """Algorithmic DRAM bytes of one tick, the roofline numerator.

    Per neuron: the four fp32 state values (V, adaptation, g_E, g_I) read and written (32 B),
    its ring slot read and cleared (16 B) and its spike bit (1/8 B).  Per delivered synapse
    (CSR): a 4-byte index, the weight (2 B fp16 or 4 B fp32) and a 1-byte delay.  Block
    storage: per spiking neuron and block of its block-column, the 32-byte tile column plus
    the block's 4-byte row/delay word.
    """
    wbytes = 2 if cfg.weight_kind == 1 else 4
    held = cfg.n if held is None else held
    per_neuron = held * 48 + held / 8
    if cfg.storage == 1:
        return per_neuron + spikes * cfg.bsr_blocks * 36
    learning = 0
    if cfg.plasticity and contacts:
        # Every contact every tick: index read, weight and three traces read and written (36 B;
        # a stored contact's potential trace is its pre trace); every neuron: post trace and rate
        # read and written (16 B) and its history bit.
        learning = contacts * 36 + held * 16 + held / 8
    return per_neuron + events * (4 + wbytes + 1) + learning


# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) per tick from one ncu capture of the
# dominant kernel on this workload (profiles/k_net_resident_scaled_tick_262144_{csr,bsr16}.md: 64 ticks
# at a 3% spike rate).  Owner-block traffic is proportional to the spikes, so it is scaled by the run's rate.
NCU_TRAFFIC = {('scaled_tick_262144_csr', 'resident'): (2.400492e9 + 4.731392e6, 64, 0.030017),
               ('scaled_tick_262144_bsr16', 'resident'): (2.698401e9 + 4.773888e6, 64, 0.030017)}


def tick_traffic(workload, mode, rate):
    entry = NCU_TRAFFIC.get((workload, mode))
    if not entry:
        return None
    total, ticks, rate0 = entry
    return total / ticks * rate / rate0


KERNEL_OF_LAUNCH = {'fused': 'k_net_fused', 'split': 'tick = k_net_alif + k_net_push',
                    'resident': 'k_net_resident (persistent, serial tick, 2,048 ticks a launch)',
                    'resident-pipelined': 'k_net_pipe (persistent, pipelined tick, 2,048 ticks a launch)',
                    'split-learning': 'tick = k_net_alif + k_net_learn + k_net_push'}


def tick_launches(mode, ticks):
    """Kernels the engine launches for one run of `ticks` ticks without per-tick outputs."""
    if mode.startswith('resident'):
        return -(-ticks // 2048)
    # split: membrane, delay-1 push, delay>=2 push; learning: membrane, learn, push
    per_tick = 1 if mode == 'fused' else 3
    graphs = ticks // 64
    return graphs * (64 * per_tick + 1) + (ticks - graphs * 64) * per_tick + (1 if graphs else 0)


def bench_ticks(name, args, dist, steps, warmup, cpu=True):
    import torch
    from neurogen_b200 import library
    from neurogen_b200.network import Topology, Network, nccl_unique_id
    lib = library()
    part = name == 'partitioned4m'
    rate = args.rate
    ticks = args.ticks or TICKS_PER_STEP[name]
    oc = oracle_tick_config(name, rate, args.neurons if part else 0)
    cfg = engine_config(oc)
    if part:
        cfg.part_rank, cfg.part_world = dist.rank, (dist.world if dist.world > 1 else 0)
    else:
        cfg.seed = cfg.seed + dist.rank  # independent replica per rank
    t0 = time.time()
    if part:
        if dist.world > 1:
            ids = [nccl_unique_id() if dist.rank == 0 else None]
            dist.pg.broadcast_object_list(ids, src=0)
            net = Network.partitioned(cfg, ids[0])
        else:
            net = Network(cfg)
        synapses = int(dist.sum(net.synapses))
    else:
        topo = Topology(cfg) if cfg.topology != 1 or cfg.weight_kind != 1 else None
        net = topo.network() if topo else Network(cfg)   # fixed fan-in fp16: drawn on the device
        synapses = net.synapses
    setup_s = time.time() - t0
    mode = net.launch
    shape = ('resident-pipelined' if net.resident_tick == 'pipelined' else
             'split-learning' if cfg.plasticity else mode)
    stream = torch.cuda.Stream()  # explicit stream: the engine enqueues on exactly this one

    def step():
        if lib.ng_net_run_device(net.h, ticks, None, None, stream.cuda_stream):
            raise RuntimeError(lib.ng_error().decode())

    flush = L2Flush() if synapses * 6 < L2_BYTES else None
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    s0, e0 = net.stats()
    with Clocks(torch.cuda.current_device()) as clk:
        elapsed = time_steps(step, stream, steps, flush)
    s1, e1 = net.stats()
    spikes, events = s1 - s0, e1 - e0
    dist.barrier()
    t_max = dist.max(elapsed)
    total_ticks = ticks * steps
    held = cfg.n // dist.world if part else cfg.n
    b_tick = tick_bytes(cfg, spikes / total_ticks, events / total_ticks, held, contacts=synapses)
    pk, src = peaks()
    if part:  # one network over all ranks: sum the ranks' bytes, compare with all their peaks
        b_tick = dist.sum(b_tick)
        spikes, events = dist.sum(spikes), dist.sum(events)
    achieved = b_tick / (t_max / total_ticks) / 1e9
    peak_total = pk['hbm_gbs'] * (dist.world if part else 1)
    rec = {
        'metric': METRIC_TICKS, 'value': total_ticks * (1 if part else dist.world) / t_max, 'unit': 'ticks/s',
        'n_gpus': dist.world, 'steps': steps, 'warmup': warmup, 'ms_per_step': t_max / steps * 1e3,
        'higher_is_better': True, 'scaling': 'strong' if part else 'weak', 'vs_baseline': None,
        'dtype': 'fp32', 'data': 'synthetic', 'config': tick_config_dict(name, oc, dist.world, ticks),
        'measured': {'spike_rate': spikes / total_ticks / cfg.n, 'events_per_tick': events / total_ticks,
                     'launch': mode, 'resident_tick': net.resident_tick, 'setup_s': round(setup_s, 2),
                     'exchange': net.exchange if part and dist.world > 1 else None},
        'synaptic_events_per_s': events * (1 if part else dist.world) / t_max,
        'roofline': {'bound': 'hbm', 'achieved': achieved, 'peak': peak_total, 'unit': 'GB/s',
                     'frac': achieved / peak_total,
                     'traffic': (tick_traffic(WORKLOAD_NAMES[name], shape, spikes / total_ticks / cfg.n)
                                 if not part else None),
                     'traffic_unit': 'bytes/tick (ncu, scaled by spike rate)', 'bytes_per_tick': b_tick,
                     'kernel': KERNEL_OF_LAUNCH[shape], 'peak_source': src},
        'gpu_launches': tick_launches(shape, ticks) * steps,
        'clocks': clk.summary(),
    }
    if not args.no_e2e:
        rec['e2e'] = e2e_ticks(lib, net, ticks, steps, warmup, dist, part)
    if cpu and dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        rec['cpu_baseline'] = cpu_baseline_ticks(name, oc, budget_s=12.0 if name == 'tick262k' else 6.0)
    net.close()
    return rec


def e2e_ticks(lib, net, ticks, steps, warmup, dist, part=False):
    """Through the C ABI with host buffers: per step, upload the full network state from
    pinned host memory, run the ticks, read back the spike/event totals and the state."""
    import ctypes as ct
    import torch
    pin = lambda shape, dt: torch.empty(shape, dtype=dt, pin_memory=True).numpy()
    st = net.get_state()
    names = ('v', 'a', 'ge', 'gi', 'ref', 'ring')
    host = {k: pin(st[k].shape, torch.float32 if st[k].dtype == np.float32 else torch.int32) for k in names}
    for k in names:
        host[k][...] = st[k]
    totals = pin((2,), torch.int64)
    ptr = lambda a: a.ctypes.data_as(ct.c_void_p)
    h2d = sum(host[k].nbytes for k in names)
    d2h = h2d + totals.nbytes

    def step():
        t0 = time.perf_counter()
        if lib.ng_net_set_state(net.h, *[ptr(host[k]) for k in names], st['tick']):
            raise RuntimeError(lib.ng_error().decode())
        if lib.ng_net_run(net.h, ticks, None, None):
            raise RuntimeError(lib.ng_error().decode())
        if lib.ng_net_stats(net.h, totals) or lib.ng_net_get_state(net.h, *[ptr(host[k]) for k in names], None):
            raise RuntimeError(lib.ng_error().decode())
        return time.perf_counter() - t0

    for _ in range(max(1, warmup)):
        step()
    dist.barrier()
    elapsed = sum(step() for _ in range(steps))
    t_max = dist.max(elapsed)
    return {'value': ticks * steps * (1 if part else dist.world) / t_max, 'unit': 'ticks/s',
            'h2d_bytes_per_step': h2d, 'd2h_bytes_per_step': d2h,
            'api': 'ng_net_set_state + ng_net_run + ng_net_stats + ng_net_get_state (host buffers)'}


def oracle_network(name, oc):
    """(oracle, scale): the workload's network on the CPU checker; partitioned4m at 1/16 of its
    neurons (same fan-in and rate; 4.2 billion synapses do not fit a host-side checker)."""
    from oracle import net as on
    scale = 1
    if name == 'partitioned4m':
        scale = 16
        oc = dict(oc, n=oc['n'] // scale, n_exc=oc['n_exc'] // scale)
    orc = on.NetOracle(oc, *on.generate(oc))
    if oc.get('plasticity'):
        orc.set_plasticity(True, stdp_rate=oc['stdp_rate'], inhibitory_rate=oc['inhibitory_rate'],
                           target_hz=oc['target_hz'], scaling_tau_ms=oc['scaling_tau_ms'])
    return orc, scale


def oracle_ticks(orc, oc, ticks):
    """Run the checker: OpenMP over all host cores, or one thread for a learning network (the
    oracle's learning step is single-threaded)."""
    if oc.get('plasticity'):
        orc.run(ticks)
    else:
        orc.run_mt(ticks)


def cpu_baseline_ticks(name, oc, budget_s):
    import multiprocessing
    t0 = time.time()
    orc, scale = oracle_network(name, oc)
    build_s = time.time() - t0
    oracle_ticks(orc, oc, 2)
    done, el = 0, 0.0
    chunk = 5 if oc['n'] > 100000 else (20 if oc.get('plasticity') else 100)
    while el < budget_s:
        t1 = time.time()
        oracle_ticks(orc, oc, chunk)
        el += time.time() - t1
        done += chunk
    cores = 1 if oc.get('plasticity') else int(os.environ.get('OMP_NUM_THREADS', multiprocessing.cpu_count()))
    how = 'on_run with learning, one thread' if oc.get('plasticity') else 'on_run_mt, OpenMP'
    sample = (f'{done} ticks of the same network (oracle/net_oracle.c {how}), {el:.1f} s; '
              f'network generation {build_s:.1f} s excluded')
    if scale > 1:
        sample += f'; 1/{scale}-scale network, time per tick x{scale}'
    return {'value': done / el / scale, 'unit': 'ticks/s', 'cores': cores, 'kind': 'port', 'sample': sample}


# ---------------------------------------------------------------------------
# Language-core workloads (our arm).
# ---------------------------------------------------------------------------
def lang_tokens(workload, sessions, steps_tokens):
    import torch
    if workload == 'bc250':
        g = torch.Generator().manual_seed(0)
        return torch.randint(0, 264, (steps_tokens, 1), generator=g).numpy().astype(np.int32)
    cols = []
    for k in sessions:
        g = torch.Generator().manual_seed(k)
        cols.append(torch.randint(0, 264, (1024,), generator=g).numpy())
    return np.stack(cols, 1).astype(np.int32)[:steps_tokens]


def lang_flops_per_token(cfg):
    c, w, R = cfg.columns, cfg.width, cfg.regions
    region = c * 12 * w + c * 29 * w + c * 64 * 64 * cfg.ticks + w * c * 100
    per_adv = R * region
    mac = (1 + cfg.idle_steps) * per_adv - c * 12 * w * cfg.idle_steps + 264 * w
    return 2 * mac


def lang_launches_per_token(cfg):
    """Kernels one pool token step enqueues (lang_engine.cpp DeviceModel::enqueue_view): per advance the
    regions' feedback projections in batches of four, then per region the input projection (sensory
    regions), the recurrent ticks (one cluster launch, or one launch per tick plus a copy for odd tick
    counts when no cluster shape fits the column count), the output projection and the LayerNorm; per
    token the readout and the activity."""
    c = cfg.columns
    cluster = (c % 4 == 0 and c // 4 <= 8) or (c % 2 == 0 and c // 2 <= 8) or c <= 8
    ticks = 1 if cluster else cfg.ticks + cfg.ticks % 2
    per = 0
    for adv in range(1 + cfg.idle_steps):
        per += -(-cfg.regions // 4)
        for r in range(cfg.regions):
            sensory = adv == 0 or r > 0
            per += int(sensory) + ticks + 2
    return per + 2


def bench_lang(name, args, dist, steps, warmup, cpu=True):
    import torch
    from neurogen_b200 import library
    from neurogen_b200.language import LanguageConfig, NativeEngine, init_packed_weights
    lib = library()
    cfg = LanguageConfig()
    w = init_packed_weights(cfg, seed=0)
    eng = NativeEngine(cfg, w)
    n_sessions = args.sessions or SESSIONS
    if name == 'bc250':
        mine = [0]
    else:
        per = n_sessions // dist.world
        mine = list(range(dist.rank * per, (dist.rank + 1) * per))
    B = len(mine)
    T = args.tokens or TOKENS_PER_STEP[name]
    toks = lang_tokens(name, mine, 1024 if name == 'sessions' else 512)
    pool = lib.ng_pool_create(eng.handle, B)
    if not pool:
        raise RuntimeError(lib.ng_error().decode())
    stream = torch.cuda.Stream()  # explicit stream: the engine enqueues on exactly this one
    d_tok = torch.from_numpy(np.ascontiguousarray(toks)).cuda()
    d_logits = torch.empty((B, 264), device='cuda')
    pos = [0]

    def step():
        for _ in range(T):
            row = d_tok[pos[0] % d_tok.shape[0]]
            if lib.ng_pool_step_device(pool, row.data_ptr(), d_logits.data_ptr(), stream.cuda_stream):
                raise RuntimeError(lib.ng_error().decode())
            pos[0] += 1

    flush = L2Flush()
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    with Clocks(torch.cuda.current_device()) as clk:
        elapsed = time_steps(step, stream, steps, flush)
    dist.barrier()
    t_max = dist.max(elapsed)
    total = B * T * steps * (dist.world if name == 'sessions' else dist.world)
    fl = lang_flops_per_token(cfg)
    pk, src = peaks()
    achieved = fl * B * T * steps / elapsed / 1e12
    rec = {
        'metric': METRIC_TOKENS, 'value': total / t_max, 'unit': 'tokens/s', 'n_gpus': dist.world,
        'steps': steps, 'warmup': warmup, 'ms_per_step': t_max / steps * 1e3,
        'higher_is_better': True, 'scaling': 'strong' if name == 'sessions' else 'weak',
        'vs_baseline': None, 'dtype': 'fp32', 'data': 'synthetic',
        'config': lang_config_dict(name, dist.world, n_sessions),
        'measured': {'sessions_per_gpu': B, 'tokens_per_step': T},
        'roofline': {'bound': 'tensor', 'achieved': achieved, 'peak': pk.get('bf16_tflops'),
                     'unit': 'TFLOP/s', 'frac': achieved / pk.get('bf16_tflops'), 'traffic': None,
                     'note': 'exact fp32 SIMT path (bit-exact with the reference); FLOPs per token 2x MACs; '
                             'a small fraction of the bf16 tensor peak by construction',
                     'peak_source': src},
        'gpu_launches': lang_launches_per_token(cfg) * T * steps,
        'clocks': clk.summary(),
    }
    if not args.no_e2e:
        tok_host = np.ascontiguousarray(toks)
        logits = np.empty((B, 264), np.float32)

        def e2e_step():
            t0 = time.perf_counter()
            for _ in range(T):
                row = np.ascontiguousarray(tok_host[pos[0] % tok_host.shape[0]])
                if lib.ng_pool_step(pool, row, logits.ctypes.data, None, None):
                    raise RuntimeError(lib.ng_error().decode())
                pos[0] += 1
            return time.perf_counter() - t0
        e2e_step()
        dist.barrier()
        el = dist.max(sum(e2e_step() for _ in range(steps)))
        rec['e2e'] = {'value': total / el, 'unit': 'tokens/s', 'h2d_bytes_per_step': B * 4 * T,
                      'd2h_bytes_per_step': B * 264 * 4 * T, 'api': 'ng_pool_step (host tokens, host logits)'}
    if cpu and dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        rec['cpu_baseline'] = cpu_baseline_lang(name, toks, budget_s=8.0)
    lib.ng_pool_destroy(pool)
    eng.close()
    if name == 'sessions':
        rec['tensor_core_projections'] = bench_lang_tc(cfg, w, d_tok, B, T, steps, warmup, dist, stream, flush)
    return rec


def bench_lang_tc(cfg, w, d_tok, B, T, steps, warmup, dist, stream, flush):
    """The same sessions with the opt-in tensor-core projections (NEUROGEN_PROJECTION=tc, read when
    the engine is created): faster, but not spike-exact, so reported beside the exact figure."""
    import torch
    from neurogen_b200 import library
    from neurogen_b200.language import NativeEngine
    lib = library()
    old = os.environ.get('NEUROGEN_PROJECTION')
    os.environ['NEUROGEN_PROJECTION'] = 'tc'
    try:
        eng = NativeEngine(cfg, w)
    finally:
        if old is None:
            del os.environ['NEUROGEN_PROJECTION']
        else:
            os.environ['NEUROGEN_PROJECTION'] = old
    pool = lib.ng_pool_create(eng.handle, B)
    if not pool:
        raise RuntimeError(lib.ng_error().decode())
    d_logits = torch.empty((B, 264), device='cuda')
    pos = [0]

    def step():
        for _ in range(T):
            row = d_tok[pos[0] % d_tok.shape[0]]
            if lib.ng_pool_step_device(pool, row.data_ptr(), d_logits.data_ptr(), stream.cuda_stream):
                raise RuntimeError(lib.ng_error().decode())
            pos[0] += 1

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    t_max = dist.max(time_steps(step, stream, steps, flush))
    lib.ng_pool_destroy(pool)
    eng.close()
    return {'value': B * T * steps * dist.world / t_max, 'unit': 'tokens/s', 'ms_per_step': t_max / steps * 1e3,
            'switch': 'NEUROGEN_PROJECTION=tc',
            'parity': ('not spike-exact: every batched projection on tcgen05 with split-tf32 operands, within '
                       'a few 1e-6 of the exact sum; the first spike flips within a few ticks '
                       '(tests/test_quoted_configs_gpu.py)')}


def cpu_baseline_lang(name, toks, budget_s):
    """The reference native library (oracle/_ref): batch 1 on one thread; the sessions workload on
    every host core, one engine per thread, each serving its own sessions."""
    import multiprocessing
    from concurrent.futures import ThreadPoolExecutor
    from neurogen_b200.language import LanguageConfig
    from oracle.lang import RefEngine, seeded_weights
    cfg = LanguageConfig()
    w = seeded_weights()
    threads = 1 if name == 'bc250' else multiprocessing.cpu_count()
    engines = [RefEngine(cfg, w) for _ in range(threads)]
    states = [np.zeros(engines[0].S, np.float32) for _ in range(threads)]
    counts = [0] * threads
    stop = time.time() + budget_s

    def work(k):
        i = 0
        while time.time() < stop:
            _, states[k], _, _ = engines[k].step(int(toks[i % len(toks), k % toks.shape[1]]), states[k])
            i += 1
        counts[k] = i

    t0 = time.time()
    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(work, range(threads)))
    el = time.time() - t0
    return {'value': sum(counts) / el, 'unit': 'tokens/s', 'cores': threads, 'kind': 'reference',
            'sample': f'{sum(counts)} tokens in {el:.1f} s on {threads} thread(s), one engine and session each, '
                      'reference native CPU library (oracle/_ref)'}


# ---------------------------------------------------------------------------
# Partition parity (N > 1).
# ---------------------------------------------------------------------------
def partition_parity(dist):
    """A 65,536-neuron network (fan-in 96, self-generated spikes) row-partitioned over the ranks:
    100 ticks, every rank recording the whole network's raster; rank 0 runs the same network whole
    on its own GPU and compares rasters, per-tick counts and totals."""
    import torch
    from neurogen_b200.network import Network, default_config, nccl_unique_id
    kw = dict(n=65536, n_exc=52428, topology='fixed_fanin', fanin=96, weight_kind='halfnormal_f16', w_mu=0.0,
              w_sigma=0.05, drive_kind='conductance', drive_p=0.03, drive_ns=18.0, seed=12)
    ids = [nccl_unique_id() if dist.rank == 0 else None]
    dist.pg.broadcast_object_list(ids, src=0)
    net = Network.partitioned(default_config(part_rank=dist.rank, part_world=dist.world, **kw), ids[0])
    spikes, counts = net.run(100)
    mine = np.array(net.stats(), np.float64)
    tot = torch.from_numpy(mine).cuda()
    dist.pg.all_reduce(tot)
    # per-tick counts of a rank cover its own neurons' spikes and the events onto them: sum over ranks
    tick_counts = torch.from_numpy(counts.astype(np.float64)).cuda()
    dist.pg.all_reduce(tick_counts)
    counts = tick_counts.cpu().numpy().astype(np.int64)
    exchange = net.exchange
    net.close()
    ok = True
    detail = {}
    if dist.rank == 0:
        full = Network(default_config(**kw))
        fs, fc = full.run(100)
        ok = (np.array_equal(spikes, fs) and np.array_equal(counts, fc) and
              tuple(int(x) for x in tot.cpu().numpy()) == full.stats())
        detail = {'ticks': 100, 'n': kw['n'], 'spikes': int(fc[:, 0].sum()), 'ranks': dist.world,
                  'exchange': exchange}
        full.close()
    flag = torch.tensor([1.0 if ok else 0.0], device='cuda')
    dist.pg.all_reduce(flag, op=dist.pg.ReduceOp.MIN)
    return dict(result='pass' if flag.item() == 1.0 else 'fail', **detail)


# ---------------------------------------------------------------------------
# Reference arm (CPU; no CUDA library).
# ---------------------------------------------------------------------------
def reference_record(name, args, world, steps, warmup):
    import multiprocessing
    cores = multiprocessing.cpu_count()
    if name in TICK_WORKLOADS:
        oc = oracle_tick_config(name, args.rate)
        orc, scale = oracle_network(name, oc)
        sample = 20 if oc['n'] > 100000 else (40 if oc.get('plasticity') else 200)
        for _ in range(warmup):
            oracle_ticks(orc, oc, sample)
        t0 = time.time()
        for _ in range(steps):
            oracle_ticks(orc, oc, sample)
        el = time.time() - t0
        value, unit = sample * steps / el / scale, 'ticks/s'
        ms_per_step = el / steps * 1e3 * scale / sample * TICKS_PER_STEP[name]
        config = tick_config_dict(name, oc, world, TICKS_PER_STEP[name])
        scaling = 'strong' if name == 'partitioned4m' else 'weak'
        kind, threads = 'port', (1 if oc.get('plasticity') else cores)
        desc = (f'{sample} ticks per step (oracle/net_oracle.c with learning, one thread)' if oc.get('plasticity')
                else f'{sample} ticks per step (oracle/net_oracle.c, OpenMP on {cores} cores)')
        if scale > 1:
            desc += f'; 1/{scale}-scale network (N={oc["n"] // scale:,}), time per tick x{scale}'
        metric = METRIC_TICKS
    else:
        from concurrent.futures import ThreadPoolExecutor
        from oracle.lang import RefEngine, seeded_weights

        class Cfg:
            columns, width, regions, ticks, idle_steps = 32, 768, 4, 2, 1
        w = seeded_weights()
        threads = 1 if name == 'bc250' else cores
        engines = [RefEngine(Cfg, w) for _ in range(threads)]
        states = [np.zeros(engines[0].S, np.float32) for _ in range(threads)]
        per_step = 8 if name == 'bc250' else 2

        def work(k):
            for i in range(per_step):
                _, states[k], _, _ = engines[k].step((k * 7 + i) % 264, states[k])

        with ThreadPoolExecutor(threads) as ex:
            for _ in range(warmup):
                list(ex.map(work, range(threads)))
            t0 = time.time()
            for _ in range(steps):
                list(ex.map(work, range(threads)))
            el = time.time() - t0
        value, unit = threads * per_step * steps / el, 'tokens/s'
        ms_per_step = el / steps * 1e3
        config = lang_config_dict(name, world)
        scaling = 'weak' if name == 'bc250' else 'strong'
        kind = 'reference'
        desc = f'{per_step} tokens per step on each of {threads} independent sessions (one engine per thread)'
        sample = per_step * threads
        metric = METRIC_TOKENS
    return {'metric': metric, 'value': value, 'unit': unit, 'n_gpus': world, 'steps': steps, 'warmup': warmup,
            'ms_per_step': ms_per_step, 'higher_is_better': True, 'scaling': scaling, 'impl': 'reference',
            'dtype': 'fp32', 'data': 'synthetic', 'config': config, 'sample_per_step': sample,
            'cpu_baseline': {'value': value, 'unit': unit, 'cores': threads, 'kind': kind, 'sample': desc},
            'e2e': {'value': value, 'unit': unit, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}


def extras_for(headline):
    return [w for w in ('bc250', 'sessions', 'tick8k', 'learn8k', 'bsr262k', 'partitioned4m') if w != headline]


def main():
    args = parse()
    dist = Dist()
    if args.impl == 'reference':
        if dist.rank == 0:
            line = reference_record(args.workload, args, dist.world, args.steps, args.warmup)
            if not args.no_extras:
                line['workloads'] = {WORKLOAD_NAMES[w]: reference_record(w, args, dist.world, 3, 1)
                                     for w in extras_for(args.workload)}
            print(json.dumps(line), flush=True)
        return
    import torch
    torch.cuda.set_device(dist.local)
    dist.init()
    run = lambda w, steps, warmup, cpu=True: (bench_lang if w in LANG_WORKLOADS else bench_ticks)(
        w, args, dist, steps, warmup, cpu)
    try:
        line = run(args.workload, args.steps, args.warmup)
        if not args.no_extras:
            line['workloads'] = {}
            for w in extras_for(args.workload):
                rec = run(w, EXTRA_STEPS[w], 3)
                line['workloads'][WORKLOAD_NAMES[w]] = rec
                line['gpu_launches_all_workloads'] = line.get('gpu_launches_all_workloads',
                                                              line['gpu_launches']) + rec['gpu_launches']
        if dist.world > 1:
            line['partition_parity'] = partition_parity(dist)
        if dist.rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        dist.close()


if __name__ == '__main__':
    main()
