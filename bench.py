"""Benchmark of the B200 engine (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Workloads (seeded synthetic inputs of the benchmark configurations):
  tick262k  (default) scaled single-GPU tick: N=262,144, fan-in 512 CSR, fp16 weights, delays
            1-8, imposed Bernoulli(0.03) spikes; one step = 10,000 ticks.  metric ticks/s.
  bsr262k   the same with the 16x16 block matrix (128 block-columns per block-row, 25% fill).
  tick8k    isolated tick: N=8,192 Erdos-Renyi 2%, lognormal fp32 weights, Bernoulli(0.02)
            conductance drive; one step = 1,000 ticks.  metric ticks/s.
  partitioned4m  N=4,194,304, fan-in 1,000, fp16, imposed Bernoulli(0.01); under torchrun the
            neurons are row-partitioned over the ranks with a per-tick NCCL all-gather of the
            spike bitmask (one network: strong scaling); one step = 1,000 ticks.
  bc250     BC-250 language core, seed-0 weights, batch 1, one step = 512 tokens.  tokens/s.
  sessions  BC-250, 256 independent sessions (split over the ranks), one step = 64 tokens per
            session.  tokens/s.
Under torchrun every rank runs its share on its own GPU (tick workloads: independent replicas;
sessions: a shard of the sessions); time is the max over ranks of CUDA-event time.

--impl reference times the reference's own CPU implementation of the workload on this host's
cores: the reference native library (oracle/_ref) for the language core, the C restatement of
the reference simulator (oracle/net_oracle.c) for the tick network, which has no native
implementation in the reference.
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


def parse():
    p = argparse.ArgumentParser()
    p.add_argument('--gpus', type=int, default=1)
    p.add_argument('--steps', type=int, default=5)
    p.add_argument('--warmup', type=int, default=3)
    p.add_argument('--workload', default='tick262k',
                   choices=['tick262k', 'bsr262k', 'tick8k', 'partitioned4m', 'bc250', 'sessions'])
    p.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    p.add_argument('--rate', type=float, default=0.03)
    p.add_argument('--no-cpu-baseline', action='store_true')
    p.add_argument('--no-e2e', action='store_true')
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
        d = json.loads(path.read_text())
        return d, 'measured'
    return dict(PEAKS_FALLBACK), 'fallback'


class Dist:
    def __init__(self):
        self.world = int(os.environ.get('WORLD_SIZE', '1'))
        self.rank = int(os.environ.get('RANK', '0'))
        self.local = int(os.environ.get('LOCAL_RANK', '0'))
        self.pg = None

    def init(self, device):
        import torch
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device('cuda', self.local))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, x):
        if not self.pg:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64, device='cuda')
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum(self, x):
        if not self.pg:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64, device='cuda')
        self.pg.all_reduce(t, op=self.pg.ReduceOp.SUM)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


class Clocks:
    """nvidia-smi sampling during the timed region."""
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


def cuda_timer(fn, stream):
    import torch
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    fn()
    end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end) / 1e3


# ---------------------------------------------------------------------------
# Tick-network workloads.
# ---------------------------------------------------------------------------
def tick_config(name, rate, rank=0, world=1):
    from neurogen_b200.network import scaled_262k, isolated_8k, partitioned_4m
    if name == 'partitioned4m':
        return partitioned_4m(rank, world, rate=0.01), 1000, 'partitioned_4194304_fanin1000'
    if name == 'tick262k':
        return scaled_262k('csr', rate=rate), 10000, 'scaled_tick_262144_csr'
    if name == 'bsr262k':
        return scaled_262k('bsr', rate=rate), 10000, 'scaled_tick_262144_bsr16'
    return isolated_8k(), 1000, 'isolated_tick_8192'


def tick_bytes(cfg, spikes, events, held=None):
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
    return per_neuron + events * (4 + wbytes + 1)


# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) per tick from one ncu capture of the
# dominant kernel on this workload (profiles/k_net_resident_scaled_tick_262144_{csr,bsr16}.md: 64 ticks
# at a 3% spike rate).  Owner-block traffic is proportional to the spikes, so it is scaled by the run's rate.
NCU_TRAFFIC = {('scaled_tick_262144_csr', 'resident'): (2.400492e9 + 4.731392e6, 64, 0.030017),
               ('scaled_tick_262144_bsr16', 'resident'): (3.276054e9 + 5.5424e6, 64, 0.030017)}


def tick_traffic(workload, mode, rate):
    entry = NCU_TRAFFIC.get((workload, mode))
    if not entry:
        return None
    total, ticks, rate0 = entry
    return total / ticks * rate / rate0


KERNEL_OF_LAUNCH = {'fused': 'k_net_fused', 'split': 'tick = k_net_alif + k_net_push',
                    'resident': 'k_net_resident (persistent, 2,048 ticks a launch)'}


def tick_launches(mode, ticks):
    """Kernels the engine launches for one run of `ticks` ticks without per-tick outputs."""
    if mode == 'resident':
        return -(-ticks // 2048)
    per_tick = 1 if mode == 'fused' else (3 if mode == 'split' else 1)
    graphs = ticks // 64
    return graphs * (64 * per_tick + 1) + (ticks - graphs * 64) * per_tick + (1 if graphs else 0)


def bench_ticks(args, dist):
    import torch
    from neurogen_b200 import library
    from neurogen_b200.network import Topology, Network, nccl_unique_id
    lib = library()
    part = args.workload == 'partitioned4m'
    cfg, ticks, wl = tick_config(args.workload, args.rate, dist.rank, dist.world)
    ticks = args.ticks or ticks
    if part and args.neurons:
        cfg.n, cfg.n_exc = args.neurons, int(args.neurons * 0.8)
    if not part:
        cfg.seed = cfg.seed + dist.rank  # independent replica per rank
    t0 = time.time()
    if part and dist.world > 1:
        ids = [nccl_unique_id() if dist.rank == 0 else None]
        dist.pg.broadcast_object_list(ids, src=0)
        net = Network.partitioned(cfg, ids[0])
        synapses = net.synapses * dist.world
    else:
        topo = Topology(cfg)
        net = topo.network()
        synapses = topo.synapses
    setup_s = time.time() - t0
    mode = net.launch  # 'fused', 'split' or 'resident'
    stream = torch.cuda.Stream()  # explicit stream: the engine enqueues on exactly this one

    def step():
        if lib.ng_net_run_device(net.h, ticks, None, None, stream.cuda_stream):
            raise RuntimeError(lib.ng_error().decode())

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    s0, e0 = net.stats()
    with Clocks(torch.cuda.current_device()) as clk:
        elapsed = 0.0
        for _ in range(args.steps):
            elapsed += cuda_timer(step, stream)
    s1, e1 = net.stats()
    spikes, events = s1 - s0, e1 - e0
    dist.barrier()
    t_max = dist.max(elapsed)
    total_ticks = ticks * args.steps
    per_tick_s = elapsed / total_ticks
    held = cfg.n // dist.world if part else cfg.n
    b_tick = tick_bytes(cfg, spikes / total_ticks, events / total_ticks, held)
    pk, src = peaks()
    if part:  # one network over all ranks: sum the ranks' bytes, compare with all their peaks
        b_tick = dist.sum(b_tick)
        spikes, events = dist.sum(spikes), dist.sum(events)
    achieved = b_tick / (t_max / total_ticks) / 1e9
    peak_total = pk['hbm_gbs'] * (dist.world if part else 1)
    line = {
        'metric': METRIC_TICKS, 'value': total_ticks * (1 if part else dist.world) / t_max, 'unit': 'ticks/s',
        'n_gpus': dist.world, 'steps': args.steps, 'warmup': args.warmup,
        'ms_per_step': t_max / args.steps * 1e3, 'higher_is_better': True,
        'scaling': 'strong' if part else 'weak',
        'vs_baseline': None, 'dtype': 'fp32', 'data': 'synthetic',
        'config': {'workload': wl, 'n': cfg.n, 'ticks_per_step': ticks,
                   'fanin': cfg.fanin if cfg.topology == 1 else None,
                   'bsr': [cfg.bsr_blocks, cfg.bsr_fill] if cfg.topology == 2 else None,
                   'spike_rate': spikes / total_ticks / cfg.n, 'weights': 'fp16' if cfg.weight_kind else 'fp32',
                   'delays': [cfg.delay_min, cfg.delay_max], 'synapses': synapses,
                   'l2': 'inputs larger than L2' if synapses * 6 > 126e6 else 'network fits in L2',
                   'parallelism': (f'rows{dist.world} + NCCL bitmask all-gather' if part and dist.world > 1
                                   else f'replicas{dist.world}'),
                   'launch': mode, 'setup_s': round(setup_s, 2)},
        'synaptic_events_per_s': events * (1 if part else dist.world) / t_max,
        'roofline': {'bound': 'hbm', 'achieved': achieved, 'peak': peak_total, 'unit': 'GB/s',
                     'frac': achieved / peak_total,
                     'traffic': tick_traffic(wl, mode, spikes / total_ticks / cfg.n) if not part else None,
                     'traffic_unit': 'bytes/tick (ncu, scaled by spike rate)', 'bytes_per_tick': b_tick,
                     'kernel': KERNEL_OF_LAUNCH[mode], 'peak_source': src},
        'gpu_launches': tick_launches(mode, ticks) * args.steps,
        'clocks': clk.summary(),
    }
    if not args.no_e2e:
        line['e2e'] = e2e_ticks(args, lib, net, cfg, ticks, dist, part)
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline and not part:
        line['cpu_baseline'] = cpu_baseline_ticks(cfg, topo)
    return line


def e2e_ticks(args, lib, net, cfg, ticks, dist, part=False):
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

    for _ in range(max(1, args.warmup)):
        step()
    dist.barrier()
    elapsed = sum(step() for _ in range(args.steps))
    t_max = dist.max(elapsed)
    return {'value': ticks * args.steps * (1 if part else dist.world) / t_max, 'unit': 'ticks/s',
            'h2d_bytes_per_step': h2d, 'd2h_bytes_per_step': d2h,
            'api': 'ng_net_set_state + ng_net_run + ng_net_stats + ng_net_get_state (host buffers)'}


def cpu_baseline_ticks(cfg, topo, budget_s=12.0):
    from oracle.net import NetOracle
    import multiprocessing
    t0 = time.time()
    orc = NetOracle(cfg, *topo.export())
    build_s = time.time() - t0
    orc.run_mt(2)
    done, el = 0, 0.0
    chunk = 5 if cfg.n > 100000 else 200
    while el < budget_s:
        t1 = time.time()
        orc.run_mt(chunk)
        el += time.time() - t1
        done += chunk
    cores = int(os.environ.get('OMP_NUM_THREADS', multiprocessing.cpu_count()))
    return {'value': done / el, 'unit': 'ticks/s', 'cores': cores, 'kind': 'port',
            'sample': f'{done} ticks of the same network (oracle/net_oracle.c on_run_mt, OpenMP), '
                      f'{el:.1f} s; oracle build {build_s:.1f} s excluded'}


# ---------------------------------------------------------------------------
# Language-core workloads.
# ---------------------------------------------------------------------------
LANG_TOKENS_PER_STEP = {'bc250': 512, 'sessions': 64}
SESSIONS = 256


def lang_tokens(workload, sessions, steps_tokens, seed_base=0):
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


def bench_lang(args, dist):
    import torch
    from neurogen_b200 import library
    from neurogen_b200.language import LanguageConfig, NativeEngine, init_packed_weights
    lib = library()
    cfg = LanguageConfig()
    w = init_packed_weights(cfg, seed=0)
    eng = NativeEngine(cfg, w)
    if args.workload == 'bc250':
        mine = [0]
    else:
        per = (args.sessions or SESSIONS) // dist.world
        mine = list(range(dist.rank * per, (dist.rank + 1) * per))
    B = len(mine)
    T = args.tokens or LANG_TOKENS_PER_STEP[args.workload]
    toks = lang_tokens(args.workload, mine, 1024 if args.workload == 'sessions' else 512)
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

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    with Clocks(torch.cuda.current_device()) as clk:
        elapsed = sum(cuda_timer(step, stream) for _ in range(args.steps))
    dist.barrier()
    t_max = dist.max(elapsed)
    total = B * T * args.steps * dist.world
    fl = lang_flops_per_token(cfg)
    pk, src = peaks()
    achieved = fl * B * T * args.steps / elapsed / 1e12
    line = {
        'metric': METRIC_TOKENS, 'value': total / t_max, 'unit': 'tokens/s', 'n_gpus': dist.world,
        'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': t_max / args.steps * 1e3,
        'higher_is_better': True, 'scaling': 'strong' if args.workload == 'sessions' else 'weak',
        'vs_baseline': None, 'dtype': 'fp32', 'data': 'synthetic',
        'config': {'workload': 'bc250_batch1' if args.workload == 'bc250' else 'bc250_sessions256',
                   'sessions': (args.sessions or SESSIONS) if args.workload == 'sessions' else 1, 'tokens_per_step': T,
                   'sessions_per_gpu': B, 'weights': 'seed-0 random init (packed 14,804,744 fp32)',
                   'l2': 'weights (59 MB) L2-resident by design', 'parallelism': f'dp{dist.world}'},
        'roofline': {'bound': 'tensor', 'achieved': achieved, 'peak': pk.get('bf16_tflops'),
                     'unit': 'TFLOP/s', 'frac': achieved / pk.get('bf16_tflops'), 'traffic': None,
                     'note': 'exact fp32 SIMT path; FLOPs per token 2x MACs', 'peak_source': src},
        'gpu_launches': lang_launches_per_token(cfg) * T * args.steps,
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
        el = dist.max(sum(e2e_step() for _ in range(args.steps)))
        line['e2e'] = {'value': total / el, 'unit': 'tokens/s', 'h2d_bytes_per_step': B * 4 * T,
                       'd2h_bytes_per_step': B * 264 * 4 * T, 'api': 'ng_pool_step (host tokens, host logits)'}
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        line['cpu_baseline'] = cpu_baseline_lang(cfg, w, toks)
    lib.ng_pool_destroy(pool)
    return line


def cpu_baseline_lang(cfg, w, toks, budget_s=10.0):
    from oracle.lang import RefEngine
    ref = RefEngine(cfg, w)
    s = np.zeros(ref.S, np.float32)
    n, t0 = 0, time.time()
    while time.time() - t0 < budget_s:
        _, s, _, _ = ref.step(int(toks[n % len(toks), 0]), s)
        n += 1
    el = time.time() - t0
    return {'value': n / el, 'unit': 'tokens/s', 'cores': 1, 'kind': 'reference',
            'sample': f'{n} tokens, one session, reference native CPU library (oracle/_ref), 1 thread'}


# ---------------------------------------------------------------------------
# Reference arm.
# ---------------------------------------------------------------------------
def reference_arm(args):
    import multiprocessing
    cores = multiprocessing.cpu_count()
    if args.workload in ('tick262k', 'bsr262k', 'tick8k', 'partitioned4m'):
        from neurogen_b200.network import Topology
        from oracle.net import NetOracle
        cfg, ticks, wl = tick_config(args.workload, args.rate)
        scale = 1
        if args.workload == 'partitioned4m':
            # 4.2 billion synapses do not fit a host-side checker: run 1/16 of the neurons with
            # the same fan-in and rate, and scale the time per tick by 16 (work per tick is
            # proportional to the neuron count).
            scale = 16
            cfg.n //= scale
            cfg.n_exc //= scale
        orc = NetOracle(cfg, *Topology(cfg).export())
        sample = 20 if cfg.n > 100000 else 200
        for _ in range(args.warmup):
            orc.run_mt(sample)
        t0 = time.time()
        for _ in range(args.steps):
            orc.run_mt(sample)
        el = time.time() - t0
        value, unit = sample * args.steps / el / scale, 'ticks/s'
        ms_per_step = el / args.steps * 1e3 * scale
        config = {'workload': wl, 'n': cfg.n * scale, 'ticks_per_step': sample,
                  'fanin': cfg.fanin if cfg.topology == 1 else None,
                  'bsr': [cfg.bsr_blocks, cfg.bsr_fill] if cfg.topology == 2 else None,
                  'spike_rate': args.rate if cfg.drive_kind == 1 else None,
                  'weights': 'fp16' if cfg.weight_kind else 'fp32', 'delays': [cfg.delay_min, cfg.delay_max]}
        scaling = 'strong' if args.workload == 'partitioned4m' else 'weak'
        kind, desc = 'port', f'{sample} ticks per step of {wl} (oracle/net_oracle.c, OpenMP)'
        if scale > 1:
            desc += f'; 1/{scale}-scale network (N={cfg.n:,}), time per tick x{scale}'
        metric = METRIC_TICKS
    else:
        from neurogen_b200.language import LanguageConfig, init_packed_weights
        from oracle.lang import RefEngine
        from concurrent.futures import ThreadPoolExecutor
        cfg = LanguageConfig()
        w = init_packed_weights(cfg, seed=0)
        wl = 'bc250_batch1' if args.workload == 'bc250' else 'bc250_sessions256'
        threads = 1 if args.workload == 'bc250' else cores
        engines = [RefEngine(cfg, w) for _ in range(threads)]
        states = [np.zeros(engines[0].S, np.float32) for _ in range(threads)]
        per_step = 8 if args.workload == 'bc250' else 2

        def work(k):
            for i in range(per_step):
                _, states[k], _, _ = engines[k].step((k * 7 + i) % 264, states[k])

        with ThreadPoolExecutor(threads) as pool:
            for _ in range(args.warmup):
                list(pool.map(work, range(threads)))
            t0 = time.time()
            for _ in range(args.steps):
                list(pool.map(work, range(threads)))
            el = time.time() - t0
        value, unit = threads * per_step * args.steps / el, 'tokens/s'
        ms_per_step = el / args.steps * 1e3
        config = {'workload': wl, 'sessions': 1 if args.workload == 'bc250' else SESSIONS,
                  'tokens_per_step': per_step * threads}
        scaling = 'weak' if args.workload == 'bc250' else 'strong'
        kind = 'reference'
        desc = f'{per_step} tokens per step on each of {threads} independent sessions (one engine per thread)'
        metric = METRIC_TOKENS
    return {'metric': metric, 'value': value, 'unit': unit, 'n_gpus': int(os.environ.get('WORLD_SIZE', '1')),
            'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': ms_per_step, 'higher_is_better': True,
            'scaling': scaling, 'impl': 'reference', 'dtype': 'fp32', 'data': 'synthetic', 'config': config,
            'cpu_baseline': {'value': value, 'unit': unit, 'cores': cores if kind == 'port' or threads > 1 else 1,
                             'kind': kind, 'sample': desc},
            'e2e': {'value': value, 'unit': unit, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}


def main():
    args = parse()
    dist = Dist()
    if args.impl == 'reference':
        if dist.rank == 0:
            print(json.dumps(reference_arm(args)), flush=True)
        return
    import torch
    torch.cuda.set_device(dist.local)
    dist.init(dist.local)
    try:
        if args.workload in ('bc250', 'sessions'):
            line = bench_lang(args, dist)
        else:
            line = bench_ticks(args, dist)
        if dist.rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        dist.close()


if __name__ == '__main__':
    main()
