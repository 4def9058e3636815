"""Neuron-partitioned networks (rows of the network split over GPUs, spike bitmask all-gathered).

CPU: each partition's generated synapses are exactly the synapses of the whole network that end on
its neurons (union over ranks == the unpartitioned network), also checked with two gloo ranks in
separate processes.  GPU (two devices): a 2-rank run equals the unpartitioned network bit for bit --
every spike of every tick, spike/event counters, and each rank's state slice.
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import ROOT
from neurogen_b200.network import Topology, default_config


def edges_sorted(e):
    pre, post, delay, w = e
    order = np.lexsort((w.view(np.int32), delay, post, pre))
    return tuple(x[order] for x in (pre, post, delay, w))


@pytest.mark.parametrize('topology', ['fixed_fanin', 'erdos_renyi'])
def test_partitions_union_to_the_whole_network(topology):
    base = dict(n=4096, n_exc=3276, topology=topology, fanin=40, p_connect=0.01, weight_kind='halfnormal_f16',
                w_mu=0.0, w_sigma=0.05, seed=21)
    full = edges_sorted(Topology(default_config(**base)).export())
    parts = [Topology(default_config(part_rank=r, part_world=4, **base)).export() for r in range(4)]
    for r, (pre, post, delay, w) in enumerate(parts):
        assert post.min() >= r * 1024 and post.max() < (r + 1) * 1024
    union = edges_sorted(tuple(np.concatenate(x) for x in zip(*parts)))
    for a, b in zip(full, union):
        assert np.array_equal(a, b)


def test_partition_validation():
    with pytest.raises(ValueError, match='divisible'):
        Topology(default_config(n=1000, part_rank=0, part_world=3))
    with pytest.raises(ValueError, match='part_rank'):
        Topology(default_config(n=1024, part_rank=4, part_world=4))
    with pytest.raises(ValueError, match='CSR'):
        Topology(default_config(n=1024, topology='bsr16', bsr_blocks=8, weight_kind='halfnormal_f16', storage='bsr',
                                part_rank=0, part_world=2))


GLOO_WORKER = r'''
import os, sys
import numpy as np
import torch.distributed as dist
sys.path[:0] = [{root!r}, {pkg!r}]
from neurogen_b200.network import Topology, default_config
dist.init_process_group('gloo')
rank, world = dist.get_rank(), dist.get_world_size()
cfg = default_config(n=2048, n_exc=1638, topology='fixed_fanin', fanin=24, seed=5, part_rank=rank, part_world=world)
pre, post, delay, w = Topology(cfg).export()
counts = [None] * world
dist.all_gather_object(counts, (len(pre), int(post.min()), int(post.max())))
if rank == 0:
    full = Topology(default_config(n=2048, n_exc=1638, topology='fixed_fanin', fanin=24, seed=5)).export()
    assert sum(c[0] for c in counts) == len(full[0]) == 2048 * 24, counts
    assert counts[0][2] < 1024 <= counts[1][1], counts
dist.barrier()
dist.destroy_process_group()
print('ok', rank)
'''


def test_two_gloo_ranks_generate_disjoint_partitions(tmp_path):
    script = tmp_path / 'w.py'
    script.write_text(GLOO_WORKER.format(root=str(ROOT), pkg=str(ROOT / 'neurogen-2.5_b200')))
    env = dict(os.environ, MASTER_ADDR='127.0.0.1')
    out = subprocess.run([sys.executable, '-m', 'torch.distributed.run', '--nnodes=1', '--nproc-per-node=2',
                          '--master-addr', '127.0.0.1', '--master-port', '29641', str(script)],
                         capture_output=True, text=True, timeout=300, env=env)
    assert out.returncode == 0, out.stderr[-3000:]
    assert out.stdout.count('ok') == 2


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason='needs two GPUs')
@pytest.mark.parametrize('exchange', ['peer', 'nccl'])
def test_two_gpu_partition_equals_whole_network(tmp_path, exchange):
    """Two ranks over NVLink with the one-sided peer exchange (default) or the NCCL all-gather:
    every rank's whole-network raster equals the unpartitioned network's (recorded ticks, after
    100 graph-replayed ticks, and again after a collective state load rewinds both ranks)."""
    env = dict(os.environ, MASTER_ADDR='127.0.0.1', NCCL_NVLS_ENABLE='0',
               NEUROGEN_PEER_EXCHANGE='1' if exchange == 'peer' else '0')
    cmd = ['timeout', '-k', '30', '300', sys.executable, '-m', 'torch.distributed.run', '--nnodes=1',
           '--nproc-per-node=2', '--master-addr', '127.0.0.1', '--master-port', '29643',
           str(ROOT / 'tests' / 'net_partition_worker.py'), str(tmp_path)]
    out = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert out.returncode == 0, out.stderr[-4000:]
    full = np.load(tmp_path / 'full.npz')
    ranks = [np.load(tmp_path / f'rank{r}.npz') for r in range(2)]
    for r in ranks:
        assert str(r['exchange']) == exchange
        assert np.array_equal(r['spikes'], full['spikes'])   # whole-network raster on every rank
        assert np.array_equal(r['mid'], full['mid'])
        assert np.array_equal(r['tail'], full['tail'])       # after 100 graph-replayed ticks
        assert np.array_equal(r['again'], full['mid'])       # rewound to tick 60 and run again
    assert full['counts'][:, 0].sum() > 1000
    assert sum(int(r['stats'][0]) for r in ranks) == int(full['stats'][0])
    assert sum(int(r['stats'][1]) for r in ranks) == int(full['stats'][1])
    half = 65536 // 2
    for k in ('v', 'a', 'ge', 'gi', 'ref'):
        assert np.array_equal(np.concatenate([r[k] for r in ranks]), full[k]), k
    ring = np.concatenate([r['ring'] for r in ranks], axis=1)
    assert np.array_equal(ring, full['ring'])
    assert ranks[0]['v'].shape[0] == half


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason='needs two GPUs')
def test_two_gpu_exchange_wait_runs_out_cleanly(tmp_path):
    """The peer exchange's wait is bounded: when one rank never runs its ticks (it stays between
    steps, nothing of it in flight), the other rank's wait gives up after its 2 s limit, the run
    raises, and the process goes on to build and run a new network on the same GPU."""
    env = dict(os.environ, MASTER_ADDR='127.0.0.1', NCCL_NVLS_ENABLE='0', NEUROGEN_PEER_EXCHANGE='1')
    cmd = ['timeout', '-k', '30', '300', sys.executable, '-m', 'torch.distributed.run', '--nnodes=1',
           '--nproc-per-node=2', '--master-addr', '127.0.0.1', '--master-port', '29645',
           str(ROOT / 'tests' / 'net_partition_worker.py'), str(tmp_path), 'stall']
    out = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert out.returncode == 0, out.stderr[-4000:]
    r = np.load(tmp_path / 'stall.npz')
    assert str(r['exchange']) == 'peer'
    assert 'timed out' in str(r['msg']), str(r['msg'])
    assert 1.5 < float(r['took']) < 60.0
    assert int(r['alive']) > 0
