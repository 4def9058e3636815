"""Worker for tests/test_partition.py: one rank of a neuron-partitioned network.

Launched as `torchrun --nproc-per-node 2 tests/net_partition_worker.py OUT`.  Every rank builds its
partition (sharing one NCCL id through torch.distributed), runs ticks recording the whole network's
spike bitmask, and saves its raster, counters and state slice; rank 0 also runs the unpartitioned
network on its own GPU for comparison.
"""
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / 'neurogen-2.5_b200')]

from neurogen_b200.network import Network, default_config, nccl_unique_id  # noqa: E402


def config(rank, world):
    return default_config(n=65536, n_exc=52428, topology='fixed_fanin', fanin=96, weight_kind='halfnormal_f16',
                          w_mu=0.0, w_sigma=0.05, drive_kind='conductance', drive_p=0.03, drive_ns=18.0,
                          seed=12, part_rank=rank, part_world=world)


def stall(out, rank, world, nccl_id):
    """Failure path of the peer exchange: rank 1 stays between steps and never runs its ticks, so
    rank 0's wait for its spikes runs out (2 s); rank 0's run must raise, and the same process must
    then build and run a new network.  No kernel or collective of rank 1 is in flight meanwhile."""
    import time
    net = Network.partitioned(config(rank, world), nccl_id)
    msg, took = '', 0.0
    if rank == 0:
        t0 = time.time()
        try:
            net.run(3)
        except ValueError as e:
            msg = str(e)
        took = time.time() - t0
        after = Network(config(0, 0))
        _, c = after.run(20)
        alive = int(c[:, 0].sum())
        after.close()
        np.savez(out / 'stall.npz', msg=np.array(msg), took=took, alive=alive, exchange=np.array(net.exchange))
    dist.barrier()
    net.close()
    dist.destroy_process_group()


def main():
    out = Path(sys.argv[1])
    rank, world, local = int(os.environ['RANK']), int(os.environ['WORLD_SIZE']), int(os.environ['LOCAL_RANK'])
    torch.cuda.set_device(local)
    import datetime
    dist.init_process_group('gloo', timeout=datetime.timedelta(seconds=120))
    ids = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(ids, src=0)
    if len(sys.argv) > 2 and sys.argv[2] == 'stall':
        stall(out, rank, world, ids[0])
        return
    net = Network.partitioned(config(rank, world), ids[0])
    spikes, counts = net.run(60)
    snap = net.get_state()              # tick 60
    mid, _ = net.run(30)
    net.run(100, record=False)          # graph path with the exchange captured
    tail, _ = net.run(5)
    st = net.get_state()
    stats = np.array(net.stats())
    net.set_state(**snap)               # collective: every rank rewinds to tick 60
    again, _ = net.run(30)
    np.savez(out / f'rank{rank}.npz', spikes=spikes, counts=counts, mid=mid, tail=tail, again=again, stats=stats,
             exchange=np.array(net.exchange), **{k: st[k] for k in ('v', 'a', 'ge', 'gi', 'ref', 'ring')})
    if rank == 0:
        full = Network(config(0, 0))
        fs, fc = full.run(60)
        fm, _ = full.run(30)
        full.run(100, record=False)
        ft, _ = full.run(5)
        fst = full.get_state()
        np.savez(out / 'full.npz', spikes=fs, counts=fc, mid=fm, tail=ft, stats=np.array(full.stats()),
                 **{k: fst[k] for k in ('v', 'a', 'ge', 'gi', 'ref', 'ring')})
    dist.barrier()
    net.close()
    dist.destroy_process_group()


if __name__ == '__main__':
    main()
