"""Generate tests/golden/net_golden.npz from the reference's NumPy simulator.

Runs neurogen/biology.py (the reference) with frozen synapses (plasticity off) and no Poisson
background, driven by a constant current into layer-4 excitatory cells, and records its spikes
and membrane voltages.  The anatomy is relabelled so that excitatory cells come first (the
network engine's convention); the dynamics are equivariant under that permutation.

Usage: python tests/golden/make_net_golden.py [/path/to/reference]
"""
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
REFERENCE = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ['NEUROGEN_REFERENCE'])
sys.path.insert(0, str(REFERENCE))

from neurogen.biology import BiologicalNetwork, BiologyConfig  # noqa: E402

TICKS = 200


def main():
    net = BiologicalNetwork(BiologyConfig(seed=3, plasticity=False, background_hz=0.0))
    a = net.anatomy
    order = np.concatenate([np.flatnonzero(a.excitatory), np.flatnonzero(~a.excitatory)])
    rank = np.empty_like(order)
    rank[order] = np.arange(len(order))
    active = net.active & (net.weight > 0)
    pre = rank[a.pre[active]].astype(np.int32)
    post = rank[a.post[active]].astype(np.int32)
    delay = a.delay[active].astype(np.int32)
    weight = np.where(net.excitatory_edge[active], net.weight[active], -net.weight[active])
    current = net.current('sensory', 0, 4, 400) + net.current('association', 1, 4, 400)
    v0 = net.voltage.copy()
    spikes, volts, ge = [], [], []
    for _ in range(TICKS):
        spikes.append(net.step(current)[order])
        volts.append(net.voltage[order].copy())
        ge.append(net.ge[order].copy())
    np.savez_compressed(
        ROOT / 'tests' / 'golden' / 'net_golden.npz',
        n=np.int32(a.size), n_exc=np.int32(a.excitatory.sum()), pre=pre, post=post, delay=delay,
        weight=weight, v0=v0[order], current=current[order], spikes=np.array(spikes),
        voltage=np.array(volts[:100]), ge=np.array(ge[:50]))
    print('spikes per tick', np.array(spikes).sum(1).mean(), 'synapses', len(pre))


if __name__ == '__main__':
    main()
