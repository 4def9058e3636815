"""Generate tests/golden/net_plastic_golden.npz from the reference's NumPy simulator with learning.

Runs neurogen/biology.py (the reference) with plasticity on (STDP, inhibitory homeostasis,
synaptic scaling; biology.py:182-218), structural rewiring and the Poisson background off, driven
by a constant current into layer-4 excitatory cells, and records every spike of 300 ticks and the
weights, traces and rates after ticks 100 and 300.  The anatomy is relabelled so that excitatory
cells come first (the network engine's convention); the dynamics are equivariant under that
permutation.  Contacts are the active ones, in the reference's contact order.

Usage: python tests/golden/make_net_plastic_golden.py [/path/to/reference]
(the reference checkout: the argument, else NEUROGEN_REFERENCE)
"""
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
REFERENCE = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ['NEUROGEN_REFERENCE'])
sys.path.insert(0, str(REFERENCE))

from neurogen.biology import BiologicalNetwork, BiologyConfig  # noqa: E402

TICKS = 300
SNAP = (100, 300)


def main():
    net = BiologicalNetwork(BiologyConfig(seed=5, plasticity=True, structural=False, background_hz=0.0))
    a = net.anatomy
    order = np.concatenate([np.flatnonzero(a.excitatory), np.flatnonzero(~a.excitatory)])
    rank = np.empty_like(order)
    rank[order] = np.arange(len(order))
    active = np.flatnonzero(net.active & (net.weight > 0))
    exc_edge = net.excitatory_edge[active]

    def signed(w):
        return np.where(exc_edge, w[active], -w[active])

    out = dict(n=np.int32(a.size), n_exc=np.int32(a.excitatory.sum()),
               pre=rank[a.pre[active]].astype(np.int32), post=rank[a.post[active]].astype(np.int32),
               delay=a.delay[active].astype(np.int32), weight=signed(net.weight),
               v0=net.voltage[order].copy())
    current = net.current('sensory', 0, 4, 400) + net.current('association', 1, 4, 400)
    out['current'] = current[order]
    spikes = []
    for t in range(1, TICKS + 1):
        spikes.append(net.step(current)[order])
        if t in SNAP:
            out[f'weight_{t}'] = signed(net.weight)
            for k in ('pre_trace', 'potential_trace', 'coactivity', 'usage'):
                out[f'{k}_{t}'] = getattr(net, k)[active].copy()
            out[f'post_trace_{t}'] = net.post_trace[order].copy()
            out[f'rate_{t}'] = net.rate[order].copy()
            out[f'voltage_{t}'] = net.voltage[order].copy()
    out['spikes'] = np.array(spikes)
    np.savez_compressed(ROOT / 'tests' / 'golden' / 'net_plastic_golden.npz', **out)
    w0, w1 = out['weight'], out[f'weight_{TICKS}']
    print('spikes per tick', out['spikes'].sum(1).mean(), 'contacts', len(w0),
          'weights changed', int((w0 != w1).sum()), 'max |dw|', float(np.abs(w1 - w0).max()))


if __name__ == '__main__':
    main()
