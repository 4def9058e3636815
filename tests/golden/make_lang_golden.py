"""Generate tests/golden/lang_golden.npz from the reference itself.

Run in a container where the reference checkout is importable (its path as the first argument, or in NEUROGEN_REFERENCE) after
`make -C oracle`.  It records, for fixed seeded inputs:

* small config (columns 3, width 17, regions 2, ticks 3, idle 1) -- the configuration of the
  reference's own parity test (tests/test_native.py:29-39) -- with raw recurrent weights
  perturbed by a seeded N(0, 0.3) so the recurrent matrix is non-uniform:
    - logits / hidden / activity / full state after every token, from the reference PyTorch
      model (neurogen/language/model.py), the independent reference;
    - SHA-256 of every output of the reference native CPU library (oracle/_ref), which the C
      restatement must reproduce bit for bit;
* the BC-250 profile (configs/language_bc250.json) at seed 0: SHA-256 of the packed weights
  and of the native library's outputs for the first tokens of the seed-0 stream.

Usage: python tests/golden/make_lang_golden.py [/path/to/reference]
"""
import hashlib
import os
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
REFERENCE = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ['NEUROGEN_REFERENCE'])
sys.path.insert(0, str(REFERENCE))
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / 'neurogen-2.5_b200'))

from neurogen.language.config import LanguageConfig as RefConfig  # noqa: E402
from neurogen.language.model import LanguageModel  # noqa: E402
from neurogen.language.native import packed_weights  # noqa: E402
from oracle.lang import RefEngine  # noqa: E402

SMALL = dict(columns=3, width=17, regions=2, ticks=3, idle_steps=1, speech_width=16, mel_bins=8)


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a, np.float32).tobytes())
    return h.hexdigest()


def small_model():
    torch.manual_seed(7)
    model = LanguageModel(RefConfig(**SMALL)).eval()
    g = torch.Generator().manual_seed(11)
    with torch.no_grad():
        for region in model.regions:
            region.raw_weight.add_(torch.randn(region.raw_weight.shape, generator=g) * .3)
    return model


def state_vec(state):
    return torch.cat([t.reshape(-1) for r in state for t in r]).numpy()


def main():
    out = {}
    model = small_model()
    weights = packed_weights(model).astype(np.float32)
    out['small_weights'] = weights
    tokens = np.array([257] + list(range(1, 24)), np.int64)
    out['small_tokens'] = tokens
    ref = RefEngine(type('C', (), SMALL)(), weights)
    st_t = None
    st_n = np.zeros(ref.S, np.float32)
    logits_t, states_t, hidden_t, act_t, dig = [], [], [], [], []
    with torch.no_grad():
        for tok in tokens:
            lt, st_t, at, ht = model.step(torch.tensor([int(tok)]), st_t)
            logits_t.append(lt[0].numpy())
            states_t.append(state_vec(st_t))
            hidden_t.append(ht[0].numpy())
            act_t.append(float(at))
            ln, st_n, an, hn = ref.step(int(tok), st_n)
            dig.append(digest(ln, st_n, hn, np.array([an], np.float32)))
        # idle advances after the tokens (reference tests/test_native.py:62-66)
        for _ in range(8):
            ht, st_t, at = model.advance(torch.zeros(1, SMALL['width']), st_t, idle=True)
            states_t.append(state_vec(st_t))
            hidden_t.append(ht[0].numpy())
            act_t.append(float(at))
            hn, st_n, an = ref.advance(np.zeros(SMALL['width'], np.float32), st_n, True)
            dig.append(digest(st_n, hn, np.array([an], np.float32)))
    out['small_torch_logits'] = np.stack(logits_t)
    out['small_torch_state'] = np.stack(states_t)
    out['small_torch_hidden'] = np.stack(hidden_t)
    out['small_torch_activity'] = np.array(act_t, np.float32)
    out['small_native_sha'] = np.array(dig)

    # BC-250 profile, seed 0.
    torch.manual_seed(0)
    bc = LanguageModel(RefConfig())
    wb = packed_weights(bc).astype(np.float32)
    out['bc250_weights_sha'] = np.array(hashlib.sha256(wb.tobytes()).hexdigest())
    g = torch.Generator().manual_seed(0)
    stream = torch.randint(0, 264, (512,), generator=g).numpy()
    out['bc250_tokens'] = stream.astype(np.int64)
    refb = RefEngine(RefConfig(), wb)
    st = np.zeros(refb.S, np.float32)
    dig, logits = [], []
    for tok in stream[:6]:
        ln, st, an, hn = refb.step(int(tok), st)
        dig.append(digest(ln, st, hn, np.array([an], np.float32)))
        logits.append(ln)
    out['bc250_native_sha'] = np.array(dig)
    out['bc250_native_logits'] = np.stack(logits)
    np.savez_compressed(ROOT / 'tests' / 'golden' / 'lang_golden.npz', **out)
    print('wrote', ROOT / 'tests' / 'golden' / 'lang_golden.npz')


if __name__ == '__main__':
    main()
