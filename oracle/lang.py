"""ORACLE (test infrastructure only): ctypes access to the language-core checkers.

* ``RefEngine`` -- the reference's own native CPU engine, compiled from its sources by
  ``oracle/Makefile`` into ``oracle/_ref/libneurogen_ref.so`` (src/native/NeuralEngine.cpp,
  src/native/CPUBackend.cpp).
* ``OracleEngine`` -- this repo's C restatement (``oracle/lang_oracle.c``), bit-identical to
  the reference library, which can also record every tick's spikes and the smallest spike
  margin.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use this module.
"""
import ctypes as ct
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF_LIB = HERE / '_ref' / 'libneurogen_ref.so'
ORACLE_LIB = HERE / 'liboracle.so'
F32 = np.ctypeslib.ndpointer(dtype=np.float32, flags='C_CONTIGUOUS')
VOCAB = 264


def _load(path):
    if not path.is_file():
        raise FileNotFoundError(f'{path} missing; run `make -C oracle`')
    return ct.CDLL(str(path))


class RefEngine:
    """Reference native engine (backend "cpu"), one handle, single session per call."""

    def __init__(self, config, weights):
        lib = self.lib = _load(REF_LIB)
        lib.ng_create.argtypes = [ct.c_int] * 5 + [F32, ct.c_size_t, ct.c_char_p]
        lib.ng_create.restype = ct.c_void_p
        lib.ng_destroy.argtypes = [ct.c_void_p]
        lib.ng_error.restype = ct.c_char_p
        lib.ng_step.argtypes = [ct.c_void_p, ct.c_int, F32, ct.c_size_t, F32, F32, F32, F32]
        lib.ng_advance.argtypes = [ct.c_void_p, F32, F32, ct.c_size_t, ct.c_int, F32, F32, F32]
        self.config = config
        w = np.ascontiguousarray(weights, dtype=np.float32)
        c = config
        self.h = lib.ng_create(c.columns, c.width, c.regions, c.ticks, c.idle_steps, w, w.size, b'cpu')
        if not self.h:
            raise ValueError(lib.ng_error().decode())
        self.S = c.regions * (5 * c.columns * 64 + c.width)

    def __del__(self):
        if getattr(self, 'h', None):
            self.lib.ng_destroy(self.h)

    def step(self, token, state):
        state = np.ascontiguousarray(state, np.float32)
        nxt = np.empty_like(state)
        logits = np.empty(VOCAB, np.float32)
        hidden = np.empty(self.config.width, np.float32)
        act = np.empty(1, np.float32)
        if self.lib.ng_step(self.h, int(token), state, self.S, nxt, logits, hidden, act):
            raise ValueError(self.lib.ng_error().decode())
        return logits, nxt, act[0], hidden

    def advance(self, x, state, idle):
        state = np.ascontiguousarray(state, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        nxt = np.empty_like(state)
        hidden = np.empty(self.config.width, np.float32)
        act = np.empty(1, np.float32)
        if self.lib.ng_advance(self.h, x, state, self.S, int(idle), nxt, hidden, act):
            raise ValueError(self.lib.ng_error().decode())
        return hidden, nxt, act[0]


class OracleEngine:
    """C restatement of the reference engine with per-tick spike recording."""

    def __init__(self, config, weights):
        lib = self.lib = _load(ORACLE_LIB)
        lib.og_create.argtypes = [ct.c_int] * 5 + [F32, ct.c_size_t]
        lib.og_create.restype = ct.c_void_p
        lib.og_destroy.argtypes = [ct.c_void_p]
        lib.og_step.argtypes = [ct.c_void_p, ct.c_int, F32, F32, F32, F32, F32, ct.c_void_p, ct.c_size_t]
        lib.og_advance.argtypes = [ct.c_void_p, F32, F32, ct.c_int, F32, F32, F32, ct.c_void_p, ct.c_size_t]
        lib.og_min_margin.restype = ct.c_double
        lib.og_min_margin.argtypes = [ct.c_void_p]
        lib.og_reset_margin.argtypes = [ct.c_void_p]
        self.config = config
        w = np.ascontiguousarray(weights, dtype=np.float32)
        c = config
        self.h = lib.og_create(c.columns, c.width, c.regions, c.ticks, c.idle_steps, w, w.size)
        if not self.h:
            raise ValueError('oracle rejected the configuration or weights')
        lib.og_reset_margin(self.h)
        self.S = c.regions * (5 * c.columns * 64 + c.width)
        self.n = c.columns * 64

    def __del__(self):
        if getattr(self, 'h', None):
            self.lib.og_destroy(self.h)

    def spikes_per_step(self):
        c = self.config
        return (1 + c.idle_steps) * c.regions * c.ticks * self.n

    def step(self, token, state, record=False):
        """-> logits, next_state, activity, hidden[, spikes uint8 [(1+idle)*R*T, n]]"""
        state = np.ascontiguousarray(state, np.float32)
        nxt = np.empty_like(state)
        logits = np.empty(VOCAB, np.float32)
        hidden = np.empty(self.config.width, np.float32)
        act = np.empty(1, np.float32)
        spikes = np.zeros(self.spikes_per_step(), np.uint8) if record else None
        if self.lib.og_step(self.h, int(token), state, nxt, logits, hidden, act,
                            None if spikes is None else spikes.ctypes.data_as(ct.c_void_p),
                            0 if spikes is None else spikes.size):
            raise ValueError('oracle step failed')
        out = (logits, nxt, act[0], hidden)
        return out + (spikes.reshape(-1, self.n),) if record else out

    def advance(self, x, state, idle):
        state = np.ascontiguousarray(state, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        nxt = np.empty_like(state)
        hidden = np.empty(self.config.width, np.float32)
        act = np.empty(1, np.float32)
        if self.lib.og_advance(self.h, x, state, int(idle), nxt, hidden, act, None, 0):
            raise ValueError('oracle advance failed')
        return hidden, nxt, act[0]

    def min_margin(self):
        return self.lib.og_min_margin(self.h)

    def reset_margin(self):
        self.lib.og_reset_margin(self.h)


def last_spikes(state, config):
    """The last_spikes field of every region of a packed state [.., S] (0/1 floats)."""
    n, w = config.columns * 64, config.width
    rs = 5 * n + w
    return np.stack([state[..., r * rs + 3 * n: r * rs + 4 * n] for r in range(config.regions)], -2)


def seeded_weights(columns=32, width=768, regions=4, seed=0):
    """Packed weights of the reference ``LanguageModel`` after ``torch.manual_seed(seed)``, for the
    CPU legs (no CUDA library).  The parameters the native stream holds are drawn with the same
    torch modules in the construction order of neurogen/language/model.py:103-116 (embedding with
    its padding row zeroed, then per region input / feedback / output Linear layers, then the
    head); constant-initialised parameters draw nothing.  Pinned by the SHA-256 of the seed-0
    BC-250 stream in tests/golden/lang_golden.npz."""
    import torch
    c, w = columns, width
    with torch.random.fork_rng(devices=[]):
        torch.manual_seed(seed)
        parts = [torch.nn.Embedding(VOCAB, w, padding_idx=256).weight]
        for _ in range(regions):
            inp = torch.nn.Linear(w, c * 12)
            fb = torch.nn.Linear(w, c * 29, bias=False)
            out = torch.nn.Linear(c * 100, w)
            parts += [torch.full((c, 64, 64), -1.8), inp.weight, inp.bias, fb.weight, out.weight, out.bias,
                      torch.ones(w), torch.zeros(w), torch.full((w,), 2.9)]
        head = torch.nn.Linear(w, VOCAB)
        parts += [head.weight, head.bias]
        return np.concatenate([p.detach().float().numpy().reshape(-1) for p in parts]).astype(np.float32)
