"""Host-side mirror of the reference's native language adapter, on the B200 engine.

Reference interface: ``neurogen/language/native.py`` (``NativeLanguageModel``,
``packed_weights``, ``library``), ``neurogen/language/config.py`` (``LanguageConfig``) and
``neurogen/language/training.py:39-45`` (``load_checkpoint``).  Names, argument meaning,
state layout and error messages follow those files; the difference is that a batch of
sessions is one engine call (``ng_step_batch``) instead of a Python loop over items
(native.py:128-137), and the compute runs on an sm_100 GPU.
"""
from dataclasses import dataclass, asdict
import ctypes as ct

import numpy as np
import torch

from ._lib import library, F32

VOCAB = 264
PAD = 256
FORMAT = 'neurogen-language-v2'
NATIVE_DEVICES = ('native-cuda',)
# Laminar table (layer, excitatory, inhibitory), neurogen/anatomy.py:9.
LAYERS = ((1, 0, 2), (2, 8, 2), (3, 8, 2), (4, 12, 3), (5, 12, 3), (6, 10, 2))


@dataclass(frozen=True)
class LanguageConfig:
    """Sizes of the language core (neurogen/language/config.py:5-29)."""
    columns: int = 32
    width: int = 768
    regions: int = 4
    ticks: int = 2
    idle_steps: int = 1
    mel_bins: int = 64
    speech_width: int = 256

    def __post_init__(self):
        for name in ('columns', 'width', 'regions', 'ticks', 'mel_bins', 'speech_width'):
            if type(getattr(self, name)) is not int or getattr(self, name) < 1:
                raise ValueError(f'{name} must be a positive integer')
        if type(self.idle_steps) is not int or not 0 <= self.idle_steps <= 16:
            raise ValueError('idle_steps must be between 0 and 16')

    @classmethod
    def preset(cls, name):
        presets = {'tiny': dict(columns=1, width=32, regions=2, speech_width=32, idle_steps=0),
                   'laptop': dict(columns=4, width=128, regions=3, speech_width=128),
                   'bc250': {}, 'large': dict(columns=64, width=1024, regions=4)}
        if name not in presets:
            raise ValueError(f'Unknown preset: {name}')
        return cls(**presets[name])


def unit_tables():
    """Per-unit layer, excitatory flag and the input/feedback/output id lists of a column."""
    layer, exc = [], []
    for lay, ne, ni in LAYERS:
        for k in range(ne + ni):
            layer.append(lay)
            exc.append(k < ne)
    layer = np.array(layer)
    exc = np.array(exc)
    input_ids = np.flatnonzero((layer == 4) & exc)
    feedback_ids = np.flatnonzero((layer >= 5) | (layer == 1))
    output_ids = np.flatnonzero(exc)
    return layer, exc, input_ids, feedback_ids, output_ids


def canonical_buffers():
    """Architecture buffers a ColumnRegion must hold (neurogen/language/model.py:40-59)."""
    layer, exc, input_ids, feedback_ids, output_ids = unit_tables()
    lay = torch.tensor(layer)
    e = torch.tensor(exc)
    mask = lay[:, None] == lay[None, :]
    for pre, post in ((4, 2), (4, 3), (2, 3), (3, 5), (5, 6), (6, 4)):
        mask |= (lay[:, None] == post) & (lay[None, :] == pre)
    mask |= (~e[None, :]) & ((lay[:, None] - lay[None, :]).abs() <= 1)
    mask.fill_diagonal_(False)
    return {
        'mask': mask.float(),
        'sign': torch.where(e, 1., -1.),
        'membrane_decay': torch.where(e, .6, .4),
        'threshold': torch.where(e, 1., .6),
        'baseline': torch.where(e, .15, .35),
        'adaptation_increment': torch.where(e, .03, 0.),
        'input_ids': torch.tensor(input_ids),
        'feedback_ids': torch.tensor(feedback_ids),
        'output_ids': torch.tensor(output_ids),
        'layer': lay,
    }


def state_size(config):
    return config.regions * (5 * config.columns * 64 + config.width)


def parameter_count(config):
    c, w = config.columns, config.width
    region = c * 4096 + c * 12 * (w + 1) + c * 29 * w + w * (c * 100 + 1) + 3 * w
    return 528 * w + 264 + config.regions * region


def packed_from_state_dict(config, sd):
    """Packed fp32 weight stream in the order of neurogen/language/native.py:46-52."""
    names = ['embedding.weight']
    for r in range(config.regions):
        p = f'regions.{r}.'
        names += [p + 'raw_weight', p + 'input.weight', p + 'input.bias', p + 'feedback.weight',
                  p + 'output.weight', p + 'output.bias', p + 'norm.weight', p + 'norm.bias',
                  p + 'memory_decay']
    names += ['head.weight', 'head.bias']
    return np.concatenate([sd[n].detach().cpu().float().numpy().reshape(-1) for n in names])


def check_architecture(config, sd):
    """Reject checkpoints whose architecture buffers differ (native.py:252-261)."""
    expected = canonical_buffers()
    for r in range(config.regions):
        for name, value in expected.items():
            key = f'regions.{r}.{name}'
            if key in sd and not torch.equal(sd[key].cpu(), value):
                raise ValueError(f'Native architecture buffer differs from simplified model: {name}')


def packed_weights(model):
    """Packed weights of a torch model with the reference parameter names."""
    return packed_from_state_dict(model.config, dict(model.named_parameters()))


def init_packed_weights(config=None, seed=0):
    """Seeded random-init weights of ``LanguageModel(config)`` as a packed stream.

    Rebuilds the parameters that the native stream holds, with the same torch modules in the
    same construction order as neurogen/language/model.py:103-116 (Embedding with padding row,
    then per region Linear input / feedback / output with torch's default init, then the head),
    so ``torch.manual_seed(seed)`` yields bit-identical values without the reference package.
    Constant-initialised parameters (raw_weight -1.8, memory_decay 2.9, LayerNorm 1/0) draw no
    random numbers.
    """
    config = config or LanguageConfig()
    c, w = config.columns, config.width
    with torch.random.fork_rng(devices=[]):
        torch.manual_seed(seed)
        sd = {'embedding.weight': torch.nn.Embedding(VOCAB, w, padding_idx=PAD).weight}
        for r in range(config.regions):
            p = f'regions.{r}.'
            sd[p + 'raw_weight'] = torch.full((c, 64, 64), -1.8)
            inp = torch.nn.Linear(w, c * 12)
            fb = torch.nn.Linear(w, c * 29, bias=False)
            out = torch.nn.Linear(c * 100, w)
            sd.update({p + 'input.weight': inp.weight, p + 'input.bias': inp.bias,
                       p + 'feedback.weight': fb.weight, p + 'output.weight': out.weight,
                       p + 'output.bias': out.bias, p + 'norm.weight': torch.ones(w),
                       p + 'norm.bias': torch.zeros(w), p + 'memory_decay': torch.full((w,), 2.9)})
        head = torch.nn.Linear(w, VOCAB)
        sd['head.weight'], sd['head.bias'] = head.weight, head.bias
        return packed_from_state_dict(config, sd).astype(np.float32)


def load_checkpoint(path):
    """Config and packed weights of a ``neurogen-language-v2`` checkpoint (training.py:39-45)."""
    payload = torch.load(path, map_location='cpu', weights_only=True)
    if payload.get('format') != FORMAT:
        raise ValueError('Unsupported language checkpoint; biological checkpoints are separate')
    config = LanguageConfig(**payload['config'])
    sd = payload['model']
    check_architecture(config, sd)
    return config, packed_from_state_dict(config, sd), payload


class NativeEngine:
    """Owns one ``ng_create`` handle: an immutable weight snapshot on the GPU."""

    def __init__(self, config, weights):
        self.lib = library()
        self.config = config
        weights = np.ascontiguousarray(weights, dtype=np.float32)
        c = config
        self.handle = self.lib.ng_create(c.columns, c.width, c.regions, c.ticks, c.idle_steps,
                                         weights, weights.size, b'cuda')
        if not self.handle:
            raise ValueError(self.lib.ng_error().decode())
        self.backend = self.lib.ng_backend(self.handle).decode()
        self.state_size = self.lib.ng_state_size(self.handle)

    def close(self):
        if getattr(self, 'handle', None):
            self.lib.ng_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()

    def _check(self, code):
        if code:
            raise ValueError(self.lib.ng_error().decode())

    def step_batch(self, tokens, state):
        """tokens int [B]; state fp32 [B, S] -> (logits, next_state, activity, hidden)."""
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        state = np.ascontiguousarray(state, dtype=np.float32)
        B = tokens.shape[0]
        nxt = np.empty_like(state)
        logits = np.empty((B, VOCAB), np.float32)
        hidden = np.empty((B, self.config.width), np.float32)
        act = np.empty(B, np.float32)
        self._check(self.lib.ng_step_batch(self.handle, tokens, B, state, self.state_size, nxt,
                                           logits, hidden, act))
        return logits, nxt, act, hidden

    def advance_batch(self, inputs, state, idle=False):
        inputs = np.ascontiguousarray(inputs, dtype=np.float32)
        state = np.ascontiguousarray(state, dtype=np.float32)
        B = inputs.shape[0]
        nxt = np.empty_like(state)
        hidden = np.empty((B, self.config.width), np.float32)
        act = np.empty(B, np.float32)
        self._check(self.lib.ng_advance_batch(self.handle, inputs, B, state, self.state_size,
                                              int(idle), nxt, hidden, act))
        return hidden, nxt, act


class NativeLanguageModel:
    """B200 counterpart of ``NativeLanguageModel`` (neurogen/language/native.py:55-162).

    State is the reference model's tuple layout: per region (voltage, trace, adaptation,
    last_spikes [B, c, 64], memory [B, w], counts [B, c, 64]), CPU float32, caller-owned and
    never mutated.  ``step`` returns (logits, state, activity, hidden) and ``advance`` returns
    (hidden, state, activity), as the reference does.
    """

    def __init__(self, config, weights, model=None, state_dict=None):
        self.config = config
        self.engine = NativeEngine(config, weights)
        self.native_backend = self.engine.backend
        self.model = model
        self._state_dict = state_dict  # checkpoint tensors for the audio projection and head (listen)
        self._versions = self._param_versions()

    @classmethod
    def from_model(cls, model, backend='native-cuda'):
        if backend not in NATIVE_DEVICES:
            raise ValueError(f'Unknown native device: {backend}')
        model.eval()
        check_architecture(model.config, model.state_dict())
        return cls(model.config, packed_weights(model), model)

    @classmethod
    def from_checkpoint(cls, path, backend='native-cuda'):
        if backend not in NATIVE_DEVICES:
            raise ValueError(f'Unknown native device: {backend}')
        config, weights, payload = load_checkpoint(path)
        return cls(config, weights, state_dict=payload['model'])

    def _param_versions(self):
        if self.model is None:
            return None
        return tuple(p._version for p in list(self.model.parameters()) + list(self.model.buffers()))

    def train(self, mode=True):
        if mode:
            raise ValueError('Native execution is inference-only. Train with PyTorch cpu/cuda/rocm, '
                             'then reload the checkpoint.')
        return self

    def eval(self):
        return self

    def initial(self, batch):
        c = self.config
        shape = (batch, c.columns, 64)
        region = lambda: tuple(torch.zeros(shape) for _ in range(4)) + (
            torch.zeros((batch, c.width)), torch.zeros(shape))
        return tuple(region() for _ in range(c.regions))

    def _shapes(self, batch):
        c = self.config
        return [(batch, c.columns, 64)] * 4 + [(batch, c.width), (batch, c.columns, 64)]

    def pack_state(self, state, batch):
        c = self.config
        if len(state) != c.regions or any(len(r) != 6 for r in state):
            raise ValueError('Invalid native region state')
        for region in state:
            for tensor, shape in zip(region, self._shapes(batch)):
                if tuple(tensor.shape) != shape or tensor.device.type != 'cpu' or tensor.dtype != torch.float32:
                    raise ValueError('Invalid native state shape/device/dtype')
        return np.ascontiguousarray(
            torch.cat([t.detach().reshape(batch, -1) for r in state for t in r], 1).numpy())

    def unpack_state(self, packed):
        batch = packed.shape[0]
        result, offset = [], 0
        for _ in range(self.config.regions):
            fields = []
            for shape in self._shapes(batch):
                size = int(np.prod(shape[1:]))
                fields.append(torch.from_numpy(packed[:, offset:offset + size].copy()).reshape(shape))
                offset += size
            result.append(tuple(fields))
        return tuple(result)

    def _call(self, inputs, state, idle, tokens):
        if self.model is not None and self._param_versions() != self._versions:
            raise ValueError('Native weights changed; reload using load_state_dict before inference')
        batch = len(inputs)
        if batch < 1:
            raise ValueError('Need at least one batch item')
        if state is None:
            state = self.initial(batch)
        packed = self.pack_state(state, batch)
        if tokens:
            logits, nxt, act, hidden = self.engine.step_batch(inputs.numpy().astype(np.int32), packed)
        else:
            x = np.ascontiguousarray(inputs.detach().cpu().float().numpy())
            hidden, nxt, act = self.engine.advance_batch(x, packed, idle)
            logits = np.zeros((batch, VOCAB), np.float32)
        return (torch.from_numpy(logits), self.unpack_state(nxt), torch.from_numpy(act).mean(),
                torch.from_numpy(hidden))

    def step(self, tokens, state=None):
        if tokens.ndim != 1 or tokens.dtype != torch.long or bool(((tokens < 0) | (tokens >= VOCAB)).any()):
            raise ValueError('Native tokens must be int64 [batch] in 0..263')
        return self._call(tokens, state, False, True)

    def advance(self, inputs, state=None, idle=False):
        if inputs.ndim != 2 or inputs.shape[1] != self.config.width:
            raise ValueError('Native inputs must have shape [batch, width]')
        _, state, activity, hidden = self._call(inputs, state, idle, False)
        return hidden, state, activity

    def __call__(self, tokens, state=None):
        """Token sequence [batch, time] (reference LanguageModel.forward, model.py:139-150)."""
        if tokens.ndim != 2 or tokens.dtype != torch.long:
            raise ValueError('tokens must be int64 [batch, time]')
        outputs, hidden, activity = [], [], []
        for token in tokens.unbind(1):
            logits, state, spikes, h = self.step(token, state)
            outputs.append(logits)
            hidden.append(h)
            activity.append(spikes)
        if not outputs:
            raise ValueError('Need at least one input token')
        return torch.stack(outputs, 1), state, torch.stack(activity).mean(), torch.stack(hidden, 1)

    forward = __call__

    def _audio_and_head(self):
        if self.model is not None:
            return self.model.audio_input, self.model.head
        sd = self._state_dict
        if sd is None or 'audio_input.weight' not in sd:
            raise ValueError('listen needs the audio projection: build from a model or a checkpoint')
        c = self.config
        audio, head = torch.nn.Linear(c.mel_bins, c.width), torch.nn.Linear(c.width, VOCAB)
        with torch.no_grad():
            audio.weight.copy_(sd['audio_input.weight'])
            audio.bias.copy_(sd['audio_input.bias'])
            head.weight.copy_(sd['head.weight'])
            head.bias.copy_(sd['head.bias'])
        return audio.eval(), head.eval()

    def listen(self, features, state=None):
        """Mel frames [batch, time, mel_bins]: each frame through the audio projection and one
        ``advance`` (non-idle), logits from the head (reference LanguageModel.listen,
        model.py:152-158).  The two projections run in torch, as in the reference; the advance runs
        on the GPU engine."""
        if features.ndim != 3 or features.shape[2] != self.config.mel_bins:
            raise ValueError('Native listen features must have shape [batch, time, mel_bins]')
        audio, head = self._audio_and_head()
        logits, activity = [], []
        with torch.no_grad():
            for frame in features.unbind(1):
                h, state, spikes = self.advance(audio(frame.float()), state)
                logits.append(head(h))
                activity.append(spikes)
        if not logits:
            raise ValueError('Need at least one feature frame')
        return torch.stack(logits, 1), state, torch.stack(activity).mean()


def config_dict(config):
    return asdict(config)


# ---------------------------------------------------------------------------
# Session files and device-resident session pools.
# ---------------------------------------------------------------------------
SESSION_FORMAT = 'neurogen-session-v2'


def session_payload(state, logits, checkpoint_id, extras=None):
    """One session in the layout ``Session.save`` writes (neurogen/language/runtime.py:95-100).

    ``state`` is the model state of one session in the reference tuple layout (batch 1) and
    ``logits`` its last logits [264].  The text decoder, sampling generator and audio front-end
    fields take the values a fresh ``Session`` holds (runtime.py:22-37) unless ``extras`` gives
    them, so the reference runtime can load the file and continue the conversation.
    """
    payload = {'format': SESSION_FORMAT, 'checkpoint_id': checkpoint_id, 'state': state,
               'logits': torch.as_tensor(logits, dtype=torch.float32),
               'random': torch.Generator().manual_seed(1).get_state(), 'decoder': ([], 0),
               'audio_state': None, 'previous_ctc': PAD, 'audio_decoder': ([], 0),
               'audio_buffer': torch.empty(0), 'audio_emitted': False}
    payload.update(extras or {})
    return payload


def save_session(path, payload):
    """Atomic write (temporary file, then rename), as training.py:31-36 does."""
    from pathlib import Path
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    temporary = path.with_name(path.name + '.tmp')
    torch.save(payload, temporary)
    temporary.replace(path)


def load_session(path, checkpoint_id):
    """A session file of this checkpoint; the reference's check and message (runtime.py:103-106)."""
    payload = torch.load(path, map_location='cpu', weights_only=True)
    if payload.get('format') != SESSION_FORMAT or payload.get('checkpoint_id') != checkpoint_id:
        raise ValueError('Session belongs to a different model checkpoint')
    return payload


class SessionPool:
    """``sessions`` independent streaming sessions whose states stay on the GPU (``ng_pool_*``).

    ``step(tokens)`` feeds one token to every session (one CUDA-graph replay) and returns the
    logits [sessions, 264].  ``save``/``load`` move one session to or from a
    ``neurogen-session-v2`` file in the reference's layout, so a conversation can move between
    this pool and the reference runtime.
    """

    def __init__(self, model, sessions):
        self.model = model
        self.lib = model.engine.lib
        self.sessions = int(sessions)
        self.h = self.lib.ng_pool_create(model.engine.handle, self.sessions)
        if not self.h:
            raise ValueError(self.lib.ng_error().decode())
        self.logits = np.zeros((self.sessions, VOCAB), np.float32)

    def close(self):
        if getattr(self, 'h', None):
            self.lib.ng_pool_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def _check(self, code):
        if code:
            raise ValueError(self.lib.ng_error().decode())

    def step(self, tokens):
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        if tokens.shape != (self.sessions,):
            raise ValueError(f'Need one token per session ({self.sessions})')
        self._check(self.lib.ng_pool_step(self.h, tokens, self.logits.ctypes.data, None, None))
        return self.logits.copy()

    def states(self):
        """Packed states [sessions, state_size] in the reference order."""
        out = np.empty((self.sessions, self.model.engine.state_size), np.float32)
        self._check(self.lib.ng_pool_store(self.h, out))
        return out

    def set_states(self, packed):
        packed = np.ascontiguousarray(packed, dtype=np.float32)
        if packed.shape != (self.sessions, self.model.engine.state_size):
            raise ValueError('Invalid native state size')
        self._check(self.lib.ng_pool_load(self.h, packed))

    def save(self, path, index, checkpoint_id, extras=None):
        """Session ``index`` to a session file."""
        state = self.model.unpack_state(self.states()[index:index + 1])
        save_session(path, session_payload(state, self.logits[index], checkpoint_id, extras))

    def load(self, path, index, checkpoint_id):
        """A session file into session ``index``; returns the payload (decoder, audio fields)."""
        payload = load_session(path, checkpoint_id)
        packed = self.states()
        packed[index] = self.model.pack_state(payload['state'], 1)[0]
        self.set_states(packed)
        self.logits[index] = np.asarray(payload['logits'], np.float32).reshape(VOCAB)
        return payload
