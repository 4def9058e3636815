"""ng_step_static: the token step that allocates no device memory of its own.

It is meant for callers that must not have a step allocate (a fixed device-memory budget, or
a streaming loop where a cudaMalloc could block on the driver's allocation lock and
synchronise the device).  Its working memory is a fixed 1 MiB array compiled into the library
and shared by every call, so these tests check that two calls in a row -- each starting from
whatever the previous call left in the array, and across two different models -- give the
same results as the ordinary ng_step, and that a model too large for the array is refused
with a clear error.  This file is collected last on purpose.
"""
import numpy as np
import pytest

from neurogen_b200.language import LanguageConfig, NativeEngine, init_packed_weights

pytestmark = pytest.mark.gpu

STATE_RTOL, STATE_ATOL = 1e-5, 1e-6   # same bars as tests/test_lang_gpu.py
LOGIT_RTOL, LOGIT_ATOL = 1e-4, 1e-6


def outputs(eng, cfg):
    return (np.empty(eng.state_size, np.float32), np.empty(264, np.float32),
            np.empty(cfg.width, np.float32), np.empty(1, np.float32))


def step(eng, cfg, fn, token, state):
    nxt, logits, hidden, act = outputs(eng, cfg)
    code = fn(eng.handle, token, state, state.size, nxt, logits, hidden, act)
    assert code == 0, eng.lib.ng_error().decode()
    return nxt, logits, hidden, act


def close(a, b):
    (sa, la, ha, aa), (sb, lb, hb, ab) = a, b
    np.testing.assert_allclose(sa, sb, rtol=STATE_RTOL, atol=STATE_ATOL)
    np.testing.assert_allclose(la, lb, rtol=LOGIT_RTOL, atol=LOGIT_ATOL)
    np.testing.assert_allclose(ha, hb, rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(aa, ab, atol=1e-7)


@pytest.mark.parametrize('cfg,seed', [
    (LanguageConfig(), 0),                                                   # BC-250 profile
    (LanguageConfig(columns=3, width=17, regions=2, ticks=3, idle_steps=1), 7),
])
def test_static_step_matches_ng_step_on_two_calls_in_a_row(cfg, seed):
    eng = NativeEngine(cfg, init_packed_weights(cfg, seed=seed))
    lib = eng.lib
    s_ref = np.zeros(eng.state_size, np.float32)
    s_new = s_ref.copy()
    for token in (257, 104):
        ref = step(eng, cfg, lib.ng_step, token, s_ref)
        new = step(eng, cfg, lib.ng_step_static, token, s_new)
        close(new, ref)
        s_ref, s_new = ref[0], new[0]


def test_warm_static_step_allocates_no_device_memory():
    """After a first call (which looks the array up and loads the kernels), further calls leave
    the device's free memory exactly unchanged: nothing is allocated per call."""
    import torch
    cfg = LanguageConfig()
    eng = NativeEngine(cfg, init_packed_weights(cfg, seed=0))
    lib = eng.lib
    s = np.zeros(eng.state_size, np.float32)
    s = step(eng, cfg, lib.ng_step_static, 257, s)[0]
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for token in (104, 101, 108, 108, 111):
        s = step(eng, cfg, lib.ng_step_static, token, s)[0]
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)


def test_static_step_rejects_models_beyond_its_buffer():
    # 1,024 columns of one region: a 327,696-float state, more than the 262,144-float buffer.
    cfg = LanguageConfig(columns=1024, width=16, regions=1, ticks=1, idle_steps=0)
    eng = NativeEngine(cfg, init_packed_weights(cfg, seed=1))
    state = np.zeros(eng.state_size, np.float32)
    nxt, logits, hidden, act = outputs(eng, cfg)
    assert eng.lib.ng_step_static(eng.handle, 1, state, state.size, nxt, logits, hidden, act) == -1
    msg = eng.lib.ng_error().decode()
    assert 'ng_step_static' in msg and '1 MiB' in msg and 'use ng_step' in msg
