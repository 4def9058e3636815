"""Session files in the reference's ``neurogen-session-v2`` layout (CPU; no GPU needed).

tests/golden/session_ref_small.pt was written by the reference runtime's own Session.save
(tests/golden/make_session_golden.py).  Our loader must read it, and the payloads our pools write
must carry the same fields with the same types, so sessions move both ways.
"""
import numpy as np
import pytest
import torch

from neurogen_b200.language import SESSION_FORMAT, load_session, save_session, session_payload

GOLDEN = __import__('pathlib').Path(__file__).resolve().parent / 'golden' / 'session_ref_small.pt'


def test_reference_session_file_loads():
    payload = load_session(GOLDEN, 'golden-checkpoint')
    assert payload['format'] == SESSION_FORMAT
    state = payload['state']
    assert len(state) == 2 and all(len(r) == 6 for r in state)
    assert tuple(state[0][0].shape) == (1, 4, 64) and tuple(state[0][4].shape) == (1, 32)
    assert tuple(payload['logits'].shape) == (264,)
    with pytest.raises(ValueError, match='different model checkpoint'):
        load_session(GOLDEN, 'another-checkpoint')


def test_our_payload_has_the_reference_fields(tmp_path):
    ref = torch.load(GOLDEN, map_location='cpu', weights_only=True)
    state = tuple(tuple(t.clone() for t in r) for r in ref['state'])
    ours = session_payload(state, ref['logits'].numpy(), 'golden-checkpoint')
    assert set(ours) == set(ref)
    for key in ref:
        assert type(ours[key]) is type(ref[key]), key
    assert ours['random'].dtype == ref['random'].dtype and ours['random'].shape == ref['random'].shape
    path = tmp_path / 'x.pt'
    save_session(path, ours)
    back = load_session(path, 'golden-checkpoint')
    for r1, r2 in zip(back['state'], ref['state']):
        for a, b in zip(r1, r2):
            assert torch.equal(a, b)
    assert np.array_equal(back['logits'].numpy(), ref['logits'].numpy())
