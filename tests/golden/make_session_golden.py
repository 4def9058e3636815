"""Writes tests/golden/session_ref_small.pt: a ``neurogen-session-v2`` file saved by the reference
runtime's own ``Session.save`` (neurogen/language/runtime.py:95-100) after one user turn, for a small
seeded model.  Run where the reference checkout is importable (its path as the first argument, or in NEUROGEN_REFERENCE):

    python tests/golden/make_session_golden.py [/path/to/reference]
"""
import os
import sys
from pathlib import Path

import torch

REFERENCE = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ['NEUROGEN_REFERENCE'])
sys.path.insert(0, str(REFERENCE))

from neurogen.language.config import LanguageConfig  # noqa: E402
from neurogen.language.model import LanguageModel  # noqa: E402
from neurogen.language.runtime import Session  # noqa: E402

OUT = Path(__file__).resolve().parent / 'session_ref_small.pt'

torch.manual_seed(0)
model = LanguageModel(LanguageConfig(columns=4, width=32, regions=2, ticks=2, idle_steps=1))
session = Session(model)
session.hear_text('hi')
session.save(OUT, 'golden-checkpoint')
print('wrote', OUT, OUT.stat().st_size, 'bytes')
