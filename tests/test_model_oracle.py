"""The whole-decoder oracle (oracle/model_oracle.py) against the reference's
own forward pass on the same seeded models (tests/golden/model.npz)."""

from __future__ import annotations

import numpy as np
import pytest
from conftest import golden
from golden.make_golden import MODEL_CASES, MODEL_NEW, MODEL_PROMPT

from expertrelay_b200 import synth
from oracle.moe_oracle import rel_l2
from oracle.model_oracle import ModelOracle


@pytest.mark.parametrize("case", range(len(MODEL_CASES)))
def test_model_oracle_matches_reference(case):
    cfg, seed = MODEL_CASES[case]
    g = golden("model")
    host = synth.make_model(cfg, seed=seed)
    o = ModelOracle(host)
    kv = o.new_cache(MODEL_PROMPT + MODEL_NEW)
    logits = o.forward(g[f"prompt{case}"], kv, all_logits=True)
    assert rel_l2(logits, g[f"prompt_logits{case}"]) < 1e-5
    tok = int(np.argmax(logits[-1]))
    for step in range(MODEL_NEW):
        assert tok == g[f"tokens{case}"][step]
        lg = o.forward([tok], kv)
        assert rel_l2(lg, g[f"step_logits{case}"][step]) < 1e-5
        tok = int(np.argmax(lg))
