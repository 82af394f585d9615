"""GPU: the whole Qwen2-MoE decoder (QwenMoeModel) against the reference's
forward pass on seeded small models (tests/golden/model.npz, GQA and
renormalised top-k in the second case): prompt logits at every position,
greedy tokens and each decode call's logits; an expert cache far smaller than
the experts, with and without the Fate prefetch, must give the same logits
bit for bit; the trace of a generation records the experts the model used."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import golden
from golden.make_golden import MODEL_CASES, MODEL_NEW, MODEL_PROMPT

from expertrelay_b200 import _lib, synth
from expertrelay_b200.model import QwenMoeModel
from expertrelay_b200.trace import ExpertTraceWriter, read_trace
from oracle.moe_oracle import rel_l2

pytestmark = pytest.mark.gpu

# the exact-fp32 paths follow the reference's float32 arithmetic to rounding;
# the tensor-core path carries activations as two int8 slices
TOL = {_lib.PATH_GEMM: 1e-4, _lib.PATH_GEMV: 1e-4, _lib.PATH_TC: 2e-3}


@pytest.mark.parametrize("case", range(len(MODEL_CASES)))
@pytest.mark.parametrize("path", [_lib.PATH_GEMM, _lib.PATH_TC])
def test_model_matches_reference(case, path, cuda):
    cfg, seed = MODEL_CASES[case]
    g = golden("model")
    model = QwenMoeModel(synth.make_model(cfg, seed=seed), device=cuda, path=path)
    kv = model.new_cache(MODEL_PROMPT + MODEL_NEW)
    logits = model.forward(g[f"prompt{case}"], kv, all_logits=True).cpu().numpy()
    assert rel_l2(logits, g[f"prompt_logits{case}"]) < TOL[path]
    tok = int(np.argmax(logits[-1]))
    for step in range(MODEL_NEW):
        assert tok == g[f"tokens{case}"][step]
        lg = model.forward([tok], kv).cpu().numpy()
        assert rel_l2(lg, g[f"step_logits{case}"][step]) < TOL[path]
        tok = int(np.argmax(lg))
    model.close()


@pytest.mark.parametrize("prefetch", [False, True, "adaptive"])
def test_small_cache_changes_nothing(prefetch, cuda):
    cfg, seed = MODEL_CASES[0]
    host = synth.make_model(cfg, seed=seed)
    g = golden("model")
    outs = []
    for slots, pf in ((None, False), (18, prefetch)):  # 18 slots for 48 records: layers evict each other
        model = QwenMoeModel(host, device=cuda, cache_records=slots, prefetch=bool(pf),
                             prefetch_adaptive=pf == "adaptive")
        tokens, _, _ = model.generate(g["prompt0"], MODEL_NEW)
        if pf == "adaptive":  # the decode calls measured every layer's window and one copy's time
            st = model.stack
            assert np.isfinite(st.window[:-1]).all() and (st.window[:-1] > 0).all()
            assert st.read_seconds is not None and 0 < st.read_seconds < 0.1
        kv = model.new_cache(MODEL_PROMPT + 1)
        outs.append((tokens, model.forward(g["prompt0"], kv, all_logits=True).cpu()))
        model.close()
    assert outs[0][0] == outs[1][0] == list(g["tokens0"])
    assert torch.equal(outs[0][1], outs[1][1])


def test_generation_trace(cuda, tmp_path):
    cfg, seed = MODEL_CASES[0]
    g = golden("model")
    model = QwenMoeModel(synth.make_model(cfg, seed=seed), device=cuda, cache_records=24, prefetch=True)
    path = tmp_path / "gen.ert"
    w = ExpertTraceWriter(path, num_layers=cfg["num_hidden_layers"], num_experts=cfg["num_experts"],
                          top_k=cfg["num_experts_per_tok"], metadata={"prompt_id": "p0"}, device=cuda)
    tokens, _, _ = model.generate(g["prompt0"], MODEL_NEW, expert_trace=w)
    model.close()
    header, rec = read_trace(path)
    L = cfg["num_hidden_layers"]
    assert len(rec) == (MODEL_PROMPT + MODEL_NEW - 1) * L  # the last token is never fed back in
    assert list(rec["token"][rec["layer"] == 0]) == list(g["prompt0"]) + tokens[:-1]
    assert np.all(rec["weights"][:, 0] >= rec["weights"][:, 1])
    for layer in range(L):
        rows = rec[rec["layer"] == layer]
        np.testing.assert_array_equal(rows["prev_token_experts"][1:], rows["experts"][:-1])
