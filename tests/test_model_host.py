"""Host side of the whole-decoder path, on the CPU: the config checks of the
reference's ModelConfig.from_hf (runtime/qwen_moe.py:70-87), the seeded
model generator's determinism and checkpoint names, and the whole-model
oracle on an input beyond the fixture (prompt, then decode calls, equal to
all-position logits of one call)."""

from __future__ import annotations

import numpy as np
import pytest
from golden.make_golden import TINY_MODEL

from expertrelay_b200 import synth
from expertrelay_b200.model import ModelConfig
from oracle.model_oracle import ModelOracle


def test_config_from_hf():
    c = ModelConfig.from_hf(synth.QWEN_MODEL)
    assert (c.hidden_size, c.num_layers, c.num_heads, c.head_dim, c.num_experts, c.top_k) == (2048, 24, 16, 128, 60, 4)
    assert c.rope_theta == 1e6 and c.rms_norm_eps == 1e-6 and not c.norm_topk_prob
    with pytest.raises(NotImplementedError, match="sliding-window"):
        ModelConfig.from_hf({**synth.QWEN_MODEL, "use_sliding_window": True})
    with pytest.raises(NotImplementedError, match="dense"):
        ModelConfig.from_hf({**synth.QWEN_MODEL, "decoder_sparse_step": 2})


def test_make_model_is_seeded_and_named_like_the_checkpoint():
    a = synth.make_model(TINY_MODEL, seed=5)
    b = synth.make_model(TINY_MODEL, seed=5)
    ta, tb = a.tensors(), b.tensors()
    assert ta.keys() == tb.keys()
    for k in ta:
        va, vb = ta[k], tb[k]
        if isinstance(va, tuple):
            assert all(np.array_equal(x, y) for x, y in zip(va, vb)), k
        else:
            assert np.array_equal(va, vb), k
    names = set(ta)
    assert {"model.embed_tokens.weight", "lm_head.weight", "model.norm.weight",
            "model.layers.0.self_attn.q_proj.bias", "model.layers.2.mlp.shared_expert_gate.weight"} <= names
    assert not np.array_equal(ta["lm_head.weight"][0], synth.make_model(TINY_MODEL, seed=6).tensors()["lm_head.weight"][0])


def test_oracle_decode_calls_equal_one_call():
    """Feeding tokens one call at a time through the KV cache gives the logits
    the all-positions call gives (the cache carries the keys and values)."""
    host = synth.make_model(TINY_MODEL, seed=9)
    o = ModelOracle(host)
    ids = np.random.default_rng(3).integers(0, TINY_MODEL["vocab_size"], 6)
    kv = o.new_cache(6)
    full = o.forward(ids, kv, all_logits=True)
    kv2 = o.new_cache(6)
    o.forward(ids[:3], kv2)
    steps = [o.forward([int(t)], kv2) for t in ids[3:]]
    for i, lg in enumerate(steps):
        np.testing.assert_allclose(lg, full[3 + i], rtol=2e-5, atol=2e-5)


def test_read_budget_and_window_follow_the_runtime():
    """The adaptive prefetch cap (runtime/qwen_moe.py:361-374): top_k until a
    window is measured, then window / copy time rounded, at least one; the
    window is a running average with weight 0.5 on the newest call."""
    from expertrelay_b200.paged import WINDOW_EMA, read_budget, update_window

    assert WINDOW_EMA == 0.5
    assert read_budget(float("nan"), 1.6e-4, 4) == 4
    assert read_budget(5e-4, 1.6e-4, 4) == 3  # 3.125 copies fit
    assert read_budget(3.0, 2.0, 4) == 2 and read_budget(5.0, 2.0, 4) == 2  # Python's round: halves to even
    assert read_budget(1e-6, 1.6e-4, 4) == 1  # always at least one
    assert read_budget(1.0, 1.6e-4, 4) == 6250  # the budget is not capped at top_k
    w = float("nan")
    for new, want in ((2e-4, 2e-4), (4e-4, 3e-4), (4e-4, 3.5e-4)):
        w = update_window(w, new)
        assert w == pytest.approx(want)
