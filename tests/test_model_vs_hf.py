"""The whole-decoder oracle against a third implementation: Hugging Face
transformers' Qwen2MoeForCausalLM, loaded with the DEQUANTIZED int8 weights
of the same seeded decoders, so both compute one fp32 model and a
difference can only come from the implementation. This is the check of
the reference's tests/test_runtime_vs_hf_transformers.py (prefill logits at
rtol = atol = 1e-4, same argmax; KV-cache decoding against transformers'
full recompute), run here on the oracle that the device model is tested
against: grouped KV heads, RoPE, softmax-then-top-k routing with and
without renormalisation, the gated shared expert. CPU only."""

from __future__ import annotations

import numpy as np
import pytest
from golden.make_golden import MODEL_CASES

from expertrelay_b200 import synth
from oracle.model_oracle import ModelOracle

torch = pytest.importorskip("torch")
transformers = pytest.importorskip("transformers")


def _deq(v) -> np.ndarray:
    if isinstance(v, tuple):  # int8 (q, scales) per output row
        q, s = v
        return q.astype(np.float32) * s[:, None]
    return np.asarray(v, dtype=np.float32)


def _hf_model(host):
    c = host.config
    hf_cfg = transformers.Qwen2MoeConfig(
        **{k: c[k] for k in ("vocab_size", "hidden_size", "num_hidden_layers", "num_attention_heads",
                             "num_key_value_heads", "num_experts", "num_experts_per_tok", "moe_intermediate_size",
                             "shared_expert_intermediate_size", "norm_topk_prob", "rms_norm_eps", "rope_theta")},
        intermediate_size=c["moe_intermediate_size"], max_position_embeddings=64, decoder_sparse_step=1,
        mlp_only_layers=[], use_sliding_window=False, tie_word_embeddings=False)
    hf_cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    hf = transformers.Qwen2MoeForCausalLM(hf_cfg).eval().float()
    tensors = host.tensors()
    state = {}
    for name, ref in hf.state_dict().items():
        if ".mlp.experts." in name:
            layer = int(name.split(".")[2])
            experts = host.blocks[layer].experts
            if name.endswith("gate_up_proj"):  # [E, 2I, H]: gate rows, then up rows
                w = np.stack([np.concatenate([_deq(e["gate_proj"]), _deq(e["up_proj"])]) for e in experts])
            else:  # down_proj [E, H, I]
                w = np.stack([_deq(e["down_proj"]) for e in experts])
        else:
            w = _deq(tensors[name])
        state[name] = torch.from_numpy(np.ascontiguousarray(w).reshape(ref.shape))
    hf.load_state_dict(state, strict=True)
    return hf


def _hf_logits(hf, tokens) -> np.ndarray:
    with torch.no_grad():
        return hf(torch.tensor([list(tokens)])).logits[0].numpy()


@pytest.mark.parametrize("case", range(len(MODEL_CASES)))
def test_oracle_prefill_and_decode_match_transformers(case):
    cfg, seed = MODEL_CASES[case]
    host = synth.make_model(cfg, seed=seed)
    hf = _hf_model(host)
    oracle = ModelOracle(host)
    tokens = [int(t) for t in np.random.default_rng(seed + 100).integers(0, cfg["vocab_size"], 10)]

    kv = oracle.new_cache(32)
    logits = oracle.forward(tokens, kv, all_logits=True)
    expected = _hf_logits(hf, tokens)
    np.testing.assert_allclose(logits, expected, rtol=1e-4, atol=1e-4)
    np.testing.assert_array_equal(logits.argmax(-1), expected.argmax(-1))

    # greedy decoding through the KV cache against transformers' full recompute
    kv = oracle.new_cache(32)
    seq = tokens[:4]
    logits = oracle.forward(seq, kv)
    for _ in range(5):
        expected_last = _hf_logits(hf, seq)[-1]
        np.testing.assert_allclose(logits, expected_last, rtol=1e-4, atol=1e-4)
        nxt = int(np.argmax(logits))
        assert nxt == int(np.argmax(expected_last))
        seq = seq + [nxt]
        logits = oracle.forward([nxt], kv)
