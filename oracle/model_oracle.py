"""CPU oracle for the whole decoder. TEST INFRASTRUCTURE ONLY.

Restates ExpertRelay's QwenMoe forward (src/expertrelay/runtime/qwen_moe.py)
in numpy: rms_norm (:121-123), the RoPE tables and rotation (:126-138,
255-256), attention with the KV cache and the causal mask (:250-276,
backends.py:90-95), the MoE block (moe_oracle.moe_block, :293-359), the
residuals, the final norm and lm_head (:376-432), over a synth.HostModel.
It is pinned against the reference's own forward pass on the same seeded
models (tests/golden/model.npz, made by tests/golden/make_golden.py).
"""

from __future__ import annotations

import numpy as np

from oracle import moe_oracle as O
from oracle.blocks import oracle_weights


def rms_norm(x, w, eps):
    variance = np.mean(x * x, axis=-1, keepdims=True)  # :121-123
    return w * (x * (1.0 / np.sqrt(variance + eps)))


def rope_tables(positions, head_dim, theta):
    inv_freq = (1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.int64).astype(np.float32) / head_dim))).astype(
        np.float32)  # :126-133
    freqs = positions.astype(np.float32)[:, None] * inv_freq[None, :]
    emb = np.concatenate([freqs, freqs], axis=-1)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


def _rotate_half(x):
    half = x.shape[-1] // 2
    return np.concatenate([-x[..., half:], x[..., :half]], axis=-1)


def attention(q, keys, values, allowed):
    """backends.py:90-95: softmax(q k^T / sqrt(d), masked) v, per head."""
    d = q.shape[-1]
    s = np.einsum("nhd,mhd->hnm", q, keys) * np.float32(1.0 / np.sqrt(d))
    s = np.where(allowed[None], s, -np.inf).astype(np.float32)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(axis=-1, keepdims=True)
    return np.einsum("hnm,mhd->nhd", p, values).astype(np.float32)


class ModelOracle:
    def __init__(self, host):
        c = host.config
        self.host, self.c = host, c
        self.H, self.L = c["hidden_size"], c["num_hidden_layers"]
        self.heads, self.kvh = c["num_attention_heads"], c["num_key_value_heads"]
        self.d = self.H // self.heads
        self.eps, self.theta = c["rms_norm_eps"], c["rope_theta"]
        self.blocks = [oracle_weights(b) for b in host.blocks]
        for bw in self.blocks:
            bw.norm_topk_prob = bool(c["norm_topk_prob"])

    def new_cache(self, max_seq):
        shape = (self.L, max_seq, self.kvh, self.d)
        return {"k": np.zeros(shape, np.float32), "v": np.zeros(shape, np.float32), "length": 0}

    def forward(self, ids, kv, all_logits=False):
        host, d = self.host, self.d
        ids = np.asarray(ids, dtype=np.int64)
        n = len(ids)
        eq, es = host.embed
        x = eq[ids].astype(np.float32) * es[ids][:, None]  # Int8Matrix.dequantized_rows
        start = kv["length"]
        end = start + n
        cos, sin = rope_tables(start + np.arange(n), d, self.theta)
        for i, lay in enumerate(host.layers):
            h = rms_norm(x, lay.input_norm, self.eps)
            q = O.int8_linear(h, *lay.proj["q_proj"], lay.bias["q_proj"]).reshape(n, self.heads, d)
            k = O.int8_linear(h, *lay.proj["k_proj"], lay.bias["k_proj"]).reshape(n, self.kvh, d)
            v = O.int8_linear(h, *lay.proj["v_proj"], lay.bias["v_proj"]).reshape(n, self.kvh, d)
            q = q * cos[:, None, :] + _rotate_half(q) * sin[:, None, :]
            k = k * cos[:, None, :] + _rotate_half(k) * sin[:, None, :]
            kv["k"][i, start:end], kv["v"][i, start:end] = k, v
            keys, values = kv["k"][i, :end], kv["v"][i, :end]
            if self.kvh != self.heads:
                rep = self.heads // self.kvh
                keys, values = np.repeat(keys, rep, axis=1), np.repeat(values, rep, axis=1)
            allowed = np.arange(end)[None, :] <= (start + np.arange(n))[:, None]
            a = attention(q, keys, values, allowed).reshape(n, self.H)
            x = x + O.int8_linear(a, *lay.proj["o_proj"])
            h = rms_norm(x, lay.post_norm, self.eps)
            x = x + O.moe_block(h, self.blocks[i]).y
        kv["length"] = end
        final = rms_norm(x if all_logits else x[-1:], host.final_norm, self.eps)
        logits = O.int8_linear(final, *host.lm_head)
        return logits if all_logits else logits[0]
