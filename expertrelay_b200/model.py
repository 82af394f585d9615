"""QwenMoeModel: the whole Qwen1.5-MoE decoder on one B200 (runtime/
qwen_moe.py:233-432), its routed experts paged through the HBM expert cache.

Per layer, as the reference's forward: input RMSNorm, attention (int8 q/k/v
with biases, RoPE, a KV cache, causal softmax attention, int8 o), the
residual, post-attention RMSNorm, the MoE block, the residual; then the
final norm and the int8 lm_head. Everything stays on the device: the
residual adds are fused into the next norm (er_rms_norm), RoPE writes the
rotated keys and the values straight into the cache (er_rope_kv), the
embedding rows are dequantized on the device (er_embed_int8), the
projections stream their int8 weights (er_int8_linear), attention is
er_attention, and the MoE block is PagedMoeStack.moe: the router and top-k
on the device, the selected experts made resident in the cache (copies from
pinned host records on the cache's copy stream), the Fate prefetch of the
next layer's guesses when a policy is given, and the block on the cached
records. Only the expert ids cross to the host each layer, to drive the
cache, as in the reference.
"""

from __future__ import annotations

import time
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .cache import HbmExpertCache, HostRecords
from .paged import PagedMoeStack
from .prefetch import PrefetchPolicy
from .trace import PHASE_DECODE, PHASE_PREFILL


@dataclass(frozen=True)
class ModelConfig:
    """The config.json fields the forward pass uses (runtime/qwen_moe.py:53-87)."""

    vocab_size: int
    hidden_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    num_experts: int
    top_k: int
    norm_topk_prob: bool
    rms_norm_eps: float
    rope_theta: float
    moe_intermediate_size: int
    shared_expert_intermediate_size: int

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    @classmethod
    def from_hf(cls, c: dict) -> ModelConfig:
        if c.get("use_sliding_window"):
            raise NotImplementedError("sliding-window attention is not implemented")
        if c.get("mlp_only_layers") or c.get("decoder_sparse_step", 1) != 1:
            raise NotImplementedError("dense (non-MoE) decoder layers are not implemented")
        return cls(c["vocab_size"], c["hidden_size"], c["num_hidden_layers"], c["num_attention_heads"],
                   c["num_key_value_heads"], c["num_experts"], c["num_experts_per_tok"], bool(c["norm_topk_prob"]),
                   float(c["rms_norm_eps"]), float(c["rope_theta"]), c["moe_intermediate_size"],
                   c["shared_expert_intermediate_size"])


class KVCache:
    """Keys and values of every layer on the device: [layers, max_seq,
    kv_heads, head_dim] fp32 each (runtime/qwen_moe.py:90-106)."""

    def __init__(self, config: ModelConfig, max_seq: int, device):
        shape = (config.num_layers, max_seq, config.num_kv_heads, config.head_dim)
        self.k = torch.zeros(shape, dtype=torch.float32, device=device)
        self.v = torch.zeros(shape, dtype=torch.float32, device=device)
        self.length = 0
        self.max_seq = max_seq

    @property
    def nbytes(self) -> int:
        return 2 * self.k.numel() * 4


def _dev(a, dtype, device) -> torch.Tensor:
    return torch.as_tensor(np.ascontiguousarray(a)).to(device=device, dtype=dtype)


class QwenMoeModel:
    """host: an expertrelay_b200.synth.HostModel (or anything with its
    fields); records: the routed experts as [layers, experts, record_size]
    uint8 (pinned host memory; default: the host blocks' records);
    cache_records: HBM slots for routed records (default: all of them);
    prefetch: the Fate policy's prefetch of the next layer's experts;
    prefetch_adaptive: cap the prefetch's copies on one-token calls at what
    fits in each layer's measured window (runtime/generate.py:112)."""

    def __init__(self, host, *, records: torch.Tensor | None = None, cache_records: int | None = None,
                 prefetch: bool = False, prefetch_adaptive: bool = False, device="cuda",
                 path: int = _lib.PATH_AUTO):
        if not torch.cuda.is_available():
            raise RuntimeError("QwenMoeModel needs a CUDA device (the B200 path has no CPU fallback)")
        self.device = dev = torch.device(device)
        if dev.index is None:
            self.device = dev = torch.device("cuda", torch.cuda.current_device())
        self.c = c = ModelConfig.from_hf(host.config)
        self.path = path
        self.embed_q, self.embed_s = _dev(host.embed[0], torch.int8, dev), _dev(host.embed[1], torch.float32, dev)
        self.head_q, self.head_s = _dev(host.lm_head[0], torch.int8, dev), _dev(host.lm_head[1], torch.float32, dev)
        self.final_norm = _dev(host.final_norm, torch.float32, dev)
        self.layers = []
        for lay in host.layers:
            w = {"in_norm": _dev(lay.input_norm, torch.float32, dev), "post_norm": _dev(lay.post_norm, torch.float32, dev)}
            # q, k and v as one projection (rows stacked: one weight stream, one launch)
            qkv = ("q_proj", "k_proj", "v_proj")
            w["qkv"] = (_dev(np.concatenate([lay.proj[m][0] for m in qkv]), torch.int8, dev),
                        _dev(np.concatenate([lay.proj[m][1] for m in qkv]), torch.float32, dev))
            w["qkv_bias"] = _dev(np.concatenate([lay.bias[m] for m in qkv]), torch.float32, dev)
            w["o_proj"] = (_dev(lay.proj["o_proj"][0], torch.int8, dev), _dev(lay.proj["o_proj"][1], torch.float32, dev))
            self.layers.append(w)
        if records is None:
            records = HostRecords.from_blocks(host.blocks)
        else:
            records = HostRecords(records, host.blocks[0].layout, pin=True)
        self.records = records
        rs = records.layout.record_size
        slots = cache_records if cache_records is not None else records.layers * records.experts
        self.cache = HbmExpertCache(records, capacity_bytes=slots * rs, device=dev)
        policy = PrefetchPolicy(top_k=c.top_k) if prefetch else None
        self.stack = PagedMoeStack(host.blocks, self.cache, prefetcher=policy, norm_topk_prob=c.norm_topk_prob)
        self.stack.prefetch_adaptive = prefetch_adaptive
        self._bad = torch.zeros(1, dtype=torch.int32, device=dev)

    def close(self) -> None:
        self.cache.close()

    def new_cache(self, max_seq: int) -> KVCache:
        return KVCache(self.c, max_seq, self.device)

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def _linear(self, x: torch.Tensor, qs, bias: torch.Tensor | None = None) -> torch.Tensor:
        q, s = qs
        n, out_dim, in_dim = x.shape[0], q.shape[0], q.shape[1]
        y = torch.empty((n, out_dim), dtype=torch.float32, device=self.device)
        _lib.check(_lib.lib().er_int8_linear(x.data_ptr(), in_dim, q.data_ptr(), s.data_ptr(),
                                             None if bias is None else bias.data_ptr(), y.data_ptr(), n, out_dim,
                                             in_dim, self._stream()), "er_int8_linear")
        return y

    def _norm(self, x: torch.Tensor, w: torch.Tensor, add: torch.Tensor | None = None) -> torch.Tensor:
        """h = rms_norm(x (+ add)); with `add`, x itself becomes x + add."""
        n, H = x.shape
        h = torch.empty_like(x)
        _lib.check(_lib.lib().er_rms_norm(x.data_ptr(), None if add is None else add.data_ptr(), w.data_ptr(),
                                          self.c.rms_norm_eps, n, H, x.data_ptr(), h.data_ptr(), self._stream()),
                   "er_rms_norm")
        return h

    def _attention(self, layer: int, h: torch.Tensor, kv: KVCache, allowed: torch.Tensor) -> torch.Tensor:
        c, w = self.c, self.layers[layer]
        n, d = h.shape[0], c.head_dim
        qkv = self._linear(h, w["qkv"], w["qkv_bias"])
        q = torch.empty((n, c.num_heads * d), dtype=torch.float32, device=self.device)
        start, end = kv.length, kv.length + n
        _lib.check(_lib.lib().er_rope_kv(qkv.data_ptr(), qkv.shape[1], q.data_ptr(), n, c.num_heads, c.num_kv_heads,
                                         d, start, c.rope_theta, kv.k[layer].data_ptr(), kv.v[layer].data_ptr(),
                                         kv.max_seq, self._stream()), "er_rope_kv")
        keys, values = kv.k[layer, :end], kv.v[layer, :end]
        if c.num_kv_heads != c.num_heads:
            rep = c.num_heads // c.num_kv_heads
            keys, values = keys.repeat_interleave(rep, dim=1), values.repeat_interleave(rep, dim=1)
        out = torch.empty((n, c.num_heads * d), dtype=torch.float32, device=self.device)
        _lib.check(_lib.lib().er_attention(q.data_ptr(), keys.contiguous().data_ptr(), values.contiguous().data_ptr(),
                                           allowed.data_ptr(), out.data_ptr(), n, end, c.num_heads, d,
                                           self._stream()), "er_attention")
        return self._linear(out, w["o_proj"])

    def forward(self, token_ids, kv: KVCache, *, all_logits: bool = False, expert_trace=None) -> torch.Tensor:
        """Run `token_ids` after what `kv` holds; logits [vocab] of the last
        position (or [n, vocab] with all_logits), on the device."""
        c = self.c
        ids = torch.as_tensor(np.asarray(token_ids, dtype=np.int64)).to(self.device)
        n = ids.shape[0]
        if kv.length + n > kv.max_seq:
            raise ValueError(f"sequence length {kv.length + n} exceeds the KV cache ({kv.max_seq})")
        x = torch.empty((n, c.hidden_size), dtype=torch.float32, device=self.device)
        _lib.check(_lib.lib().er_embed_int8(self.embed_q.data_ptr(), self.embed_s.data_ptr(), c.vocab_size,
                                            c.hidden_size, ids.data_ptr(), n, x.data_ptr(), self._bad.data_ptr(),
                                            self._stream()), "er_embed_int8")
        if expert_trace is not None:
            positions = kv.length + np.arange(n)
            expert_trace.begin(positions, np.asarray(token_ids), PHASE_PREFILL if kv.length == 0 else PHASE_DECODE)
        # causal: query start + i sees keys 0 .. start + i (the same for every layer)
        start, end = kv.length, kv.length + n
        allowed = (torch.arange(end, device=self.device)[None, :]
                   <= (start + torch.arange(n, device=self.device))[:, None]).to(torch.uint8)
        h = self._norm(x, self.layers[0]["in_norm"])
        for layer in range(c.num_layers):
            a = self._attention(layer, h, kv, allowed)
            h = self._norm(x, self.layers[layer]["post_norm"], add=a)
            y = self.stack.moe(layer, h, self.path, trace=expert_trace)
            if layer + 1 < c.num_layers:
                h = self._norm(x, self.layers[layer + 1]["in_norm"], add=y)
        kv.length += n
        if expert_trace is not None:
            expert_trace.end()
        rows = slice(None) if all_logits else slice(n - 1, n)
        xf, yf = x[rows].contiguous(), y[rows].contiguous()
        final = self._norm(xf, self.final_norm, add=yf)
        logits = self._linear(final, (self.head_q, self.head_s))
        if int(self._bad.item()):
            self._bad.zero_()
            raise ValueError(f"token ids outside [0, {c.vocab_size})")
        return logits if all_logits else logits[0]

    def generate(self, prompt, new_tokens: int, *, max_seq: int | None = None, expert_trace=None):
        """Greedy decoding (runtime/generate.py): the prompt in one call, then
        one token per call. Returns (generated ids, seconds of the prompt call,
        seconds per decode call)."""
        prompt = [int(t) for t in prompt]
        kv = self.new_cache(max_seq or len(prompt) + new_tokens)
        torch.cuda.synchronize(self.device)
        t0 = time.perf_counter()
        logits = self.forward(prompt, kv, expert_trace=expert_trace)
        tok = int(torch.argmax(logits).item())
        t_prompt = time.perf_counter() - t0
        out, step = [tok], []
        for _ in range(new_tokens - 1):
            t1 = time.perf_counter()
            logits = self.forward([tok], kv, expert_trace=expert_trace)
            tok = int(torch.argmax(logits).item())
            step.append(time.perf_counter() - t1)
            out.append(tok)
        return out, t_prompt, step
