"""PagedMoeStack: MoE layers whose routed experts live in an HbmExpertCache.

The runtime's cache hooks around the MoE block (runtime/qwen_moe.py:
293-351), on the GPU: per layer, the router and top-k run on the device, the
selected expert ids come back to the host, the cache makes those records
resident (copies from pinned host memory on its copy stream, which the
compute stream waits for) and the block runs on them through its expert
table. With a prefetch policy, the next layer's router applied to this
layer's input (the Fate guess, qwen_moe.py:314-320) picks experts whose
copies start while this layer computes, keeping this layer's experts
(qwen_moe.py:326-336).
"""

from __future__ import annotations

import numpy as np
import torch

from . import _lib
from .cache import HbmExpertCache
from .moe import MoeBlock
from .prefetch import PrefetchPolicy


class PagedMoeStack:
    """blocks: one HostBlock-like per layer (router, shared_gate, shared,
    shared_inter, layout, top_k); their routed records are the cache's
    source (HostRecords.from_blocks)."""

    def __init__(
        self,
        blocks,
        cache: HbmExpertCache,
        *,
        prefetcher: PrefetchPolicy | None = None,
        norm_topk_prob: bool = False,
    ):
        self.cache = cache
        self.norm_topk_prob = norm_topk_prob
        self.prefetcher = prefetcher
        self.prefetch_enabled = prefetcher is not None
        self.layers = [
            MoeBlock(router=b.router, shared_gate=b.shared_gate, shared=b.shared, layout=b.layout,
                     shared_inter=b.shared_inter, records=None, top_k=b.top_k, norm_topk_prob=norm_topk_prob,
                     device=cache.device)
            for b in blocks
        ]
        self.num_experts = self.layers[0].num_experts
        self.top_k = self.layers[0].top_k
        # per layer, the expert table staged in pinned memory so its copy to the
        # device is asynchronous (a layer's buffer is reused only a forward later)
        self._table_host = [torch.empty(self.num_experts, dtype=torch.int64, pin_memory=True) for _ in self.layers]
        self.prefetches_skipped_low_confidence = 0

    def moe(self, layer: int, h: torch.Tensor, path: int = _lib.PATH_AUTO, *, trace=None,
            return_routing: bool = False):
        """One layer's MoE block output for h [n, H] (the layer's QwenMoe._moe).
        `trace`: an ExpertTraceWriter between begin() and end(); this layer's
        router logits, choices, weights and the Fate logits for the next
        layer go to it (qwen_moe.py:311-338). return_routing: also the
        [n, k] int64 expert ids."""
        blk = self.layers[layer]
        cache = self.cache
        n = h.shape[0]
        logits = blk.router_logits(h)
        idx = torch.empty((n, self.top_k), dtype=torch.int64, device=h.device)
        wts = torch.empty((n, self.top_k), dtype=torch.float32, device=h.device)
        stream = torch.cuda.current_stream(h.device).cuda_stream
        rc = _lib.lib().er_router_topk(logits.data_ptr(), n, self.num_experts, self.top_k, idx.data_ptr(), None,
                                       wts.data_ptr(), stream)
        _lib.check(rc, "er_router_topk")
        has_next = layer + 1 < len(self.layers)
        fate = None
        if (self.prefetch_enabled or trace is not None) and has_next:
            # the next layer's router on this layer's input (the Fate guess),
            # queued before the ids are read back so one wait covers both
            fate = self.layers[layer + 1].router_logits(h)
        needed = np.unique(idx.cpu().numpy())  # the host decides which records to fetch
        addrs = cache.acquire(layer, needed)
        table = self._table_host[layer].numpy().view(np.uint64)
        table[:] = int(addrs[0])  # unrouted experts: never read
        table[needed] = addrs
        blk.use_arena(cache.arena_base, cache.num_slots)
        blk.set_expert_table(self._table_host[layer])
        if self.prefetch_enabled and has_next:
            choice = self.prefetcher.choose(fate.cpu().numpy())
            self.prefetches_skipped_low_confidence += choice.skipped_low_confidence
            cache.prefetch(layer + 1, choice.experts, keep=[(layer, int(e)) for e in needed])
        if trace is not None:
            if self.norm_topk_prob:  # the block's weights, renormalised as it uses them
                wts = wts / wts.sum(dim=-1, keepdim=True)
            trace.layer(layer, logits, idx, wts, fate)
        y = blk.forward(h, logits=logits, path=path)
        cache.end_layer(layer)
        return (y, idx) if return_routing else y

    def forward(self, h: torch.Tensor, path: int = _lib.PATH_AUTO, *, trace=None) -> torch.Tensor:
        """All layers in order, each adding its MoE output to the residual
        stream: h <- h + moe_l(h). `trace`: a writer between begin() and
        end() (the caller's, who knows the tokens' positions and ids)."""
        for layer in range(len(self.layers)):
            h = h + self.moe(layer, h, path, trace=trace)
        return h
