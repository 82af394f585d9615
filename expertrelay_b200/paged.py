"""PagedMoeStack: MoE layers whose routed experts live in an HbmExpertCache.

The runtime's cache hooks around the MoE block (runtime/qwen_moe.py:
293-351), on the GPU: per layer, the router and top-k run on the device, the
selected expert ids come back to the host, the cache makes those records
resident (copies from pinned host memory on its copy stream, which the
compute stream waits for) and the block runs on them through its expert
table. With a prefetch policy, the next layer's router applied to this
layer's input (the Fate guess, qwen_moe.py:314-320) picks experts whose
copies start while this layer computes, keeping this layer's experts
(qwen_moe.py:326-336). This layer's own records are acquired (their copies
queued) before the guess is prefetched, so they are always copied first (the
reference's prefill pipelining, qwen_moe.py:324-325, is the only order here).

prefetch_adaptive caps the guess's new copies on one-token calls at what
fits in the layer's window (qwen_moe.py:361-374): the device time from this
layer's block to the next layer's block, measured with CUDA events on the
compute stream during the previous one-token call and smoothed per layer,
divided by the time of one record copy (pinned host -> HBM, measured once).
"""

from __future__ import annotations

import numpy as np
import torch

from . import _lib
from .cache import HbmExpertCache
from .moe import MoeBlock
from .prefetch import PrefetchPolicy

WINDOW_EMA = 0.5  # weight of the newest call in a layer's window estimate (qwen_moe.py:227)


def read_budget(window_s: float, read_s: float, top_k: int) -> int:
    """New prefetch copies that fit before the next layer needs its experts,
    at least one; top_k while no window has been measured
    (qwen_moe.py:361-367, one copy stream)."""
    if not np.isfinite(window_s):
        return top_k
    return max(1, int(round(window_s / read_s)))


def update_window(old: float, new: float, ema: float = WINDOW_EMA) -> float:
    """Running per-layer window estimate (qwen_moe.py:369-374)."""
    return new if np.isnan(old) else old + ema * (new - old)


def measure_copy_seconds(cache: HbmExpertCache, repeats: int = 3) -> float:
    """Seconds of one record copy from the cache's host source to HBM, timed
    with CUDA events on a private stream (one warm-up copy first)."""
    src = cache.source.record(0, 0)
    dst = torch.empty(src.numel(), dtype=torch.uint8, device=cache.device)
    stream = torch.cuda.Stream(cache.device)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        dst.copy_(src, non_blocking=True)
        t0.record(stream)
        for _ in range(repeats):
            dst.copy_(src, non_blocking=True)
        t1.record(stream)
    t1.synchronize()
    return t0.elapsed_time(t1) / 1e3 / repeats


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
        # the adaptive read budget: a switch that is safe to flip between calls
        self.prefetch_adaptive = False
        self.window = np.full(len(self.layers), np.nan)  # seconds hiding layer L+1's prefetch
        self.read_seconds: float | None = None  # one record copy, measured on first use
        self._mark = [torch.cuda.Event(enable_timing=True) for _ in self.layers]
        self._marked = np.zeros(len(self.layers), dtype=bool)

    def _update_windows(self) -> None:
        """Fold the previous one-token call's block-to-block times into the
        per-layer windows (its events are complete: the call's result was
        read back before this one began, else the pair is skipped)."""
        for layer in range(len(self.layers) - 1):
            if self._marked[layer] and self._marked[layer + 1] and self._mark[layer + 1].query():
                w = self._mark[layer].elapsed_time(self._mark[layer + 1]) / 1e3
                self.window[layer] = update_window(self.window[layer], w)
        self._marked[:] = False

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
        if layer == 0:
            self._update_windows()
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
        adaptive = self.prefetch_adaptive and n == 1
        if self.prefetch_enabled and has_next:
            choice = self.prefetcher.choose(fate.cpu().numpy())
            self.prefetches_skipped_low_confidence += choice.skipped_low_confidence
            budget = None
            if adaptive:
                if self.read_seconds is None:
                    self.read_seconds = measure_copy_seconds(cache)
                budget = read_budget(self.window[layer], self.read_seconds, self.top_k)
            cache.prefetch(layer + 1, choice.experts, keep=[(layer, int(e)) for e in needed], max_new_reads=budget)
        if adaptive:  # this layer's block starts here on the compute stream
            self._mark[layer].record(torch.cuda.current_stream(h.device))
            self._marked[layer] = True
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
