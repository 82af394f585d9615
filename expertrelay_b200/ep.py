"""Expert parallelism for the MoE block: one process per GPU, the routed
experts of a layer spread over the ranks, tokens staying on their rank.

The reference computes every expert in one process (runtime/qwen_moe.py:
340-359). Here rank r holds experts [lo_r, hi_r) (contiguous, sizes differing
by at most one: 30/30 at 2 GPUs, 15 x 4 at 4, 8,8,8,8,7,7,7,7 at 8) and the
replicated router, shared gate and shared expert. Per layer, on each rank:

  1. route its tokens (router + softmax/top-k, same kernels as the block);
  2. count the (token, slot) pairs bound for each rank and exchange the
     counts (all-to-all of ints; one exchange and one host read-back for
     all of a call's microbatches);
  3. pack the pairs' token rows by destination, with their local expert id
     and routing weight interleaved in one int32 [rows, 2] buffer, and send
     both (two all-to-alls per microbatch);
  4. compute the received rows with its own experts (er_moe_rows), results
     in fp32 or, with return_bf16, rounded to bf16 (half the bytes back);
  5. send the results back (all-to-all), the reverse of 3;
  6. add each token's slots in ascending expert id, plus the gated shared
     expert computed locally (er_moe_shared, er_moe_combine); the shared
     expert needs only the rank's own tokens, so it is queued right after
     routing and, on GPUs, runs on a side stream beside steps 2-5.

The exchanges are asynchronous: every microbatch is packed and its rows sent
before any is computed, so microbatch j+1's rows travel over NVLink while
microbatch j's experts run; the results go back the same way. With fp32
results each routed row's result depends only on that row and the combine
adds in the reference's order, so the output equals the single-GPU block's
on the same router logits bit for bit; bf16 results round each routed
contribution once (within the bf16 tolerance). On one rank there is nothing
to exchange and the layer runs as the block (ops.block) when the ops offer it.

The collectives are torch.distributed's (NCCL over NVLink on GPUs); the
steps on each rank are an `ops` object: EpCudaOps runs them through the
library; tests may pass host implementations to exercise the exchange.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from ._lib import MoeRowsIO, MoeWeights
from .moe import MoeBlock
from .store import FMT_INT8


def expert_partition(num_experts: int, ranks: int) -> list[tuple[int, int]]:
    """Contiguous [lo, hi) expert ranges per rank, the larger ones first."""
    if ranks < 1 or num_experts < ranks:
        raise ValueError(f"cannot spread {num_experts} experts over {ranks} ranks")
    base, extra = divmod(num_experts, ranks)
    out, lo = [], 0
    for r in range(ranks):
        hi = lo + base + (1 if r < extra else 0)
        out.append((lo, hi))
        lo = hi
    return out


def owner_tables(num_experts: int, ranks: int) -> tuple[np.ndarray, np.ndarray]:
    """owner[e] = rank holding expert e; local[e] = its index on that rank."""
    owner = np.empty(num_experts, dtype=np.int32)
    local = np.empty(num_experts, dtype=np.int32)
    for r, (lo, hi) in enumerate(expert_partition(num_experts, ranks)):
        owner[lo:hi] = r
        local[lo:hi] = np.arange(hi - lo, dtype=np.int32)
    return owner, local


class EpCudaOps:
    """The per-rank steps on this rank's GPU, through the library. `block`: the
    layer's HostBlock (router, shared expert, all routed records; only the
    records of experts [lo, hi) are uploaded)."""

    def __init__(self, block, rank: int, ranks: int, device, path: int = _lib.PATH_AUTO, return_bf16: bool = False):
        self.device = torch.device(device)
        # AUTO resolved as the single-GPU block resolves it for int8 records in
        # an arena (the tensor-core path), the same for the routed rows and the
        # shared expert; for int4 records the library picks by row count
        self.path = _lib.PATH_TC if path == _lib.PATH_AUTO and block.layout.fmt == FMT_INT8 else path
        self.ranks = ranks
        self.lo, self.hi = expert_partition(block.num_experts, ranks)[rank]
        self.top_k, self.hidden, self.num_experts = block.top_k, block.hidden, block.num_experts
        # router, shared gate and shared expert (replicated); no routed records here
        self.full = MoeBlock(router=block.router, shared_gate=block.shared_gate, shared=block.shared,
                             layout=block.layout, shared_inter=block.shared_inter, records=None, top_k=block.top_k,
                             device=self.device)
        owner, local = owner_tables(block.num_experts, ranks)
        self.owner = torch.from_numpy(owner).to(self.device)
        self.local = torch.from_numpy(local).to(self.device)
        rs = block.layout.record_size
        recs = block.records()[self.lo : self.hi]
        self.records = torch.from_numpy(np.ascontiguousarray(recs)).to(self.device)
        n_local = self.hi - self.lo
        self.table = torch.arange(n_local, dtype=torch.int64, device=self.device) * rs + self.records.data_ptr()
        fw = self.full._w
        # this rank's experts as a block of n_local experts
        self.w_rows = MoeWeights(
            hidden=fw.hidden, num_experts=n_local, top_k=1, inter=fw.inter, shared_inter=fw.shared_inter,
            expert_fmt=fw.expert_fmt, group=fw.group, norm_topk_prob=0, router_w=None, shared_gate_w=None,
            expert_records=self.table.data_ptr(), shared_record=None,
            record_arena=self.records.data_ptr(),
            arena_slots=n_local,
        )
        if ranks == 1:  # every expert here: the block itself serves the layer
            self.full.use_arena(self.records.data_ptr(), n_local)
            self.full.set_expert_table(self.table)
        self.return_dtype = torch.bfloat16 if return_bf16 else torch.float32
        self._route_scratch: torch.Tensor | None = None
        self.cursor = torch.zeros(ranks, dtype=torch.int32, device=self.device)
        self._ws: torch.Tensor | None = None  # the routed rows' workspace
        # the shared expert runs on a side stream, beside the exchange and the
        # routed rows, with a workspace of its own
        self._ws_shared: torch.Tensor | None = None
        self._side = torch.cuda.Stream(self.device)

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def _workspace(self, nbytes: int) -> torch.Tensor:
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=self.device)
        return self._ws

    def route(self, h: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(router logits [n, E], expert ids int32 [n, k], weights [n, k])."""
        n = h.shape[0]
        idx = torch.empty((n, self.top_k), dtype=torch.int32, device=self.device)
        w = torch.empty((n, self.top_k), dtype=torch.float32, device=self.device)
        if n == 0:  # an empty microbatch still takes part in the exchange
            return torch.empty((0, self.num_experts), dtype=torch.float32, device=self.device), idx, w
        logits = torch.empty((n, self.num_experts), dtype=torch.float32, device=self.device)
        L = _lib.lib()
        nbytes = L.er_route_scratch_bytes(n, self.num_experts)
        if self._route_scratch is None or self._route_scratch.numel() < nbytes:
            self._route_scratch = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=self.device)
        sc = self._route_scratch
        dtype = _lib.DTYPE_BF16 if h.dtype == torch.bfloat16 else _lib.DTYPE_F32
        h = h.contiguous()
        _lib.check(L.er_route(h.data_ptr(), dtype, n, self.hidden, self.full.router.data_ptr(), self.num_experts,
                              self.top_k, 0, sc.data_ptr(), sc.numel(), logits.data_ptr(), idx.data_ptr(),
                              w.data_ptr(), self._stream()), "er_route")
        return logits, idx, w

    def count(self, idx: torch.Tensor) -> torch.Tensor:
        counts = torch.empty(self.ranks, dtype=torch.int32, device=self.device)
        n = idx.shape[0]
        _lib.check(_lib.lib().er_ep_count(idx.data_ptr(), n, self.top_k, self.owner.data_ptr(), self.num_experts,
                                          self.ranks, counts.data_ptr(), self._stream()), "er_ep_count")
        return counts

    def pack(self, h: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, offsets: torch.Tensor, total: int):
        """(rows [total, H], meta int32 [total, 2] = (local expert id, weight
        bits), pos_of [n, k])."""
        n = h.shape[0]
        dtype = _lib.DTYPE_BF16 if h.dtype == torch.bfloat16 else _lib.DTYPE_F32
        x_send = torch.empty((total, self.hidden), dtype=h.dtype, device=self.device)
        meta = torch.empty((total, 2), dtype=torch.int32, device=self.device)
        pos_of = torch.empty((n, self.top_k), dtype=torch.int32, device=self.device)
        _lib.check(_lib.lib().er_ep_pack(
            h.data_ptr(), dtype, self.hidden, idx.data_ptr(), w.data_ptr(), n, self.top_k, self.owner.data_ptr(),
            self.local.data_ptr(), self.num_experts, self.ranks, offsets.data_ptr(), self.cursor.data_ptr(),
            x_send.data_ptr(), meta.data_ptr(), meta.data_ptr() + 4, 2, pos_of.data_ptr(), self._stream()),
            "er_ep_pack")
        return x_send, meta, pos_of

    def rows(self, x: torch.Tensor, meta: torch.Tensor) -> torch.Tensor:
        """This rank's experts on received rows; [m, H] fp32 (bf16 with return_bf16)."""
        m = x.shape[0]
        y = torch.empty((m, self.hidden), dtype=self.return_dtype, device=self.device)
        if m == 0:
            return y
        expert = meta[:, 0].contiguous()
        weight = meta[:, 1].contiguous().view(torch.float32)
        ws = self._workspace(_lib.lib().er_moe_rows_workspace_bytes(C.byref(self.w_rows), m, self.path))
        io = MoeRowsIO(x=x.data_ptr(), x_dtype=_lib.DTYPE_BF16 if x.dtype == torch.bfloat16 else _lib.DTYPE_F32,
                       m=m, expert=expert.data_ptr(), weight=weight.data_ptr(), y=y.data_ptr(), path=self.path,
                       y_dtype=_lib.DTYPE_BF16 if self.return_dtype == torch.bfloat16 else _lib.DTYPE_F32)
        _lib.check(_lib.lib().er_moe_rows(C.byref(self.w_rows), C.byref(io), ws.data_ptr(), ws.numel(),
                                          self._stream()), "er_moe_rows")
        return y

    def block(self, h: torch.Tensor, logits: torch.Tensor) -> torch.Tensor:
        """One rank holds every expert: the whole block on these logits."""
        if self.ranks != 1:
            raise RuntimeError("the whole block runs only when one rank holds every expert")
        return self.full.forward(h, logits=logits, path=self.path)

    def shared(self, h: torch.Tensor) -> torch.Tensor:
        """The gated shared expert of this rank's tokens, queued on a side
        stream after the work already queued for h, so that it overlaps the
        exchange and the routed rows; combine() waits for it."""
        n = h.shape[0]
        y = torch.empty((n, self.hidden), dtype=torch.float32, device=self.device)
        if n == 0:
            return y
        w = self.full._w
        nbytes = _lib.lib().er_moe_shared_workspace_bytes(C.byref(w), n, self.path)
        if self._ws_shared is None or self._ws_shared.numel() < nbytes:
            self._side.synchronize()  # the old workspace may still be in use there
            self._ws_shared = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=self.device)
        ws = self._ws_shared
        self._side.wait_stream(torch.cuda.current_stream(self.device))
        dtype = _lib.DTYPE_BF16 if h.dtype == torch.bfloat16 else _lib.DTYPE_F32
        _lib.check(_lib.lib().er_moe_shared(C.byref(w), h.data_ptr(), dtype, n, y.data_ptr(), self.path,
                                            ws.data_ptr(), ws.numel(), self._side.cuda_stream), "er_moe_shared")
        done = torch.cuda.Event()
        done.record(self._side)
        y.er_ready = done  # what combine() waits for
        # the caching allocator must not hand these to other work before the side stream is done
        y.record_stream(self._side)
        h.record_stream(self._side)
        return y

    def combine(self, y_ret, pos_of, idx, y_s) -> torch.Tensor:
        n = idx.shape[0]
        y = torch.empty((n, self.hidden), dtype=torch.float32, device=self.device)
        ready = getattr(y_s, "er_ready", None)
        if ready is not None:
            torch.cuda.current_stream(self.device).wait_event(ready)
        rows_dtype = _lib.DTYPE_BF16 if y_ret.dtype == torch.bfloat16 else _lib.DTYPE_F32
        _lib.check(_lib.lib().er_moe_combine(y_ret.data_ptr() if y_ret.numel() else None, rows_dtype,
                                             pos_of.data_ptr(), idx.data_ptr(), y_s.data_ptr(), n, self.top_k,
                                             self.hidden, y.data_ptr(), self._stream()), "er_moe_combine")
        return y


class ExpertParallelMoe:
    """One rank's part of an expert-parallel MoE layer (see the module
    docstring). `ops` provides route/count/pack/rows/shared/combine on this
    rank's tensors; `group` is the torch.distributed group (default: world)."""

    def __init__(self, ops, *, group=None):
        self.ops = ops
        self.group = group
        self.ranks = dist.get_world_size(group) if dist.is_initialized() else 1
        if self.ranks != ops.ranks:
            raise ValueError(f"ops are laid out for {ops.ranks} ranks, the group has {self.ranks}")
        self.last_counts: tuple[list[int], list[int]] | None = None

    def _a2a(self, out, inp, out_splits, in_splits, async_op=False):
        if self.ranks == 1:
            out.copy_(inp)
            return None
        return dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group, async_op=async_op)

    def forward(self, h):
        return self.forward_many([h])[0]

    __call__ = forward

    def forward_many(self, hs, phases: dict | None = None):
        """forward() over several microbatches of this rank's tokens (every
        rank passes the same number). Each microbatch is routed, its shared
        expert queued (on a side stream with the CUDA steps) and its rows
        counted; one exchange and one host read-back cover all their counts.
        Then every microbatch is packed and its rows and meta sent
        asynchronously, each is computed as its rows arrive and its results
        sent back asynchronously, and each is combined as its results
        arrive. last_counts then holds the rows sent to / received from each
        rank, summed over the microbatches.

        phases: a dict to time the steps instead, with CUDA events on the
        current stream (accumulated in ms under route, counts, pack,
        dispatch, rows, return, combine); the steps then run one after
        another, not overlapped, so their sum exceeds the overlapped call."""
        ops = self.ops
        timer = _PhaseTimer(phases)
        if self.ranks == 1 and phases is None and hasattr(ops, "block"):
            out = []
            for h in hs:
                logits, idx, _ = ops.route(h)
                out.append(ops.block(h, logits) if h.shape[0] else torch.empty_like(h, dtype=torch.float32))
            total = sum(int(h.shape[0]) for h in hs) * int(getattr(ops, "top_k", 0))
            self.last_counts = ([total], [total])
            return out
        routed = []
        timer.start("route")
        for h in hs:
            _, idx, w = ops.route(h)
            y_s = ops.shared(h) if phases is None else None
            routed.append([h, idx, w, y_s, ops.count(idx)])
        if not routed:
            return []
        timer.start("counts")
        # counts[j, r]: microbatch j's rows for rank r; exchanged as [r, j]
        counts = torch.stack([r[4] for r in routed]).t().contiguous()
        recv_counts = counts
        if self.ranks > 1:
            recv_counts = torch.empty_like(counts)
            self._a2a(recv_counts, counts, None, None)
        send_all = counts.cpu().numpy().T.astype(np.int64)  # [microbatch, rank]
        recv_all = recv_counts.cpu().numpy().T.astype(np.int64)
        self.last_counts = ([int(v) for v in send_all.sum(0)], [int(v) for v in recv_all.sum(0)])
        if phases is not None:
            timer.start("shared")
            for r in routed:
                r[3] = ops.shared(r[0])
                ready = getattr(r[3], "er_ready", None)
                if ready is not None:  # the side stream's work, inside this phase's events
                    torch.cuda.current_stream().wait_event(ready)
        # pack every microbatch and start sending its rows
        timer.start("pack")
        sent = []
        for (h, idx, w, _, _), send, recv in zip(routed, send_all, recv_all):
            send, recv = [int(v) for v in send], [int(v) for v in recv]
            offsets = torch.tensor(np.concatenate([[0], np.cumsum(send)[:-1]]).astype(np.int32), device=idx.device)
            x_send, meta_send, pos_of = ops.pack(h, idx, w, offsets, sum(send))
            sent.append((x_send, meta_send, pos_of, send, recv))
        timer.start("dispatch")
        arrivals = []
        for x_send, meta_send, _, send, recv in sent:
            if self.ranks == 1:  # the packed rows are the received rows
                arrivals.append((x_send, meta_send, []))
                continue
            x_recv = x_send.new_empty((sum(recv), x_send.shape[1]))
            meta_recv = meta_send.new_empty((sum(recv), 2))
            works = [self._a2a(x_recv, x_send, recv, send, async_op=True),
                     self._a2a(meta_recv, meta_send, recv, send, async_op=True)]
            if phases is not None:
                for wk in works:
                    wk.wait()
                works = []
            arrivals.append((x_recv, meta_recv, works))
        # compute each microbatch's rows as they arrive, send the results back
        timer.start("rows")
        returns = []
        for (x_recv, meta_recv, works), (x_send, _, _, send, recv) in zip(arrivals, sent):
            for wk in works:
                wk.wait()
            y_recv = ops.rows(x_recv, meta_recv)
            returns.append((y_recv, send, recv))
        timer.start("return")
        backs = []
        for y_recv, send, recv in returns:
            if self.ranks == 1:
                backs.append((y_recv, []))
                continue
            y_ret = y_recv.new_empty((sum(send), y_recv.shape[1]))
            wk = self._a2a(y_ret, y_recv, send, recv, async_op=True)
            if phases is not None:
                wk.wait()
                wk = None
            backs.append((y_ret, [wk] if wk is not None else []))
        timer.start("combine")
        out = []
        for (y_ret, works), (h, idx, _, y_s, _), (_, _, pos_of, _, _) in zip(backs, routed, sent):
            for wk in works:
                wk.wait()
            out.append(ops.combine(y_ret, pos_of, idx, y_s))
        timer.stop()
        return out


class _PhaseTimer:
    """CUDA events between the steps of forward_many (a no-op without a dict
    or a GPU)."""

    def __init__(self, phases: dict | None):
        self.phases = phases
        self.name = None
        self.ev = None

    def _event(self):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def start(self, name: str) -> None:
        if self.phases is None or not torch.cuda.is_available():
            return
        e = self._event()
        self.stop(e)
        self.name, self.ev = name, e

    def stop(self, end=None) -> None:
        if self.phases is None or self.name is None:
            return
        end = end or self._event()
        end.synchronize()
        self.phases[self.name] = self.phases.get(self.name, 0.0) + self.ev.elapsed_time(end)
        self.name = None
