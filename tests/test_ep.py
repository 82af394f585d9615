"""Expert parallelism, host side: the expert partition and the exchange of
ExpertParallelMoe (counts, rows out, results back, combine) on two and four
gloo ranks on the CPU.

The per-rank steps run on the host here (HostOps, built on the oracle), with
the same contracts as the CUDA steps (expertrelay_b200.ep.EpCudaOps): rows of
one destination in any order, pos_of recording where each pair went. The
output of both ranks must match the oracle's whole block on each rank's
tokens. The CUDA steps over NCCL are tests/test_gpu_ep.py.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from helpers import oracle_weights

from expertrelay_b200 import synth
from expertrelay_b200.ep import ExpertParallelMoe, expert_partition, owner_tables
from oracle import moe_oracle as O

SHAPE = {"hidden": 64, "inter": 32, "shared_inter": 48, "num_experts": 10, "top_k": 3}


def test_expert_partition_matches_the_plan():
    assert expert_partition(60, 1) == [(0, 60)]
    assert expert_partition(60, 2) == [(0, 30), (30, 60)]
    assert [hi - lo for lo, hi in expert_partition(60, 4)] == [15] * 4
    assert [hi - lo for lo, hi in expert_partition(60, 8)] == [8, 8, 8, 8, 7, 7, 7, 7]
    owner, local = owner_tables(60, 8)
    assert owner[0] == 0 and owner[59] == 7 and local[32] == 0 and local[59] == 6
    with pytest.raises(ValueError):
        expert_partition(3, 4)


class HostOps:
    """The per-rank steps of ExpertParallelMoe on CPU tensors, on the oracle."""

    def __init__(self, block, rank: int, ranks: int):
        self.ranks = ranks
        self.w = oracle_weights(block)
        self.k = block.top_k
        self.lo, self.hi = expert_partition(block.num_experts, ranks)[rank]
        self.owner, self.local = owner_tables(block.num_experts, ranks)

    def route(self, h):
        logits = O.linear(h.numpy(), self.w.router)
        probs = O.softmax(logits)
        idx = O.top_k_desc(probs, self.k)
        w = np.take_along_axis(probs, idx, axis=-1)
        return torch.from_numpy(logits), torch.from_numpy(idx.astype(np.int32)), torch.from_numpy(w)

    def count(self, idx):
        return torch.from_numpy(np.bincount(self.owner[idx.numpy().ravel()], minlength=self.ranks).astype(np.int32))

    def pack(self, h, idx, w, offsets, total):
        n, k = idx.shape
        x = np.empty((total, h.shape[1]), np.float32)
        meta = np.empty((total, 2), np.int32)  # (local expert id, weight bits)
        w_send = meta[:, 1].view(np.float32)
        e_send = meta[:, 0]
        pos_of = np.empty((n, k), np.int32)
        cursor = offsets.numpy().copy()
        # destination by destination, pairs in reverse order: any order is allowed
        for t in reversed(range(n)):
            for j in range(k):
                e = int(idx[t, j])
                d = self.owner[e]
                p = cursor[d]
                cursor[d] += 1
                x[p], e_send[p], w_send[p], pos_of[t, j] = h[t].numpy(), self.local[e], w[t, j], p
        return torch.from_numpy(x), torch.from_numpy(meta), torch.from_numpy(pos_of)

    def rows(self, x, meta):
        x, meta = x.numpy(), np.ascontiguousarray(meta.numpy())
        expert, weight = meta[:, 0].copy(), meta[:, 1].copy().view(np.float32)
        y = np.zeros_like(x)
        for e in np.unique(expert):
            r = np.nonzero(expert == e)[0]
            m = self.w.experts[self.lo + int(e)]
            act = O.silu(O.int8_linear(x[r], m["gate_proj"].q, m["gate_proj"].scales)) * O.int8_linear(
                x[r], m["up_proj"].q, m["up_proj"].scales)
            y[r] = O.int8_linear(act, m["down_proj"].q, m["down_proj"].scales) * weight[r][:, None]
        return torch.from_numpy(y)

    def shared(self, h):
        h = h.numpy()
        sh = self.w.shared
        s = O.int8_linear(O.silu(O.int8_linear(h, sh["gate_proj"].q, sh["gate_proj"].scales))
                          * O.int8_linear(h, sh["up_proj"].q, sh["up_proj"].scales),
                          sh["down_proj"].q, sh["down_proj"].scales)
        return torch.from_numpy(O.sigmoid(O.linear(h, self.w.shared_gate)) * s)

    def combine(self, y_ret, pos_of, idx, y_s):
        idx, pos_of, y_ret = idx.numpy(), pos_of.numpy(), y_ret.numpy()
        y = np.zeros_like(y_s.numpy())
        for t in range(idx.shape[0]):
            for j in np.argsort(idx[t], kind="stable"):  # ascending expert id
                y[t] += y_ret[pos_of[t, j]]
        return torch.from_numpy(y + y_s.numpy())


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        block = synth.make_block(9, **SHAPE)
        n = 5 + 7 * rank  # ragged: the ranks hold different token counts
        h = torch.from_numpy(synth.make_tokens(30 + rank, n, SHAPE["hidden"]))
        ep = ExpertParallelMoe(HostOps(block, rank, world))
        y = ep(h).numpy()
        ref = O.moe_block(h.numpy(), oracle_weights(block)).y
        counts = ep.last_counts
        # several microbatches with one count exchange; one of them empty on rank 0
        parts = [torch.from_numpy(synth.make_tokens(40 + rank + j, m, SHAPE["hidden"]))
                 for j, m in enumerate((3 + rank, 0 if rank == 0 else 2, 6))]
        many = ep.forward_many(parts)
        err_many = max(O.rel_l2(y_j.numpy(), O.moe_block(p.numpy(), oracle_weights(block)).y)
                       for y_j, p in zip(many, parts) if p.shape[0])
        assert all(y_j.shape == p.shape for y_j, p in zip(many, parts))
        # the timed, one-step-after-another variant gives the same outputs
        timed = ep.forward_many(parts, phases={})
        assert all(torch.equal(a, b) for a, b in zip(many, timed))
        assert sum(ep.last_counts[0]) == sum(p.shape[0] for p in parts) * SHAPE["top_k"]
        results[rank] = (max(O.rel_l2(y, ref), err_many), counts)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_exchange_on_gloo_matches_the_whole_block(world):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        mp.start_processes(_rank_main, args=(world, _free_port(), results), nprocs=world, start_method="spawn")
        res = dict(results)
    assert sorted(res) == list(range(world))
    for rank, (err, (send, recv)) in res.items():
        assert err < 1e-5, f"rank {rank}: rel-L2 {err:.2e}"
        assert sum(send) == (5 + 7 * rank) * SHAPE["top_k"]
    # what rank a sent to rank b is what rank b received from rank a
    for a in range(world):
        for b in range(world):
            assert res[a][1][0][b] == res[b][1][1][a], f"rank {a} -> rank {b}"
