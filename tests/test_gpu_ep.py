"""GPU: expert parallelism through the library (EpCudaOps) over NCCL.

Each rank's output must equal, bit for bit, the single-GPU block on the same
tokens routed from the same logits: every routed row is computed from that
row alone and the combine adds in the block's order. One rank runs without
collectives; two ranks need two GPUs (skipped otherwise).
"""

from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from expertrelay_b200 import _lib, synth
from expertrelay_b200.ep import EpCudaOps, ExpertParallelMoe
from expertrelay_b200.moe import MoeBlock

pytestmark = pytest.mark.gpu

PATHS = {"auto": _lib.PATH_AUTO, "gemv": _lib.PATH_GEMV, "gemm": _lib.PATH_GEMM, "tc": _lib.PATH_TC}


def _expected(block, h, path, device, ep):
    """The single-GPU block on the router logits the expert-parallel layer
    routes from (the same top-k kernel then picks the same experts)."""
    mb = MoeBlock.from_host_block(block, device=device)
    return mb.forward(h, logits=ep.ops.route(h)[0], path=path)


@pytest.mark.parametrize("m", [8, 200])
@pytest.mark.parametrize("path", ["tc", "gemv", "gemm"])
def test_rows_with_an_expert_id_out_of_range_come_back_nan(cuda, path, m):
    """A row bound for an expert this rank does not hold (id = the rank's
    expert count) makes the tallies disagree with the rows: the plan reports
    it and holds no work items, no expert kernel reads a record, and every
    row comes back NaN rather than a silent partial result. The same rows
    with valid ids come back finite, before and after."""
    block = synth.make_block(4, num_experts=16)
    ops = EpCudaOps(block, 0, 1, cuda, PATHS[path])
    x = torch.from_numpy(synth.make_tokens(5, m)).to(cuda)
    meta = torch.zeros((m, 2), dtype=torch.int32, device=cuda)
    meta[:, 0] = torch.arange(m, dtype=torch.int32, device=cuda) % 16
    meta[:, 1] = torch.full((m,), 0.25, device=cuda).view(torch.int32)
    y_ok = ops.rows(x, meta).clone()
    bad = meta.clone()
    bad[m // 2, 0] = 16
    y_bad = ops.rows(x, bad).clone()
    y_again = ops.rows(x, meta).clone()
    torch.cuda.synchronize()
    assert torch.isfinite(y_ok).all()
    assert torch.isnan(y_bad).all()
    assert torch.equal(y_again, y_ok)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("path", list(PATHS))
def test_one_rank_equals_the_block(cuda, path, dtype):
    """One rank: the layer is the block; the exchange path (taken when the
    steps are timed) gives the same bits."""
    block = synth.make_block(4, num_experts=16)
    ep = ExpertParallelMoe(EpCudaOps(block, 0, 1, cuda, PATHS[path]))
    hs = []
    for n in (3, 40, 300):
        h = torch.from_numpy(synth.make_tokens(60 + n, n)).to(cuda).to(dtype)
        y = ep(h)
        ref = _expected(block, h, PATHS[path], cuda, ep)
        torch.cuda.synchronize()
        assert torch.equal(y, ref), f"n={n}"
        hs.append(h)
    # the same batches as microbatches of one call (one count read-back), and
    # through pack / rows / combine with the steps timed
    phases = {}
    for h, y, y2 in zip(hs, ep.forward_many(hs), ep.forward_many(hs, phases=phases)):
        ref = _expected(block, h, PATHS[path], cuda, ep)
        torch.cuda.synchronize()
        assert torch.equal(y, ref), f"forward_many, n={h.shape[0]}"
        assert torch.equal(y2, ref), f"forward_many through the exchange steps, n={h.shape[0]}"
    assert {"route", "counts", "shared", "pack", "dispatch", "rows", "return", "combine"} <= set(phases)


def test_bf16_results_within_the_bf16_tolerance(cuda):
    """Routed results sent back in bf16: each rank's output within the bf16
    tolerance (rel-L2 1e-2) of the oracle on the same bf16 tokens and
    logits, and close to the fp32-return output."""
    from helpers import oracle_weights

    from oracle import moe_oracle as O

    block = synth.make_block(5, num_experts=16)
    h = torch.from_numpy(synth.make_tokens(77, 200)).to(cuda).to(torch.bfloat16)
    ep32 = ExpertParallelMoe(EpCudaOps(block, 0, 1, cuda, _lib.PATH_TC))
    ep16 = ExpertParallelMoe(EpCudaOps(block, 0, 1, cuda, _lib.PATH_TC, return_bf16=True))
    y32 = ep32.forward_many([h], phases={})[0]
    y16 = ep16.forward_many([h], phases={})[0]
    logits = ep32.ops.route(h)[0]
    ref = O.moe_block(h.float().cpu().numpy(), oracle_weights(block), logits=logits.cpu().numpy())
    assert O.rel_l2(y16.cpu().numpy(), ref.y) < 1e-2
    assert O.rel_l2(y16.cpu().numpy(), y32.cpu().numpy()) < 5e-3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=120))
    try:
        block = synth.make_block(4)  # Qwen shapes: 60 experts, 30 per rank
        for path, dtype in ((_lib.PATH_TC, torch.float32), (_lib.PATH_GEMV, torch.float32),
                            (_lib.PATH_TC, torch.bfloat16)):
            ep = ExpertParallelMoe(EpCudaOps(block, rank, world, dev, path))
            if dtype == torch.bfloat16:  # results back in bf16: within the bf16 rounding of the fp32 ones
                ep16 = ExpertParallelMoe(EpCudaOps(block, rank, world, dev, path, return_bf16=True))
                h = torch.from_numpy(synth.make_tokens(50 + rank, 64 + 16 * rank)).to(dev).to(dtype)
                y16, y32 = ep16(h), ep(h)
                torch.cuda.synchronize()
                rel = ((y16 - y32).norm() / y32.norm()).item()
                if not rel < 5e-3:
                    raise AssertionError(f"rank {rank}: bf16 results differ from fp32 by rel-L2 {rel:.2e}")
            for n in (8, 96 + 32 * rank):  # ragged across ranks
                h = torch.from_numpy(synth.make_tokens(70 + 10 * rank + n, n)).to(dev).to(dtype)
                y = ep(h)
                ref = _expected(block, h, path, dev, ep)
                torch.cuda.synchronize()
                if not torch.equal(y, ref):
                    diff = (y - ref).abs().max().item()
                    raise AssertionError(f"rank {rank} path {path} {dtype} n={n}: max diff {diff}")
            hs = [torch.from_numpy(synth.make_tokens(90 + 10 * rank + n, n)).to(dev).to(dtype)
                  for n in (16, 0 if rank == 0 else 5, 200 + 24 * rank)]  # rank 0 has an empty microbatch
            for j, (h, y) in enumerate(zip(hs, ep.forward_many(hs))):
                if h.shape[0] == 0:
                    if y.shape != h.shape:
                        raise AssertionError(f"rank {rank}: empty microbatch gave {tuple(y.shape)}")
                    continue
                ref = _expected(block, h, path, dev, ep)
                torch.cuda.synchronize()
                if not torch.equal(y, ref):
                    raise AssertionError(f"rank {rank} path {path} {dtype} forward_many microbatch {j} differs")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_over_nccl_equal_the_block():
    mp.start_processes(_rank_main, args=(2, _free_port()), nprocs=2, start_method="spawn")
