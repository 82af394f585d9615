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


def _expected(block, h, path, device):
    mb = MoeBlock.from_host_block(block, device=device)
    return mb.forward(h, logits=mb.router_logits(h), path=path)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("path", list(PATHS))
def test_one_rank_equals_the_block(cuda, path, dtype):
    block = synth.make_block(4, num_experts=16)
    ep = ExpertParallelMoe(EpCudaOps(block, 0, 1, cuda, PATHS[path]))
    hs = []
    for n in (3, 40, 300):
        h = torch.from_numpy(synth.make_tokens(60 + n, n)).to(cuda).to(dtype)
        y = ep(h)
        ref = _expected(block, h, PATHS[path], cuda)
        torch.cuda.synchronize()
        assert torch.equal(y, ref), f"n={n}"
        hs.append(h)
    # the same batches as microbatches of one call (one count read-back)
    for h, y in zip(hs, ep.forward_many(hs)):
        ref = _expected(block, h, PATHS[path], cuda)
        torch.cuda.synchronize()
        assert torch.equal(y, ref), f"forward_many, n={h.shape[0]}"


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
            for n in (8, 96 + 32 * rank):  # ragged across ranks
                h = torch.from_numpy(synth.make_tokens(70 + 10 * rank + n, n)).to(dev).to(dtype)
                y = ep(h)
                ref = _expected(block, h, path, dev)
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
                ref = _expected(block, h, path, dev)
                torch.cuda.synchronize()
                if not torch.equal(y, ref):
                    raise AssertionError(f"rank {rank} path {path} {dtype} forward_many microbatch {j} differs")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_over_nccl_equal_the_block():
    mp.start_processes(_rank_main, args=(2, _free_port()), nprocs=2, start_method="spawn")
