"""GPU: er_moe_block_noalloc, the MoE-block entry point for callers that
cannot allocate device memory (a runtime whose allocator already owns all
of HBM, or an FFI host with no device allocator). Its scratch is a fixed
array inside the library instead of a caller workspace, so its output must
equal what er_moe_block computes with a workspace, call after call, and a
batch too big for the fixed scratch must be refused before any launch.

Collected last on purpose (test_zz_*), so a failure here cannot hide the
result of any other test in a run that stops at the first failure."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from expertrelay_b200 import _lib, synth
from expertrelay_b200.moe import MoeBlock
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

# the tolerance of the fp32 block tests (tests/test_gpu_moe.py FP32_FMA_TOL)
TOL = 1e-4


def _noalloc(mb: MoeBlock, h: torch.Tensor, path: int) -> torch.Tensor:
    y = torch.empty((h.shape[0], mb.hidden), dtype=torch.float32, device=h.device)
    io = _lib.MoeIO(h=h.data_ptr(), h_dtype=_lib.DTYPE_F32, n=h.shape[0], y=y.data_ptr(), path=path)
    stream = torch.cuda.current_stream(h.device).cuda_stream
    _lib.check(_lib.lib().er_moe_block_noalloc(C.byref(mb._w), C.byref(io), stream), "er_moe_block_noalloc")
    return y


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(cuda):
    block, x = synth.make_workload("decode8_int8", seed=0)
    mb = MoeBlock.from_host_block(block, device=cuda)
    # two calls in a row on different batches and paths: the second sees the
    # first one's leftovers in the shared scratch
    for tokens, path in ((x, _lib.PATH_AUTO), (synth.make_tokens(17, 40), _lib.PATH_GEMM)):
        h = torch.from_numpy(tokens).to(cuda)
        y = _noalloc(mb, h, path)
        ref = mb.forward(h, path=path)
        torch.cuda.synchronize()
        err = O.rel_l2(y.cpu().numpy(), ref.cpu().numpy())
        assert err < TOL, f"rel-L2 {err:.2e} between the two entry points"


# the fixed scratch of er_moe_block_noalloc (csrc/er_moe_noalloc.cu)
SCRATCH_BYTES = 8 << 20


def test_noalloc_refuses_batches_beyond_its_scratch(cuda):
    block = synth.make_block(2, num_experts=8)
    mb = MoeBlock.from_host_block(block, device=cuda)
    # the largest batch whose workspace fits the scratch: it runs, one more is refused
    fit = 1
    while mb.workspace_bytes(fit + 1) <= SCRATCH_BYTES:
        fit += 1
    over = fit + 1
    h = torch.zeros((over, block.hidden), dtype=torch.float32, device=cuda)
    y = torch.full((over, block.hidden), 7.0, device=cuda)
    io = _lib.MoeIO(h=h.data_ptr(), h_dtype=_lib.DTYPE_F32, n=over, y=y.data_ptr(), path=_lib.PATH_AUTO)
    rc = _lib.lib().er_moe_block_noalloc(C.byref(mb._w), C.byref(io), None)
    assert rc == _lib.ER_ENOSPACE and "fixed scratch" in _lib.last_error()
    torch.cuda.synchronize()
    assert bool((y == 7.0).all()), "nothing may be written when the batch is refused"
    ok = torch.from_numpy(synth.make_tokens(3, fit, block.hidden)).to(cuda)
    ref = mb.forward(ok)
    got = _noalloc(mb, ok, _lib.PATH_AUTO)
    torch.cuda.synchronize()
    assert O.rel_l2(got.cpu().numpy(), ref.cpu().numpy()) < TOL
    assert np.isfinite(got.cpu().numpy()).all()
