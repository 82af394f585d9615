"""GPU: the tensor-core kernels' bounded waits give up cleanly.

Every mbarrier wait in the tcgen05 kernels has a time bound; when one runs
out, the CTA raises its abort flag, the block's plan gets error bit 8, the
combine writes NaN rows and the kernel returns with the GPU context intact.
Here a test hook (er_tc_test_stall) shortens the bound to 1 ms and makes
the MMA issuer of one int8 decode kernel withhold the accumulator of its
launch's last work item. That item is the last its CTA runs, so when the
epilogue's wait runs out every copy the CTA issued has already landed: no
transfer is in flight into shared memory. The next call, with the hook
reset, must compute the normal result.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from helpers import oracle_weights

from expertrelay_b200 import _lib, synth
from expertrelay_b200.moe import MoeBlock
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

WAIT_NS = 1_000_000  # 1 ms


@pytest.fixture(scope="module")
def small_block(cuda):
    blk = synth.make_block(8, hidden=256, inter=128, shared_inter=384, num_experts=16, top_k=4)
    return blk, MoeBlock.from_host_block(blk, device=cuda)


@pytest.mark.parametrize("stall", [1, 2], ids=["gate_up", "down"])
def test_a_wait_that_runs_out_returns_an_error_and_nan_rows(small_block, cuda, stall):
    blk, mb = small_block
    x = synth.make_tokens(5, 8, blk.hidden)
    h = torch.from_numpy(x).to(cuda)
    L = _lib.lib()
    _lib.check(L.er_tc_test_stall(WAIT_NS, stall), "er_tc_test_stall")
    try:
        y = mb.forward(h, path=_lib.PATH_TC)
        bits = mb.error_bits(8, _lib.PATH_TC)
    finally:
        _lib.check(L.er_tc_test_stall(0, 0), "er_tc_test_stall")
    assert bits & 8, f"error bits {bits}: the expired wait was not reported"
    assert torch.isnan(y).all(), "rows of a failed block must be NaN"
    # the context still works: the next call computes the block
    y2, lg, idx, _ = mb.forward(h, path=_lib.PATH_TC, return_routing=True)
    assert mb.error_bits(8, _lib.PATH_TC) == 0
    ref = O.moe_block(x, oracle_weights(blk), logits=lg.cpu().numpy())
    np.testing.assert_array_equal(idx.cpu().numpy(), ref.selected)
    assert O.rel_l2(y2.cpu().numpy(), ref.y) < 1e-3
    assert torch.cuda.synchronize() is None


def test_hook_rejects_unknown_modes():
    assert _lib.lib().er_tc_test_stall(0, 3) == _lib.ER_EINVAL
