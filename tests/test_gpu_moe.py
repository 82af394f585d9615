"""GPU: the whole MoE block (er_moe_block through MoeBlock) against the
oracle and the reference's own outputs.

Tolerances (relative L2 over the block output):
  * fp32 activations: 1e-3 (the hot path's stated bound); the fp32-FMA
    paths (GEMV, SIMT GEMM) are also held to 1e-4 to catch regressions;
  * bf16 activations: 1e-2 against the fp32 oracle run on the same
    bf16-rounded inputs.
Top-k expert ids are compared exactly whenever both sides route from the
same logits.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch
from conftest import golden
from helpers import gptq_oracle_weights, oracle_weights

from expertrelay_b200 import _lib, synth
from expertrelay_b200.moe import HostPipeline, MoeBlock
from expertrelay_b200.store import FMT_INT4, FMT_INT8, RecordLayout
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-3
FP32_FMA_TOL = 1e-4
BF16_TOL = 1e-2
PATHS = {"gemv": _lib.PATH_GEMV, "gemm": _lib.PATH_GEMM}
# the tensor-core path (int8 records only): int8 weights x two int8 activation slices
PATHS_INT8 = {**PATHS, "tc": _lib.PATH_TC}
TOL = {"gemv": FP32_FMA_TOL, "gemm": FP32_FMA_TOL, "tc": FP32_TOL}
# int4 records: the tensor-core path unpacks the codes in shared memory
PATHS_INT4 = PATHS_INT8


def _run(block: MoeBlock, x: np.ndarray, path: int, logits: np.ndarray | None = None, dtype=torch.float32):
    dev = block.device
    h = torch.from_numpy(x).to(dev).to(dtype)
    lg = None if logits is None else torch.from_numpy(np.ascontiguousarray(logits, np.float32)).to(dev)
    y, lo, idx, w = block.forward(h, logits=lg, path=path, return_routing=True)
    torch.cuda.synchronize()
    return y.cpu().numpy(), lo.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy()


def _mini_block(fmt: str, cuda) -> MoeBlock:
    g = golden("moe_mini")
    tag = f"mini_{fmt}"
    lay = RecordLayout(FMT_INT8, 64, 32) if fmt == "int8" else RecordLayout(FMT_INT4, 64, 32, 16)
    from expertrelay_b200.store import parse_record

    sh = parse_record(RecordLayout(FMT_INT8, 64, 48), g[f"{tag}_shared_record"])
    return MoeBlock(router=g[f"{tag}_router"], shared_gate=g[f"{tag}_shared_gate"], shared=sh, layout=lay,
                    shared_inter=48, records=g[f"{tag}_records"], top_k=4, device=cuda)


@pytest.mark.parametrize(("fmt", "path"), [("int8", p) for p in PATHS_INT8] + [("int4", p) for p in PATHS])
def test_small_block_matches_reference(cuda, fmt, path):
    g = golden("moe_mini")
    blk = _mini_block(fmt, cuda)
    x = g[f"mini_{fmt}_x"]
    y, lg, idx, w = _run(blk, x, PATHS_INT8[path])
    np.testing.assert_allclose(lg, g[f"mini_{fmt}_logits"], rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(idx, g[f"mini_{fmt}_sel"])
    assert O.rel_l2(y, g[f"mini_{fmt}_y"]) < TOL[path]


@pytest.fixture(scope="module")
def decode8(cuda):
    blk, x = synth.make_workload("decode8_int8", seed=0)
    g = golden("moe_qwen")
    digest = hashlib.sha256(np.ascontiguousarray(blk.records()).tobytes()).hexdigest().encode()
    assert digest == g["decode8_records_sha"].tobytes(), "synthetic weights differ from the fixture's"
    return blk, x, MoeBlock.from_host_block(blk, device=cuda), g


@pytest.mark.parametrize("path", list(PATHS_INT8))
def test_decode8_matches_reference(decode8, path):
    blk, x, dev, g = decode8
    y, lg, idx, w = _run(dev, x, PATHS_INT8[path])
    np.testing.assert_allclose(lg, g["decode8_logits"], rtol=1e-4, atol=1e-5)
    np.testing.assert_array_equal(idx, g["decode8_sel"])
    assert O.rel_l2(y, g["decode8_y_blocked"]) < TOL[path]
    # routing pinned to the reference's logits: ids bit-exact, same output
    y2, _, idx2, w2 = _run(dev, x, PATHS_INT8[path], logits=g["decode8_logits"])
    np.testing.assert_array_equal(idx2, g["decode8_sel"])
    np.testing.assert_allclose(w2, np.take_along_axis(O.softmax(g["decode8_logits"]), idx2, -1), rtol=1e-6)
    assert O.rel_l2(y2, g["decode8_y_blocked"]) < TOL[path]


@pytest.mark.parametrize("path", ["gemv", "tc"])
def test_decode8_bf16_activations(decode8, path):
    blk, x, dev, g = decode8
    xb = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    y, lg, idx, _ = _run(dev, x, PATHS_INT8[path], dtype=torch.bfloat16)
    ref = O.moe_block(xb, oracle_weights(blk))
    np.testing.assert_array_equal(idx, ref.selected)
    assert O.rel_l2(y, ref.y) < BF16_TOL


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("n", [65, 128, 129, 1000])
def test_router_logits_accuracy(decode8, n, dtype):
    """Batches of more than 64 tokens take the tensor-core router (tf32
    products of exact hi/lo splits: three for fp32 tokens, two for bf16 ones,
    which are exact in tf32; fp32 accumulation): the logits stay within fp32
    rounding of the float64 product, and top-k ids follow them (partial
    128-token tiles included)."""
    blk, _, dev, _ = decode8
    x = synth.make_tokens(300 + n, n)
    tdt = torch.float32
    if dtype == "bf16":
        tdt = torch.bfloat16
        x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    _, lg, idx, _ = _run(dev, x, _lib.PATH_TC, dtype=tdt)
    ref = x.astype(np.float64) @ blk.router.astype(np.float64).T
    np.testing.assert_allclose(lg, ref, rtol=1e-5, atol=2e-6)
    order = np.argsort(-ref, axis=1, kind="stable")
    srt = np.take_along_axis(ref, order, 1)
    k = blk.top_k
    clear = np.min(srt[:, :k] - srt[:, 1 : k + 1], axis=1) > 1e-5  # no near-tie inside or at the cut
    assert clear.mean() > 0.99
    np.testing.assert_array_equal(idx[clear], order[clear, :k])


@pytest.mark.parametrize("n", [1, 3, 17, 70, 300])
@pytest.mark.parametrize("path", list(PATHS_INT8))
def test_decode_shapes_against_oracle(decode8, n, path):
    blk, _, dev, _ = decode8
    if n > 70 and path == "gemv":
        pytest.skip("the weight-streaming path is for decode-sized batches")
    x = synth.make_tokens(100 + n, n)
    ow = oracle_weights(blk)
    y, lg, idx, _ = _run(dev, x, PATHS_INT8[path])
    ref = O.moe_block(x, ow, logits=lg)  # same routing decision on both sides
    np.testing.assert_array_equal(idx, ref.selected)
    assert O.rel_l2(y, ref.y) < TOL[path]


def test_edge_routing_cases(decode8):
    """Every token on the same experts (one group holds all rows, the rest
    none), exact logit ties, and an empty batch."""
    blk, _, dev, _ = decode8
    n = 12
    x = synth.make_tokens(5, n)
    ow = oracle_weights(blk)
    lg = np.full((n, 60), -3.0, dtype=np.float32)
    lg[:, [59, 0, 31, 7]] = [4.0, 3.0, 2.0, 1.0]
    for name, path in PATHS_INT8.items():
        y, _, idx, _ = _run(dev, x, path, logits=lg)
        assert (idx == [59, 0, 31, 7]).all()
        assert O.rel_l2(y, O.moe_block(x, ow, logits=lg).y) < TOL[name]
    ties = np.zeros((n, 60), dtype=np.float32)
    y, _, idx, w = _run(dev, x, _lib.PATH_GEMV, logits=ties)
    assert (idx == [0, 1, 2, 3]).all()
    ref = O.moe_block(x, ow, logits=ties, tie_rule="lower_index")
    np.testing.assert_array_equal(idx, ref.selected)
    assert O.rel_l2(y, ref.y) < FP32_FMA_TOL
    empty = dev.forward(torch.empty((0, 2048), dtype=torch.float32, device=dev.device))
    assert tuple(empty.shape) == (0, 2048)


@pytest.mark.parametrize("path", list(PATHS_INT8))
def test_captured_graph_replays_and_follows_the_expert_table(decode8, path):
    """A forward captured as a CUDA graph gives the eager result on replay,
    and re-reads the expert table: remapping two experts' records after the
    capture changes the replayed output exactly as it changes the eager one."""
    blk, x, dev, _ = decode8
    h = torch.from_numpy(x).to(dev.device)
    cap = dev.capture(8, path=PATHS_INT8[path])
    y_graph = cap(h).clone()
    y_eager = dev.forward(h, path=PATHS_INT8[path])
    torch.cuda.synchronize()
    assert torch.equal(y_graph, y_eager)
    table = dev.expert_table.clone()
    swapped = table.clone()
    swapped[[0, 1]] = table[[1, 0]]  # expert 0 now computes with expert 1's record and vice versa
    try:
        dev.set_expert_table(swapped)
        y_swap_graph = cap.replay().clone()
        y_swap_eager = dev.forward(h, path=PATHS_INT8[path])
        torch.cuda.synchronize()
        assert torch.equal(y_swap_graph, y_swap_eager)
        _, _, idx, _ = dev.forward(h, path=PATHS_INT8[path], return_routing=True)
        if bool(((idx == 0) | (idx == 1)).any()):
            assert not torch.equal(y_swap_graph, y_graph)
    finally:
        dev.set_expert_table(table)


@pytest.mark.parametrize("path", ["tc", "gemv"])
def test_host_pipeline_matches_the_graph(decode8, path):
    """HostPipeline: host batches queued back to back (the copies of
    neighbouring batches overlapping each batch's compute, two graph slots
    reused in turn) come back in their own pinned host buffers, each equal to
    the captured graph's output for that batch."""
    _, x, dev, _ = decode8
    rng = np.random.default_rng(5)
    batches = [x] + [rng.standard_normal(x.shape).astype(np.float32) for _ in range(4)]
    hs = [torch.from_numpy(b).pin_memory() for b in batches]
    ys = [torch.full(b.shape, float("nan"), dtype=torch.float32).pin_memory() for b in batches]
    pipe = HostPipeline(dev, x.shape[0], path=PATHS_INT8[path], depth=2)
    for h, y in zip(hs, ys):
        pipe.submit(h, y)
    pipe.sync()
    cap = dev.capture(x.shape[0], path=PATHS_INT8[path])
    for h, y in zip(hs, ys):
        want = cap(h.to(dev.device)).cpu()
        assert torch.equal(y, want)
    with pytest.raises(ValueError):
        pipe.submit(hs[0][:4].clone().pin_memory(), ys[0][:4].clone().pin_memory())
    with pytest.raises(ValueError):
        pipe.submit(hs[0].clone(), ys[0])  # not pinned


@pytest.mark.parametrize("path", list(PATHS_INT8))
def test_stage_events_time_an_eager_call(decode8, path):
    """Stage events passed to an eager (uncaptured) call are recorded in
    stage order, and the stages add up to the whole call."""
    _, x, dev, _ = decode8
    h = torch.from_numpy(x).to(dev.device)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(_lib.MOE_STAGES) + 1)]
    y = dev.forward(h, path=PATHS_INT8[path], stage_events=ev)
    torch.cuda.synchronize()
    stages = [ev[i].elapsed_time(ev[i + 1]) for i in range(len(_lib.MOE_STAGES))]
    assert all(s >= 0.0 for s in stages)
    assert abs(sum(stages) - ev[0].elapsed_time(ev[-1])) < 1e-2
    assert torch.equal(y, dev.forward(h, path=PATHS_INT8[path]))


@pytest.fixture(scope="module")
def gptq_block(cuda):
    blk = synth.make_block(3, fmt="gptq_asym", group=128)
    return blk, MoeBlock.from_host_block(blk, device=cuda), gptq_oracle_weights(blk)


GPTQ_CASES = [(1, "gemv"), (1, "gemm"), (8, "gemv"), (64, "gemm"), (512, "gemm"),
              (1, "tc"), (8, "tc"), (17, "tc"), (64, "tc"), (130, "tc"), (512, "tc")]


@pytest.mark.parametrize(("n", "path"), GPTQ_CASES)
def test_gptq_asym_block_against_gptq_formula(gptq_block, n, path):
    """Asymmetric GPTQ experts: the oracle uses weights dequantized from the
    raw GPTQ v1 tensors (qweight/qzeros/scales/g_idx), in float64. The
    tensor-core path (codes q - z unpacked in shared memory, exact int32 sums
    per group of 128 inputs times the group's fp16 scale) is held to the fp32
    tolerance; the fp32-FMA paths also to the tighter one."""
    blk, dev, ow = gptq_block
    x = synth.make_tokens(200 + n, n)
    y, lg, idx, _ = _run(dev, x, PATHS_INT4[path])
    exact = O.moe_block_f64(x, ow, logits=lg)
    ref32 = O.moe_block(x, ow, logits=lg)
    np.testing.assert_array_equal(idx, ref32.selected)
    assert O.rel_l2(y, exact) < FP32_TOL
    if path != "tc":
        assert O.rel_l2(y, ref32.y) < FP32_FMA_TOL


def test_gptq_asym_tc_is_the_default_and_repeats(gptq_block):
    """With the records in an arena the default path is the tensor-core one,
    and its output does not change from call to call."""
    _, dev, _ = gptq_block
    h = torch.from_numpy(synth.make_tokens(9, 40)).to(dev.device)
    y_auto = dev.forward(h, path=_lib.PATH_AUTO)
    y_tc = dev.forward(h, path=_lib.PATH_TC)
    y_again = dev.forward(h, path=_lib.PATH_TC)
    torch.cuda.synchronize()
    assert torch.equal(y_auto, y_tc) and torch.equal(y_tc, y_again)


@pytest.mark.parametrize(("group", "n"), [(128, 3), (64, 24), (32, 70)])
def test_int4_store_block_tc_groups(cuda, group, n):
    """Symmetric int4 store records (value = nibble - 8) on the tensor-core
    path at several group sizes (1, 2 and 4 groups per 128-input block) and
    token counts over one and several token tiles."""
    blk = synth.make_block(40 + group, fmt="int4", group=group, num_experts=16)
    dev = MoeBlock.from_host_block(blk, device=cuda)
    x = synth.make_tokens(group + n, n)
    y, lg, idx, _ = _run(dev, x, _lib.PATH_TC)
    ow = oracle_weights(blk)
    ref = O.moe_block(x, ow, logits=lg)
    np.testing.assert_array_equal(idx, ref.selected)
    assert O.rel_l2(y, ref.y) < FP32_TOL


def test_int4_store_block(cuda):
    """Symmetric int4 store records (value = nibble - 8, rtn_absmax7 g128)."""
    blk = synth.make_block(4, fmt="int4", group=128, num_experts=16)
    dev = MoeBlock.from_host_block(blk, device=cuda)
    x = synth.make_tokens(4, 6)
    for name, path in PATHS_INT4.items():
        y, lg, idx, _ = _run(dev, x, path)
        ref = O.moe_block(x, oracle_weights(blk), logits=lg)
        np.testing.assert_array_equal(idx, ref.selected)
        assert O.rel_l2(y, ref.y) < TOL[name]


@pytest.fixture(scope="module")
def prefill(cuda):
    blk, x = synth.make_workload("prefill4096_int8_zipf", seed=0)
    return blk, x, MoeBlock.from_host_block(blk, device=cuda), golden("moe_qwen")


@pytest.fixture(scope="module")
def prefill_oracle(prefill):
    """The oracle's block output on the reference's own router logits (the
    oracle is pinned to the reference at this size by test_oracle_full)."""
    blk, x, _, g = prefill
    return O.moe_block(x, oracle_weights(blk), logits=g["prefill_logits"])


def _sketch(y: np.ndarray) -> np.ndarray:
    # the seeded directions the fixture projects every output row on
    # (tests/golden/make_golden.py prefill_sketch_matrix)
    return y.astype(np.float64) @ np.random.default_rng(7).standard_normal((y.shape[1], 8))


@pytest.mark.parametrize("path", ["gemm", "tc"])
def test_prefill4096_zipf_against_reference(prefill, prefill_oracle, path):
    """The benched workload (4096 tokens, int8 experts, Zipf routing) routed
    from the reference's own router logits: every token's ids bit-exact, and
    all 4096 output rows within the fp32 tolerance of the oracle (rel-L2 over
    the whole output) and of the reference (rel-L2 of every row's projection
    on 8 seeded directions, and every row's norm)."""
    blk, x, dev, g = prefill
    sel = g["prefill_sel"].astype(np.int64)
    y, _, idx, w = _run(dev, x, PATHS_INT8[path], logits=g["prefill_logits"])
    np.testing.assert_array_equal(idx, sel)
    np.testing.assert_array_equal(idx, prefill_oracle.selected)
    np.testing.assert_allclose(w, prefill_oracle.weights, rtol=1e-6)
    assert O.rel_l2(y, prefill_oracle.y) < TOL[path]
    assert O.rel_l2(_sketch(y), g["prefill_y_sketch"]) < TOL[path]
    np.testing.assert_allclose(np.linalg.norm(y.astype(np.float64), axis=1), g["prefill_y_rownorm"], rtol=1e-3)
    assert O.rel_l2(y[:32], g["prefill_y_head"]) < TOL[path]
    counts = np.bincount(idx.ravel(), minlength=60)
    assert counts.max() > 8 * np.median(counts)


@pytest.mark.parametrize("path", ["gemm", "tc"])
def test_prefill4096_zipf_own_router(prefill, path):
    """The block's own fp32 router: its logits match the reference's, and
    only tokens whose k-th and (k+1)-th probabilities are too close for a
    different summation order may route differently."""
    _, x, dev, g = prefill
    y, lg, idx, _ = _run(dev, x, PATHS_INT8[path])
    np.testing.assert_allclose(lg, g["prefill_logits"], rtol=1e-4, atol=1e-5)
    same = (idx == g["prefill_sel"].astype(np.int64)).all(axis=1)
    assert same.mean() > 0.999, f"{(~same).sum()} tokens routed differently"
    np.testing.assert_allclose(np.linalg.norm(y.astype(np.float64), axis=1)[same], g["prefill_y_rownorm"][same],
                               rtol=1e-3)


def test_prefill4096_zipf_bf16_activations(prefill):
    """The benched workload with bf16 activations on the tensor-core path,
    against the fp32 oracle on the same bf16-rounded tokens and the same
    router logits (the device's, from those tokens): ids exact, rel-L2
    within the bf16 tolerance."""
    blk, x, dev, _ = prefill
    xb = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    y, lg, idx, _ = _run(dev, x, _lib.PATH_TC, dtype=torch.bfloat16)
    ref = O.moe_block(xb, oracle_weights(blk), logits=lg)
    np.testing.assert_array_equal(idx, ref.selected)
    assert O.rel_l2(y, ref.y) < BF16_TOL


@pytest.mark.parametrize("path", ["gemm", "tc"])
def test_prefill_output_repeats_bit_for_bit(prefill, path):
    """The dispatch claims expert-sorted positions with atomics, so the order
    of the rows inside one expert's range differs from call to call; every
    output element depends only on its own token's row, so the block output
    and the routing must not."""
    _, x, dev, _ = prefill
    h = torch.from_numpy(x).to(dev.device)
    y1, _, idx1, w1 = dev.forward(h, path=PATHS_INT8[path], return_routing=True)
    y1 = y1.clone()
    y2, _, idx2, w2 = dev.forward(h, path=PATHS_INT8[path], return_routing=True)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    assert torch.equal(idx1, idx2) and torch.equal(w1, w2)
