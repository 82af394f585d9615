"""GPU: expert-usage traces packed on the device (er_trace_pack_layer).

The device writer, fed the reference writer's inputs, must write the
reference's files byte for byte; on larger random calls (Qwen1.5-MoE-A2.7B
routing shapes, int32 ids, many layers) it must equal the oracle; and a
paged MoE stack that traces must record exactly the experts it routed to.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import golden
from golden.make_golden import TRACE_CASES, trace_inputs

from expertrelay_b200.trace import ExpertTraceWriter, read_trace
from oracle.trace_oracle import TraceOracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", range(len(TRACE_CASES)))
def test_device_writer_matches_reference_files(case, cuda, tmp_path):
    layers, experts, k, _ = TRACE_CASES[case]
    path = tmp_path / "t.ert"
    w = ExpertTraceWriter(path, num_layers=layers, num_experts=experts, top_k=k,
                          metadata={"prompt_id": f"case{case}", "model": "synthetic"}, device=cuda)
    for call in trace_inputs(case):
        w.begin(call["positions"], call["tokens"], call["phase"])
        for layer, lc in enumerate(call["layers"]):
            fate = None if lc["fate"] is None else torch.from_numpy(lc["fate"]).to(cuda)
            w.layer(layer, torch.from_numpy(lc["logits"]).to(cuda), torch.from_numpy(lc["selected"]).to(cuda),
                    torch.from_numpy(lc["weights"]).to(cuda), fate)
        w.end()
    got = path.read_bytes()
    ref = golden("trace")[f"file{case}"].tobytes()
    assert len(got) == len(ref)
    if got != ref:
        diff = np.nonzero(np.frombuffer(got, np.uint8) != np.frombuffer(ref, np.uint8))[0]
        pytest.fail(f"{len(diff)} bytes differ from the reference's file, first at {diff[:8]}")


def test_device_writer_matches_oracle_at_model_shapes(cuda, tmp_path):
    layers, experts, k = 24, 60, 4
    rng = np.random.default_rng(7)
    path = tmp_path / "t.ert"
    meta = {"prompt_id": "big"}
    w = ExpertTraceWriter(path, num_layers=layers, num_experts=experts, top_k=k, metadata=meta, device=cuda)
    o = TraceOracle(layers, experts, k, meta)
    pos = 0
    for n, phase in ((37, 0), (1, 1), (1, 1), (4, 1)):
        positions, tokens = np.arange(pos, pos + n), rng.integers(0, 151936, n)
        pos += n
        w.begin(positions, tokens, phase)
        o.begin(positions, tokens, phase)
        for layer in range(layers):
            logits = rng.normal(0, 4, (n, experts)).astype(np.float32)
            sel = np.argsort(-logits, axis=1, kind="stable")[:, :k]
            wts = rng.random((n, k)).astype(np.float32)
            fate = rng.normal(0, 4, (n, experts)).astype(np.float32) if layer + 1 < layers else None
            w.layer(layer, torch.from_numpy(logits).to(cuda), torch.from_numpy(sel.astype(np.int32)).to(cuda),
                    torch.from_numpy(wts).to(cuda), None if fate is None else torch.from_numpy(fate).to(cuda))
            o.layer(layer, logits, sel, wts, fate)
        w.end()
        o.end()
    assert path.read_bytes() == bytes(o.data)
    header, rec = read_trace(path)
    assert len(rec) == (37 + 1 + 1 + 4) * layers


def test_paged_stack_trace_records_its_routing(cuda, tmp_path):
    from expertrelay_b200 import _lib, synth
    from expertrelay_b200.cache import HbmExpertCache, HostRecords
    from expertrelay_b200.paged import PagedMoeStack

    shape = {"hidden": 256, "inter": 128, "shared_inter": 384, "num_experts": 16, "top_k": 4}
    blocks = [synth.make_block(80 + layer, **shape) for layer in range(3)]
    source = HostRecords.from_blocks(blocks)
    cache = HbmExpertCache(source, capacity_bytes=24 * source.layout.record_size)
    stack = PagedMoeStack(blocks, cache)
    path = tmp_path / "t.ert"
    w = ExpertTraceWriter(path, num_layers=3, num_experts=16, top_k=4, metadata={"prompt_id": "stack"}, device=cuda)
    x = torch.from_numpy(synth.make_tokens(3, 5, 256)).to(cuda)
    routed = []
    w.begin(np.arange(5), np.arange(100, 105), 0)
    h = x
    for layer in range(3):
        y, idx = stack.moe(layer, h, _lib.PATH_AUTO, trace=w, return_routing=True)
        routed.append(idx.cpu().numpy())
        h = h + y
    w.end()
    _, rec = read_trace(path)
    for layer in range(3):
        np.testing.assert_array_equal(rec["experts"][rec["layer"] == layer], routed[layer])
    # the Fate prediction is recorded from layer 1 on
    assert np.all(rec["fate_experts"][rec["layer"] == 0] == 255)
    assert np.all(rec["fate_experts"][rec["layer"] > 0] < 16)
