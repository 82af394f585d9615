"""Expert-usage trace format (runtime/expert_trace.py), on the CPU: the
oracle reproduces the reference writer's files byte for byte, the reader
accepts them and rejects foreign and truncated files like the reference's,
and the library's record size agrees with the record layout."""

from __future__ import annotations

import numpy as np
import pytest
from conftest import golden
from golden.make_golden import TRACE_CASES, trace_inputs

from oracle.trace_oracle import TraceOracle
from oracle.trace_oracle import record_dtype as oracle_dtype


def _oracle_file(case: int) -> bytes:
    layers, experts, k, _ = TRACE_CASES[case]
    o = TraceOracle(layers, experts, k, {"prompt_id": f"case{case}", "model": "synthetic"})
    for call in trace_inputs(case):
        o.begin(call["positions"], call["tokens"], call["phase"])
        for layer, lc in enumerate(call["layers"]):
            o.layer(layer, lc["logits"], lc["selected"], lc["weights"], lc["fate"])
        o.end()
    return bytes(o.data)


@pytest.mark.parametrize("case", range(len(TRACE_CASES)))
def test_oracle_matches_reference_files(case):
    ref = golden("trace")[f"file{case}"].tobytes()
    assert _oracle_file(case) == ref


@pytest.mark.parametrize("case", range(len(TRACE_CASES)))
def test_reader_on_reference_files(case, tmp_path):
    from expertrelay_b200.trace import NO_EXPERT, PHASE_DECODE, PHASE_PREFILL, read_trace, record_dtype

    layers, experts, k, n0 = TRACE_CASES[case]
    path = tmp_path / "t.ert"
    path.write_bytes(golden("trace")[f"file{case}"].tobytes())
    header, rec = read_trace(path)
    assert header["num_layers"] == layers and header["num_experts"] == experts and header["top_k"] == k
    assert header["prompt_id"] == f"case{case}" and header["record_itemsize"] == rec.dtype.itemsize
    assert rec.dtype == record_dtype(experts, k) == oracle_dtype(experts, k)
    assert len(rec) == (n0 + 2) * layers
    assert set(rec["phase"][rec["position"] < n0]) == {PHASE_PREFILL}
    assert set(rec["phase"][rec["position"] >= n0]) == {PHASE_DECODE}
    # no Fate prediction at a call's first layer
    assert np.all(rec["fate_experts"][rec["layer"] == 0] == NO_EXPERT)
    assert np.all(rec["fate_experts"][rec["layer"] > 0] < experts)
    # previous-token experts chain across calls; none before the first token
    for layer in range(layers):
        rows = rec[rec["layer"] == layer]
        assert np.all(rows["prev_token_experts"][0] == NO_EXPERT)
        np.testing.assert_array_equal(rows["prev_token_experts"][1:], rows["experts"][:-1])
    assert np.isinf(rec["logits"][0, 0])  # 70000 overflows float16, as in the reference


def test_reader_rejects_truncated_and_foreign_files(tmp_path):
    from expertrelay_b200.trace import read_trace

    path = tmp_path / "t.ert"
    path.write_bytes(golden("trace")["file0"].tobytes()[:-3])
    with pytest.raises(ValueError, match="truncated"):
        read_trace(path)
    path.write_bytes(b"NOTATRACE" + b"\0" * 20)
    with pytest.raises(ValueError, match="magic"):
        read_trace(path)


def test_record_size_from_the_library():
    from expertrelay_b200 import _lib
    from expertrelay_b200.trace import record_dtype

    for experts, k in ((8, 2), (60, 4), (64, 8), (254, 1)):
        assert _lib.lib().er_trace_record_bytes(experts, k) == record_dtype(experts, k).itemsize
    assert _lib.lib().er_trace_record_bytes(255, 4) == 0  # u8 ids stop at 254
    assert _lib.lib().er_trace_record_bytes(60, 9) == 0
    with pytest.raises(ValueError, match="u8 expert ids"):
        record_dtype(255, 4)
