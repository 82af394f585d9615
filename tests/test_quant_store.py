"""The package's store encodings and record layouts against the reference's
bytes (tests/golden/ from ExpertRelay's own quantizers, packers, record
serializers and committed store manifests)."""

from __future__ import annotations

import json

import numpy as np
import pytest
from conftest import GOLDEN, golden

from expertrelay_b200 import quant
from expertrelay_b200.store import FMT_INT4, FMT_INT4_ZP, FMT_INT8, RecordLayout, parse_record, serialize_record
from oracle import moe_oracle as O


def test_quantizers_bit_exact():
    q = golden("quant")
    v, s = quant.int8_rowwise(q["i8_w"])
    np.testing.assert_array_equal(v, q["i8_q"])
    np.testing.assert_array_equal(s, q["i8_s"])
    v, s = quant.int4_rtn_absmax7(q["i4_w"], 32)
    np.testing.assert_array_equal(v, q["i4_q"])
    np.testing.assert_array_equal(s, q["i4_s"])
    v, s = quant.int4_rtn_absmax7(q["i4_bump_w"], 8)
    np.testing.assert_array_equal(v, q["i4_bump_q"])
    np.testing.assert_array_equal(s, q["i4_bump_s"])
    v, s = quant.int4_rtn_gptq_grid(q["gg_w"], 16)
    np.testing.assert_array_equal(v, q["gg_q"])
    np.testing.assert_array_equal(s, q["gg_s"])
    np.testing.assert_array_equal(quant.pack_nibbles(q["pack_q"]), q["pack_p"])
    np.testing.assert_array_equal(quant.unpack_nibbles(q["pack_p"]).astype(np.int16) - 8, q["pack_q"])


def test_bad_group_size_is_rejected():
    with pytest.raises(ValueError):
        quant.int4_rtn_absmax7(np.zeros((2, 30), np.float32), 8)
    with pytest.raises(ValueError):
        RecordLayout(FMT_INT4, 30, 16, 8)


def test_gptq_v1_packing_matches_the_formula():
    g = golden("gptq")
    t = {k: g[f"sym_{k}"] for k in ("qweight", "qzeros", "scales", "g_idx", "bias")}
    packed, scales, zeros = quant.gptq_to_zp_matrix(t, 16)
    assert (zeros == 8).all()
    np.testing.assert_array_equal(packed, g["sym_store_packed"])
    np.testing.assert_array_equal(quant.dequant_int4(packed, scales, 16, zeros), g["sym_ref_w"])
    # an asymmetric layer round-trips through the zero-point record exactly
    rng = np.random.default_rng(5)
    w = rng.normal(0, 0.02, (24, 256)).astype(np.float32)
    t = quant.gptq_asym_rtn(w, 128)
    ref = O.gptq_dequantize(t["qweight"], t["qzeros"], t["scales"], t["g_idx"])
    packed, scales, zeros = quant.gptq_to_zp_matrix(t, 128)
    np.testing.assert_array_equal(quant.dequant_int4(packed, scales, 128, zeros), ref)
    assert zeros.min() >= 1 and zeros.max() <= 15 and len(np.unique(zeros)) > 1
    # round to nearest: at most half a step off, nothing clipped for these weights
    step = np.repeat(scales.astype(np.float32), 128, axis=1)
    assert np.all(np.abs(w - ref) <= step * (0.5 + 1e-3))
    bad = dict(t, g_idx=np.roll(t["g_idx"], 1))
    with pytest.raises(ValueError):
        quant.gptq_to_zp_matrix(bad, 128)


def test_record_sizes_match_committed_store_manifests():
    manifests = json.loads((GOLDEN / "store_manifests.json").read_text())
    assert manifests, "no manifests recorded"
    for name, d in manifests.items():
        lay = RecordLayout.from_dict(d)
        assert lay.record_size == d["record_size"], name
        assert lay.weights_bytes == d["weights_bytes"] and lay.scales_bytes == d["scales_bytes"], name
        mine = lay.to_dict()
        for k in ("record_size", "weights_bytes", "scales_bytes", "matrices", "alignment"):
            assert mine[k] == d[k], (name, k)
    assert RecordLayout(FMT_INT8, 2048, 1408).record_size == 8_671_232
    assert RecordLayout(FMT_INT4, 2048, 1408, 128).record_size == 4_460_544


def test_records_serialize_to_reference_bytes():
    g = golden("layout")
    l8 = RecordLayout(FMT_INT8, 32, 16)
    mats8 = {m: (g[f"rec8_{m}_q"], g[f"rec8_{m}_s"]) for m in ("gate_proj", "up_proj", "down_proj")}
    np.testing.assert_array_equal(serialize_record(l8, mats8), g["rec8"])
    l4 = RecordLayout(FMT_INT4, 32, 16, 8)
    mats4 = {m: (g[f"rec4_{m}_p"], g[f"rec4_{m}_s"]) for m in ("gate_proj", "up_proj", "down_proj")}
    np.testing.assert_array_equal(serialize_record(l4, mats4), g["rec4"])
    back = parse_record(l4, g["rec4"])
    for m, (p, s) in mats4.items():
        np.testing.assert_array_equal(back[m][0], p)
        np.testing.assert_array_equal(back[m][1], s)
    assert RecordLayout.from_dict(l4.to_dict()) == l4


def test_zero_point_record_round_trip():
    rng = np.random.default_rng(2)
    lay = RecordLayout(FMT_INT4_ZP, 64, 32, 16)
    mats = {}
    for m, (r, c) in lay.matrices:
        mats[m] = (
            rng.integers(0, 256, (r, c // 2), dtype=np.uint8),
            rng.uniform(0.01, 0.1, (r, c // 16)).astype(np.float16),
            rng.integers(1, 16, (r, c // 16), dtype=np.uint8),
        )
    rec = serialize_record(lay, mats)
    assert rec.size % 4096 == 0
    back = parse_record(lay, rec)
    for m in mats:
        for a, b in zip(back[m], mats[m]):
            np.testing.assert_array_equal(a, b)
    assert RecordLayout.from_dict(lay.to_dict()) == lay
