"""The oracle against the reference's own outputs (tests/golden/, made by
tests/golden/make_golden.py from ExpertRelay itself). This pins the oracle
before any GPU result is compared with it."""

from __future__ import annotations

import numpy as np
import pytest
from conftest import golden

from oracle import moe_oracle as O


@pytest.fixture(scope="module")
def q():
    return golden("quant")


def test_int8_quantizer_matches_reference(q):
    qq, s = O.quantize_rowwise_int8(q["i8_w"])
    np.testing.assert_array_equal(qq, q["i8_q"])
    np.testing.assert_array_equal(s, q["i8_s"])
    assert qq.min() >= -127 and s[7] == 0 and (qq[7] == 0).all()
    w_hat = O.dequantize_rowwise_int8(qq, s)
    assert np.all(np.abs(q["i8_w"] - w_hat) <= s[:, None] * (0.5 + 1e-6))


def test_int4_quantizers_match_reference(q):
    v, s = O.quantize_groupwise_int4(q["i4_w"], 32)
    np.testing.assert_array_equal(v, q["i4_q"])
    np.testing.assert_array_equal(s, q["i4_s"])
    v, s = O.quantize_groupwise_int4(q["i4_bump_w"], 8)
    np.testing.assert_array_equal(s, q["i4_bump_s"])
    assert float(s[0, 0]) * 7 >= q["i4_bump_w"][0, 0]
    v, s = O.quantize_groupwise_int4_gptq_grid(q["gg_w"], 16)
    np.testing.assert_array_equal(v, q["gg_q"])
    np.testing.assert_array_equal(s, q["gg_s"])
    assert (v == -8).any()


def test_pack_matches_reference(q):
    np.testing.assert_array_equal(O.pack_int4(q["pack_q"]), q["pack_p"])
    np.testing.assert_array_equal(O.unpack_int4(q["pack_p"]), q["pack_q"])
    p = q["pack_p"]
    assert (p[0, 0] & 0x0F) == q["pack_q"][0, 0] + 8 and (p[0, 0] >> 4) == q["pack_q"][0, 1] + 8


def test_gptq_formula_and_conversion_match_reference():
    g = golden("gptq")
    t = {k: g[f"sym_{k}"] for k in ("qweight", "qzeros", "scales", "g_idx", "bias")}
    np.testing.assert_array_equal(O.gptq_dequantize(t["qweight"], t["qzeros"], t["scales"], t["g_idx"]), g["sym_ref_w"])
    packed, scales = O.gptq_to_int4(*t.values(), group=16)
    np.testing.assert_array_equal(packed, g["sym_store_packed"])
    np.testing.assert_array_equal(scales, g["sym_store_scales"])
    np.testing.assert_array_equal(O.dequantize_groupwise_int4(packed, scales, 16), g["sym_ref_w"])
    a = {k: g[f"asym_{k}"] for k in ("qweight", "qzeros", "scales", "g_idx")}
    np.testing.assert_array_equal(O.gptq_dequantize(*a.values()), g["asym_ref_w"])
    k = {x: g[f"k_{x}"] for x in ("qweight", "qzeros", "scales", "g_idx")}
    np.testing.assert_array_equal(O.gptq_dequantize(*k.values()), g["k_ref_w"])


@pytest.mark.parametrize("change", ["zero", "g_idx", "bias"])
def test_gptq_conversion_refuses_like_reference(change):
    g = golden("gptq")
    t = {k: g[f"sym_{k}"].copy() for k in ("qweight", "qzeros", "scales", "g_idx", "bias")}
    if change == "zero":
        t["qzeros"] = (t["qzeros"].view(np.uint32) - np.uint32(0x11111111)).view(np.int32)  # stored 6 -> zero 7
    elif change == "g_idx":
        t["g_idx"] = np.roll(t["g_idx"], 1)
    else:
        t["bias"][3] = 0.5
    with pytest.raises(ValueError):
        O.gptq_to_int4(*t.values(), group=16)


def test_linear_kernels_match_reference():
    g = golden("linear")
    for n in (1, 3, 40):
        x = g[f"i8_x{n}"]
        y = O.int8_linear(x, g["i8_q"], g["i8_s"])
        np.testing.assert_allclose(y, g[f"i8_y{n}_blocked"], rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(y, g[f"i8_y{n}_fused"], rtol=1e-5, atol=1e-5)
        yb = O.int8_linear(x, g["i8_q"], g["i8_s"], g["i8_bias"])
        np.testing.assert_allclose(yb, g[f"i8_y{n}_bias"], rtol=1e-6, atol=1e-6)
    for n in (1, 4, 20):
        x = g[f"i4_x{n}"]
        y = O.int4_linear(x, g["i4_p"], g["i4_s"], 32)
        np.testing.assert_allclose(y, g[f"i4_y{n}_blocked"], rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(y, g[f"i4_y{n}_fused"], rtol=1e-5, atol=1e-5)


def _mini_weights(g, fmt):
    from expertrelay_b200.store import FMT_INT4, FMT_INT8, RecordLayout, parse_record

    tag = f"mini_{fmt}"
    lay = RecordLayout(FMT_INT8, 64, 32) if fmt == "int8" else RecordLayout(FMT_INT4, 64, 32, 16)
    experts = []
    for rec in g[f"{tag}_records"]:
        mats = parse_record(lay, rec)
        if fmt == "int8":
            experts.append({m: O.Int8Mat(*mats[m]) for m in mats})
        else:
            experts.append({m: O.Int4Mat(mats[m][0], mats[m][1], 16) for m in mats})
    sh = parse_record(RecordLayout(FMT_INT8, 64, 48), g[f"{tag}_shared_record"])
    return O.BlockWeights(g[f"{tag}_router"], g[f"{tag}_shared_gate"], {m: O.Int8Mat(*sh[m]) for m in sh}, experts)


@pytest.mark.parametrize("fmt", ["int8", "int4"])
def test_moe_block_matches_reference_small(fmt):
    g = golden("moe_mini")
    w = _mini_weights(g, fmt)
    out = O.moe_block(g[f"mini_{fmt}_x"], w)
    np.testing.assert_array_equal(out.selected, g[f"mini_{fmt}_sel"])
    np.testing.assert_allclose(out.logits, g[f"mini_{fmt}_logits"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(out.y, g[f"mini_{fmt}_y"], rtol=1e-5, atol=1e-6)
    exact = O.moe_block_f64(g[f"mini_{fmt}_x"], w)
    assert O.rel_l2(out.y, exact) < 1e-5


def test_top_k_tie_rules():
    probs = np.array([[0.1, 0.3, 0.3, 0.2, 0.1]], dtype=np.float32)
    assert O.top_k_lower_index(probs, 3).tolist() == [[1, 2, 3]]
    rng = np.random.default_rng(0)
    p = rng.random((200, 60)).astype(np.float32)
    np.testing.assert_array_equal(O.top_k_desc(p, 4), O.top_k_lower_index(p, 4))
