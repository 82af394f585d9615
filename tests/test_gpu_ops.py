"""GPU: the Backend-protocol ops, weight reconstruction and the router,
through the C ABI, against float64 math and the oracle (same cases as the
reference's tests/test_runtime_int8_linear.py, test_store_int4.py,
test_store_gptq.py and test_runtime_backends.py)."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch
from conftest import golden

from expertrelay_b200 import _lib, quant
from expertrelay_b200.backend import B200Backend, make_backend
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

# the reference's kernel tests compare with float64 at rtol = atol = 1e-5
RTOL = ATOL = 1e-5


@pytest.fixture(scope="module")
def be(cuda):
    return B200Backend()


def _case(n, out_dim, in_dim, seed=0):
    rng = np.random.default_rng(seed)
    q, s = quant.int8_rowwise(rng.normal(0, 0.05, (out_dim, in_dim)).astype(np.float32))
    x = rng.normal(0, 1, (n, in_dim)).astype(np.float32)
    exact = x.astype(np.float64) @ (q.astype(np.float64) * s.astype(np.float64)[:, None]).T
    return x, q, s, exact


@pytest.mark.parametrize("n", [1, 2, 3, 4, 40])
@pytest.mark.parametrize(("out_dim", "in_dim"), [(300, 96), (7, 1000), (1, 1), (1408, 2048)])
def test_int8_linear_matches_float64(be, n, out_dim, in_dim):
    x, q, s, exact = _case(n, out_dim, in_dim, seed=3)
    y = be.int8_linear(x, q, s)
    assert y.dtype == np.float32 and y.shape == (n, out_dim)
    np.testing.assert_allclose(y, exact, rtol=RTOL, atol=ATOL * max(1.0, np.sqrt(in_dim / 96)))


def test_int8_linear_bias_and_strided_input(be):
    x, q, s, exact = _case(4, 50, 64, seed=4)
    bias = np.arange(50, dtype=np.float32)
    wide = np.zeros((4, 128), dtype=np.float32)
    wide[:, ::2] = x
    np.testing.assert_allclose(be.int8_linear(wide[:, ::2], q, s, bias), exact + bias, rtol=RTOL, atol=ATOL)


def test_int8_linear_matches_reference_outputs(be):
    g = golden("linear")
    for n in (1, 3, 40):
        np.testing.assert_allclose(be.int8_linear(g[f"i8_x{n}"], g["i8_q"], g["i8_s"]), g[f"i8_y{n}_blocked"],
                                   rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(be.int8_linear(g[f"i8_x{n}"], g["i8_q"], g["i8_s"], g["i8_bias"]),
                                   g[f"i8_y{n}_bias"], rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("n", [1, 4, 5, 20])
def test_int4_linear_matches_float64(be, n):
    rng = np.random.default_rng(3)
    v, s = quant.int4_rtn_absmax7(rng.normal(0, 0.05, (300, 128)).astype(np.float32), 32)
    packed = quant.pack_nibbles(v)
    x = rng.normal(0, 1, (n, 128)).astype(np.float32)
    exact = x.astype(np.float64) @ quant.dequant_int4(packed, s, 32).astype(np.float64).T
    np.testing.assert_allclose(be.int4_linear(x, packed, s, 32), exact, rtol=RTOL, atol=ATOL)


def test_int4_linear_matches_reference_outputs(be):
    g = golden("linear")
    for n in (1, 4, 20):
        np.testing.assert_allclose(be.int4_linear(g[f"i4_x{n}"], g["i4_p"], g["i4_s"], 32), g[f"i4_y{n}_blocked"],
                                   rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("n", [1, 4, 20])
def test_int4_linear_on_gptq_weights(be, n):
    g = golden("gptq")
    t = {k: g[f"k_{k}"] for k in ("qweight", "qzeros", "scales", "g_idx", "bias")}
    packed, s = O.gptq_to_int4(*t.values(), group=32)
    x = np.random.default_rng(4).normal(0, 1, (n, 128)).astype(np.float32)
    exact = x.astype(np.float64) @ g["k_ref_w"].astype(np.float64).T
    np.testing.assert_allclose(be.int4_linear(x, packed, s, 32), exact, rtol=RTOL, atol=ATOL)


# (rows, out, in): the few-rows vector kernel, the router-shaped rows kernel,
# the tiled kernel, and an unaligned width that falls back to the tiled one
@pytest.mark.parametrize(("n", "out_dim", "in_dim"), [(4, 7, 32), (40, 60, 2048), (40, 300, 96), (1, 60, 2050)])
def test_linear_matches_float64(be, n, out_dim, in_dim):
    rng = np.random.default_rng(1)
    w = rng.normal(0, 0.1, (out_dim, in_dim)).astype(np.float32)
    x = rng.normal(0, 1, (n, in_dim)).astype(np.float32)
    tol = ATOL * max(1.0, np.sqrt(in_dim / 96))
    np.testing.assert_allclose(be.linear(x, w), x.astype(np.float64) @ w.T, rtol=RTOL, atol=tol)
    b = rng.normal(0, 1, out_dim).astype(np.float32)
    np.testing.assert_allclose(be.linear(x, w, b), x.astype(np.float64) @ w.T + b, rtol=RTOL, atol=tol)


# (queries, keys, heads, head dim): vector kernel (d % 4 == 0) and the scalar one
@pytest.mark.parametrize(("n", "k", "heads", "d"), [(3, 8, 4, 16), (1, 300, 16, 128), (5, 37, 2, 130)])
def test_attention_matches_float64(be, n, k, heads, d):
    rng = np.random.default_rng(2)
    q, keys, values = (rng.normal(0, 1, (m, heads, d)).astype(np.float32) for m in (n, k, k))
    allowed = np.arange(k)[None, :] <= (k - n + np.arange(n))[:, None]
    scores = np.einsum("qhd,khd->hqk", q.astype(np.float64), keys) / np.sqrt(d)
    scores = np.where(allowed[None], scores, -np.inf)
    probs = np.exp(scores - scores.max(-1, keepdims=True))
    probs /= probs.sum(-1, keepdims=True)
    exact = np.einsum("hqk,khd->qhd", probs, values)
    out = be.attention(q, keys, values, allowed)
    assert out.shape == (n, heads, d) and out.dtype == np.float32
    np.testing.assert_allclose(out, exact, rtol=RTOL, atol=ATOL)


def test_unknown_backend_is_rejected():
    with pytest.raises(ValueError):
        make_backend("tpu")


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def test_dequant_is_bit_exact(cuda):
    L = _lib.lib()
    rng = np.random.default_rng(7)
    q, s = quant.int8_rowwise(rng.normal(0, 0.02, (300, 96)).astype(np.float32))
    w = torch.empty((300, 96), dtype=torch.float32, device=cuda)
    # operands stay referenced until the asynchronous kernels have run
    qd, sd = _t(q, cuda), _t(s, cuda)
    _lib.check(L.er_dequant_int8(qd.data_ptr(), sd.data_ptr(), w.data_ptr(), 300, 96, None), "dq8")
    np.testing.assert_array_equal(w.cpu().numpy(), O.dequantize_rowwise_int8(q, s))
    v, s4 = quant.int4_rtn_absmax7(rng.normal(0, 0.02, (64, 256)).astype(np.float32), 32)
    p = quant.pack_nibbles(v)
    w4 = torch.empty((64, 256), dtype=torch.float32, device=cuda)
    pd, s4d = _t(p, cuda), _t(s4.view(np.uint16), cuda)
    _lib.check(L.er_dequant_int4(pd.data_ptr(), s4d.data_ptr(), None, 32, w4.data_ptr(), 64, 256, None), "dq4")
    np.testing.assert_array_equal(w4.cpu().numpy(), O.dequantize_groupwise_int4(p, s4, 32))
    # asymmetric GPTQ: bit-exact against the GPTQ formula itself
    t = quant.gptq_asym_rtn(rng.normal(0, 0.02, (48, 256)).astype(np.float32), 128)
    pk, sc, zr = quant.gptq_to_zp_matrix(t, 128)
    wz = torch.empty((48, 256), dtype=torch.float32, device=cuda)
    pkd, scd, zrd = _t(pk, cuda), _t(sc.view(np.uint16), cuda), _t(zr, cuda)
    _lib.check(L.er_dequant_int4(pkd.data_ptr(), scd.data_ptr(), zrd.data_ptr(), 128, wz.data_ptr(), 48, 256, None),
               "dqz")
    np.testing.assert_array_equal(wz.cpu().numpy(), O.gptq_dequantize(t["qweight"], t["qzeros"], t["scales"], t["g_idx"]))


def _router(logits: np.ndarray, k: int, dev):
    n, e = logits.shape
    lg = _t(logits.astype(np.float32), dev)
    idx = torch.empty((n, k), dtype=torch.int64, device=dev)
    w = torch.empty((n, k), dtype=torch.float32, device=dev)
    _lib.check(_lib.lib().er_router_topk(lg.data_ptr(), n, e, k, idx.data_ptr(), None, w.data_ptr(), None), "topk")
    torch.cuda.synchronize()
    return idx.cpu().numpy(), w.cpu().numpy()


@pytest.mark.parametrize(("n", "e", "k"), [(1, 60, 4), (1000, 60, 4), (37, 8, 2), (5, 256, 8), (3, 4, 4)])
def test_router_topk_bit_exact_on_same_logits(cuda, n, e, k):
    logits = np.random.default_rng(n + e).normal(0, 1, (n, e)).astype(np.float32)
    idx, w = _router(logits, k, cuda)
    probs = O.softmax(logits)
    np.testing.assert_array_equal(idx, O.top_k_desc(probs, k))
    np.testing.assert_allclose(w, np.take_along_axis(probs, idx, axis=-1), rtol=1e-6, atol=1e-7)


def test_router_ties_go_to_the_lower_expert_id(cuda):
    logits = np.zeros((3, 60), dtype=np.float32)  # all equal: experts 0..3
    logits[1, [7, 9, 40, 41, 50]] = 1.0  # a 5-way tie for 4 places
    logits[2, :] = np.nan
    logits[2, 10] = 2.0
    idx, w = _router(logits, 4, cuda)
    assert idx[0].tolist() == [0, 1, 2, 3]
    assert idx[1].tolist() == [7, 9, 40, 41]
    assert idx[2, 0] == 10
    np.testing.assert_allclose(w[0], 1 / 60, rtol=1e-6)
    np.testing.assert_array_equal(idx[:2], O.top_k_lower_index(logits[:2], 4))
