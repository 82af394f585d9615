"""CPU oracle for the MoE-block hot path. TEST INFRASTRUCTURE ONLY.

This module restates, in plain numpy, the arithmetic of ExpertRelay's
`QwenMoe._moe` (src/expertrelay/runtime/qwen_moe.py:293-359) and of the
kernels and formats it calls. It is the checker the CUDA path is compared
against; nothing in `expertrelay_b200/` imports it. Only `tests/`,
`__graft_entry__.smoke()` and `bench.py`'s CPU-baseline legs use it.

Parity pinning: every function here is checked against golden vectors
produced by running the reference itself (tests/golden/make_golden.py ->
tests/golden/*.npz, checked by tests/test_oracle_golden.py).

Conventions follow the reference exactly:
  * activations and accumulation are float32 (numpy BLAS sgemm);
  * int8 weights: per-output-row float32 scale, applied to the output;
  * int4 weights: two codes per byte, even input column in the low nibble,
    value = nibble - zero (zero = 8 for the store's symmetric encoding),
    times a float16 group scale along the input dimension;
  * router: softmax over all experts, top-k largest first, no
    renormalisation (norm_topk_prob is False for Qwen1.5-MoE-A2.7B);
  * experts run in ascending id, each on all its tokens, and their weighted
    outputs are accumulated into the routed sum in that order;
  * the shared expert is gated by sigmoid(h @ w_gate^T).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

# ----------------------------------------------------------------------------
# elementwise pieces (runtime/qwen_moe.py:149-166)
# ----------------------------------------------------------------------------


def silu(x: np.ndarray) -> np.ndarray:
    """x / (1 + e^-x) in the input's dtype (runtime/qwen_moe.py:149-150)."""
    return x / (1.0 + np.exp(-x))


def sigmoid(x: np.ndarray) -> np.ndarray:
    """1 / (1 + e^-x) (runtime/qwen_moe.py:153-154)."""
    return 1.0 / (1.0 + np.exp(-x))


def softmax(x: np.ndarray) -> np.ndarray:
    """Row softmax with the row max subtracted first (runtime/qwen_moe.py:157-159)."""
    shifted = x - np.max(x, axis=-1, keepdims=True)
    e = np.exp(shifted)
    return e / np.sum(e, axis=-1, keepdims=True)


def top_k_desc(probs: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest entries per row, largest first
    (runtime/qwen_moe.py:162-166): a partial selection of the k largest, then
    a stable sort of those k by descending value. With exact ties at the
    boundary the partial selection decides membership; see
    `top_k_lower_index` for the deterministic rule the CUDA path uses."""
    cand = np.argpartition(-probs, k - 1, axis=-1)[:, :k]
    vals = np.take_along_axis(probs, cand, axis=-1)
    order = np.argsort(-vals, axis=-1, kind="stable")
    return np.take_along_axis(cand, order, axis=-1)


def top_k_lower_index(values: np.ndarray, k: int) -> np.ndarray:
    """Top-k largest first with exact ties broken by the lower index. Equal
    to `top_k_desc` whenever the k-th and (k+1)-th values differ and the top
    k are distinct, which holds for continuous seeded data."""
    n, e = values.shape
    idx = np.broadcast_to(np.arange(e), (n, e))
    # lexsort: last key is primary -> sort by -value, then by index
    order = np.lexsort((idx, -values), axis=-1)
    return order[:, :k]


# ----------------------------------------------------------------------------
# weight formats (store/quantize.py, store/int4.py, store/gptq.py,
# bench/gptq_conversion_check.py)
# ----------------------------------------------------------------------------

INT8_MAX = 127
INT4_MAX = 7
GPTQ_MAXQ = 15
GPTQ_ZERO = 8


def quantize_rowwise_int8(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Symmetric per-row absmax int8 (store/quantize.py:34-42):
    scale = max|W_r| / 127 in float32, Q = clip(rint(W / scale), -127, 127);
    an all-zero row keeps scale 0 and divides by 1."""
    w = np.asarray(w, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError(f"expected a 2-D weight matrix, got shape {w.shape}")
    scale = (np.max(np.abs(w), axis=1) / INT8_MAX).astype(np.float32)
    div = np.where(scale > 0, scale, np.float32(1.0))
    q = np.clip(np.rint(w / div[:, None]), -INT8_MAX, INT8_MAX).astype(np.int8)
    return q, scale


def dequantize_rowwise_int8(q: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """q * scale_row in float32 (store/quantize.py:45-46)."""
    return q.astype(np.float32) * scales.astype(np.float32)[:, None]


def quantize_groupwise_int4(w: np.ndarray, group: int) -> tuple[np.ndarray, np.ndarray]:
    """Symmetric RTN on -7..7 with float16 group scales (store/int4.py:89-106).
    The float16 scale is raised one ulp at a time until 7*scale covers the
    group's absmax, then values are rounded with the stored scale."""
    w = np.asarray(w, dtype=np.float32)
    rows, cols = w.shape
    if cols % group or group % 2:
        raise ValueError(f"{cols} columns don't split into groups of {group} (even)")
    g = w.reshape(rows, cols // group, group)
    absmax = np.max(np.abs(g), axis=2)
    s = (absmax / INT4_MAX).astype(np.float16)
    short = s.astype(np.float32) * INT4_MAX < absmax
    while short.any():
        s[short] = np.nextafter(s[short], np.float16(np.inf))
        short = s.astype(np.float32) * INT4_MAX < absmax
    div = np.where(s > 0, s.astype(np.float32), np.float32(1.0))
    q = np.clip(np.rint(g / div[:, :, None]), -INT4_MAX, INT4_MAX).astype(np.int8)
    return q.reshape(rows, cols), s


def quantize_groupwise_int4_gptq_grid(w: np.ndarray, group: int) -> tuple[np.ndarray, np.ndarray]:
    """RTN on GPTQ's symmetric 4-bit grid (store/int4.py:109-124): per group
    xmax = max(|min(w,0)|, max(w,0)); xmin = -xmax if the group has a
    negative weight else 0; an all-zero group uses (-1, 1); scale =
    (xmax - xmin) / 15 stored in float16; value = clip(rint(w/scale)+8, 0, 15) - 8."""
    w = np.asarray(w, dtype=np.float32)
    rows, cols = w.shape
    if cols % group or group % 2:
        raise ValueError(f"{cols} columns don't split into groups of {group} (even)")
    g = w.reshape(rows, cols // group, group)
    lo = np.minimum(np.min(g, axis=2), 0)
    hi = np.maximum(np.maximum(np.max(g, axis=2), 0), np.abs(lo))
    lo = np.where(lo < 0, -hi, lo)
    empty = (lo == 0) & (hi == 0)
    lo = np.where(empty, -1, lo)
    hi = np.where(empty, 1, hi)
    s = ((hi - lo) / GPTQ_MAXQ).astype(np.float16)
    codes = np.clip(np.rint(g / s.astype(np.float32)[:, :, None]) + GPTQ_ZERO, 0, GPTQ_MAXQ)
    return (codes - GPTQ_ZERO).astype(np.int8).reshape(rows, cols), s


def pack_int4(q: np.ndarray) -> np.ndarray:
    """Values -8..7 -> nibbles value+8, even column low (store/int4.py:127-130)."""
    u = (q.astype(np.int16) + 8).astype(np.uint8)
    return (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    """Inverse of pack_int4 (store/int4.py:133-139)."""
    rows, half = packed.shape
    q = np.empty((rows, 2 * half), dtype=np.int8)
    q[:, 0::2] = (packed & 0x0F).astype(np.int8) - 8
    q[:, 1::2] = (packed >> 4).astype(np.int8) - 8
    return q


def dequantize_groupwise_int4(packed: np.ndarray, scales: np.ndarray, group: int) -> np.ndarray:
    """(nibble - 8) * float32(scale of the column's group) (store/int4.py:142-144)."""
    q = unpack_int4(packed).astype(np.float32)
    return q * np.repeat(scales.astype(np.float32), group, axis=1)


def gptq_dequantize(qweight: np.ndarray, qzeros: np.ndarray, scales: np.ndarray, g_idx: np.ndarray) -> np.ndarray:
    """The GPTQ v1 formula, general form (bench/gptq_conversion_check.py:42-55):
    W[o, i] = (code[i, o] - (stored_zero[g_idx[i], o] + 1)) * scales[g_idx[i], o]
    with 8 codes per int32, lowest bits first; qweight [I/8, O] packs along the
    input dim, qzeros [I/G, O/8] along the output dim. Returns float32 [O, I]."""
    qw = np.ascontiguousarray(qweight).view(np.uint32)
    qz = np.ascontiguousarray(qzeros).view(np.uint32)
    in8, out = qw.shape
    codes = np.empty((in8 * 8, out), dtype=np.int32)
    for b in range(8):
        codes[b::8] = ((qw >> np.uint32(4 * b)) & 0xF).astype(np.int32)
    groups, out8 = qz.shape
    zeros = np.empty((groups, out8 * 8), dtype=np.int32)
    for b in range(8):
        zeros[:, b::8] = ((qz >> np.uint32(4 * b)) & 0xF).astype(np.int32) + 1
    gi = np.asarray(g_idx, dtype=np.int64)
    w = (codes - zeros[gi]).astype(np.float32) * scales[gi].astype(np.float32)
    return np.ascontiguousarray(w.T)


def gptq_to_int4(qweight, qzeros, scales, g_idx, bias, group: int) -> tuple[np.ndarray, np.ndarray]:
    """Lossless GPTQ v1 -> store int4 conversion, refusing what the store
    encoding can't hold (store/gptq.py:51-74): zero points other than 8, a
    g_idx other than i // group, a non-zero bias."""
    qw = np.ascontiguousarray(qweight).view(np.uint32)
    qz = np.ascontiguousarray(qzeros).view(np.uint32)
    in_dim, out_dim = qw.shape[0] * 8, qw.shape[1]
    if qz.shape != (in_dim // group, out_dim // 8) or scales.shape != (in_dim // group, out_dim):
        raise ValueError(f"shapes don't match group size {group}: {qz.shape}, {scales.shape}")
    if not np.array_equal(np.asarray(g_idx), np.arange(in_dim) // group):
        raise ValueError("g_idx is not i // group (desc_act?): not supported")
    stored = np.stack([(qz >> np.uint32(4 * b)) & 0xF for b in range(8)], axis=-1).reshape(qz.shape[0], -1)
    if not (stored == GPTQ_ZERO - 1).all():
        raise ValueError(f"zero points {np.unique(stored) + 1} are not all {GPTQ_ZERO}")
    if bias is not None and np.any(bias):
        raise ValueError("non-zero bias: not supported")
    codes = np.stack([(qw >> np.uint32(4 * b)) & 0xF for b in range(8)], axis=1).reshape(in_dim, out_dim).T
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    return np.ascontiguousarray(packed), np.ascontiguousarray(scales.T, dtype=np.float16)


# ----------------------------------------------------------------------------
# linear kernels (runtime/int8_linear.py, runtime/int4_linear.py,
# runtime/backends.py:86-88)
# ----------------------------------------------------------------------------

BLOCK_ROWS_DECODE = 128  # runtime/int8_linear.py:40
BLOCK_ROWS_PREFILL = 512  # runtime/int8_linear.py:41
DECODE_MAX_ROWS = 4  # runtime/int8_linear.py:42


def _block_rows(n: int) -> int:
    return BLOCK_ROWS_DECODE if n <= DECODE_MAX_ROWS else BLOCK_ROWS_PREFILL


def linear(x: np.ndarray, w: np.ndarray, bias: np.ndarray | None = None) -> np.ndarray:
    """x @ W^T (+ bias), float32 weights (runtime/backends.py:86-88)."""
    y = x @ w.T
    return y + bias if bias is not None else y


def int8_linear(x: np.ndarray, q: np.ndarray, scales: np.ndarray, bias: np.ndarray | None = None) -> np.ndarray:
    """The reference's "blocked" int8 kernel (runtime/int8_linear.py:129-138):
    convert a block of weight rows to float32, multiply, then scale the whole
    output by the per-row scales and add the bias."""
    n = x.shape[0]
    rows, cols = q.shape
    out = np.empty((n, rows), dtype=np.float32)
    step = _block_rows(n)
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        wblk = q[r0:r1].astype(np.float32)
        np.matmul(x, wblk.T, out=out[:, r0:r1])
    out *= scales
    if bias is not None:
        out += bias
    return out


def int4_linear(
    x: np.ndarray,
    packed: np.ndarray,
    scales: np.ndarray,
    group: int,
    bias: np.ndarray | None = None,
    zeros: np.ndarray | None = None,
) -> np.ndarray:
    """The reference's "blocked" int4 kernel (runtime/int4_linear.py:110-119):
    unpack a block of rows to float32 (nibble - 8), multiply each group by its
    float16 scale (as float32), then one matmul. `zeros` [out, in/group]
    (values 0..16) generalises the fixed 8 to GPTQ's asymmetric zero points;
    None means the store's symmetric encoding."""
    n = x.shape[0]
    rows, half = packed.shape
    cols = 2 * half
    s32 = scales.astype(np.float32)
    out = np.empty((n, rows), dtype=np.float32)
    step = _block_rows(n)
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        p = packed[r0:r1]
        wblk = np.empty((r1 - r0, cols), dtype=np.float32)
        wblk[:, 0::2] = (p & 0x0F).astype(np.float32)
        wblk[:, 1::2] = (p >> 4).astype(np.float32)
        if zeros is None:
            wblk -= 8.0
        else:
            wblk -= np.repeat(zeros[r0:r1].astype(np.float32), group, axis=1)
        wblk.reshape(r1 - r0, cols // group, group)[...] *= s32[r0:r1, :, None]
        np.matmul(x, wblk.T, out=out[:, r0:r1])
    if bias is not None:
        out += bias
    return out


# ----------------------------------------------------------------------------
# the MoE block (runtime/qwen_moe.py:293-359)
# ----------------------------------------------------------------------------


@dataclass
class Int8Mat:
    """int8 [out, in] + float32 [out] (runtime/weights.py:51-66)."""

    q: np.ndarray
    scales: np.ndarray


@dataclass
class Int4Mat:
    """packed uint8 [out, in/2] + float16 [out, in/G] (runtime/weights.py:69-80);
    `zeros` (uint8 [out, in/G], values 0..16) only for asymmetric GPTQ."""

    packed: np.ndarray
    scales: np.ndarray
    group: int
    zeros: np.ndarray | None = None


@dataclass
class BlockWeights:
    """One MoE layer's weights, named after the reference's tensors:
    router = mlp.gate.weight [E, H] f32; shared_gate = mlp.shared_expert_gate.weight
    [1, H] f32; shared = mlp.shared_expert.{gate,up,down}_proj (int8);
    experts[e] = {"gate_proj", "up_proj", "down_proj"} as Int8Mat or Int4Mat."""

    router: np.ndarray
    shared_gate: np.ndarray
    shared: dict[str, Int8Mat]
    experts: list[dict[str, Int8Mat | Int4Mat]]
    top_k: int = 4
    norm_topk_prob: bool = False


@dataclass
class BlockOutputs:
    y: np.ndarray
    logits: np.ndarray
    probs: np.ndarray
    selected: np.ndarray
    weights: np.ndarray
    routed: np.ndarray
    shared: np.ndarray
    gate: np.ndarray
    unique_experts: list[int] = field(default_factory=list)


def _mat_linear(m: Int8Mat | Int4Mat, x: np.ndarray) -> np.ndarray:
    """runtime/qwen_moe.py:261-264: int4 matrices go to int4_linear, else int8_linear."""
    if isinstance(m, Int4Mat):
        return int4_linear(x, m.packed, m.scales, m.group, zeros=m.zeros)
    return int8_linear(x, m.q, m.scales)


def moe_block(
    h: np.ndarray, w: BlockWeights, logits: np.ndarray | None = None, tie_rule: str = "reference"
) -> BlockOutputs:
    """`QwenMoe._moe` (runtime/qwen_moe.py:293-359) over in-memory weights.
    `logits`, when given, replaces the router product (line 303) so the
    routing decision can be pinned to the logits another implementation
    computed; everything after it is unchanged. tie_rule "lower_index"
    replaces the reference's partial selection by the deterministic rule
    (exact ties to the lower expert id); the two agree unless probabilities
    tie exactly."""
    h = np.asarray(h, dtype=np.float32)
    n, hidden = h.shape
    if logits is None:
        logits = linear(h, w.router)  # qwen_moe.py:303
    logits = np.asarray(logits, dtype=np.float32)
    probs = softmax(logits)  # :304
    if tie_rule == "reference":
        selected = top_k_desc(probs, w.top_k)  # :305
    else:
        selected = top_k_lower_index(logits, w.top_k)
    weights = np.take_along_axis(probs, selected, axis=-1)  # :306
    if w.norm_topk_prob:  # :307-308
        weights = weights / weights.sum(axis=-1, keepdims=True)

    routed = np.zeros((n, hidden), dtype=np.float32)  # :340
    uniq = [int(e) for e in np.unique(selected)]
    for e in uniq:  # :341, ascending expert id
        tok, slot = np.nonzero(selected == e)  # :342
        mats = w.experts[e]
        x = h[tok]
        act = silu(_mat_linear(mats["gate_proj"], x)) * _mat_linear(mats["up_proj"], x)
        y = _mat_linear(mats["down_proj"], act)  # :345-348
        np.add.at(routed, tok, y * weights[tok, slot][:, None])  # :349

    sh = w.shared  # :353-357
    shared = int8_linear(
        silu(int8_linear(h, sh["gate_proj"].q, sh["gate_proj"].scales))
        * int8_linear(h, sh["up_proj"].q, sh["up_proj"].scales),
        sh["down_proj"].q,
        sh["down_proj"].scales,
    )
    gate = sigmoid(linear(h, w.shared_gate))  # :358
    y = routed + gate * shared  # :359
    return BlockOutputs(y, logits, probs, selected, weights, routed, shared, gate, uniq)


def moe_block_f64(h: np.ndarray, w: BlockWeights, logits: np.ndarray | None = None) -> np.ndarray:
    """The same block in float64 on the exactly dequantized weights: the
    reference arithmetic without float32 rounding. Used for the asymmetric
    GPTQ case (which the reference's own path refuses, store/gptq.py:67-69)
    and to measure how far the float32 oracle itself is from exact."""
    h64 = np.asarray(h, dtype=np.float64)
    if logits is None:
        logits = h64 @ w.router.astype(np.float64).T
    logits = np.asarray(logits, dtype=np.float64)
    probs = softmax(logits)
    selected = top_k_desc(probs, w.top_k)
    weights = np.take_along_axis(probs, selected, axis=-1)

    def dq(m):
        if isinstance(m, Int4Mat):
            if m.zeros is None:
                return dequantize_groupwise_int4(m.packed, m.scales, m.group).astype(np.float64)
            codes = np.empty((m.packed.shape[0], 2 * m.packed.shape[1]), dtype=np.float64)
            codes[:, 0::2] = m.packed & 0x0F
            codes[:, 1::2] = m.packed >> 4
            z = np.repeat(m.zeros.astype(np.float64), m.group, axis=1)
            s = np.repeat(m.scales.astype(np.float64), m.group, axis=1)
            return (codes - z) * s
        return m.q.astype(np.float64) * m.scales.astype(np.float64)[:, None]

    routed = np.zeros_like(h64)
    for e in np.unique(selected):
        tok, slot = np.nonzero(selected == e)
        mats = w.experts[int(e)]
        x = h64[tok]
        act = silu(x @ dq(mats["gate_proj"]).T) * (x @ dq(mats["up_proj"]).T)
        y = act @ dq(mats["down_proj"]).T
        np.add.at(routed, tok, y * weights[tok, slot][:, None])
    sh = w.shared
    shared = (silu(h64 @ dq(sh["gate_proj"]).T) * (h64 @ dq(sh["up_proj"]).T)) @ dq(sh["down_proj"]).T
    gate = sigmoid(h64 @ w.shared_gate.astype(np.float64).T)
    return routed + gate * shared


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    """||a - b||_2 / ||b||_2 over all elements, in float64."""
    a64, b64 = np.asarray(a, np.float64), np.asarray(b, np.float64)
    den = np.linalg.norm(b64)
    return float(np.linalg.norm(a64 - b64) / den) if den > 0 else float(np.linalg.norm(a64))
