"""Weight encodings of the expert store, host side (numpy).

These write exactly the bytes the reference's store tools write, so a store
built by the reference loads here unchanged and vice versa:

  int8     store/quantize.py:34-42   per-row absmax / 127 (float32 scale),
                                     round half to even, clip to +-127
  int4     store/int4.py:89-106      symmetric RTN on -7..7, float16 group
                                     scale raised ulp by ulp until 7*scale
                                     covers the group absmax
  gptq     store/int4.py:109-124     RTN on GPTQ's symmetric grid (-8..7)
  packing  store/int4.py:127-139     two codes per byte, value + 8, even
                                     input column in the low nibble
  GPTQ v1  store/gptq.py:9-29        qweight [I/8, O] / qzeros [I/G, O/8] int32
                                     (8 codes per word, lowest bits first,
                                     zeros stored minus one) + scales [I/G, O]

plus one encoding the reference store cannot hold (store/gptq.py:67-69
refuses it): asymmetric 4-bit RTN with a zero point per group, produced as
GPTQ v1 tensors and converted losslessly to the ER_FMT_INT4_ZP record.
"""

from __future__ import annotations

import numpy as np

I8_LIMIT = 127
I4_LIMIT = 7
GPTQ_LEVELS = 15
GPTQ_SYM_ZERO = 8


def int8_rowwise(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """[rows, cols] -> (int8 codes, float32 scales [rows])."""
    w = np.asarray(w, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError(f"expected a 2-D weight matrix, got shape {w.shape}")
    amax = np.abs(w).max(axis=1)
    scales = (amax / I8_LIMIT).astype(np.float32)
    safe = scales.copy()
    safe[safe == 0] = 1.0
    codes = np.rint(w / safe[:, None])
    np.clip(codes, -I8_LIMIT, I8_LIMIT, out=codes)
    return codes.astype(np.int8), scales


def _groups(w: np.ndarray, group: int) -> np.ndarray:
    w = np.asarray(w, dtype=np.float32)
    rows, cols = w.shape
    if group <= 0 or group % 2 or cols % group:
        raise ValueError(f"{cols} columns don't split into groups of {group} (even)")
    return w.reshape(rows, cols // group, group)


def int4_rtn_absmax7(w: np.ndarray, group: int) -> tuple[np.ndarray, np.ndarray]:
    """[rows, cols] -> (int8 values -7..7, float16 scales [rows, cols/group])."""
    g = _groups(w, group)
    amax = np.abs(g).max(axis=2)
    scales = (amax / I4_LIMIT).astype(np.float16)
    while True:  # never let float16 rounding shrink a scale into clipping
        low = scales.astype(np.float32) * I4_LIMIT < amax
        if not low.any():
            break
        scales[low] = np.nextafter(scales[low], np.float16(np.inf))
    safe = scales.astype(np.float32)
    safe[safe == 0] = 1.0
    vals = np.clip(np.rint(g / safe[..., None]), -I4_LIMIT, I4_LIMIT)
    return vals.astype(np.int8).reshape(w.shape), scales


def int4_rtn_gptq_grid(w: np.ndarray, group: int) -> tuple[np.ndarray, np.ndarray]:
    """RTN on GPTQ's symmetric 4-bit grid: values -8..7, float16 scales."""
    g = _groups(w, group)
    neg = np.minimum(g.min(axis=2), 0)
    top = np.maximum(np.maximum(g.max(axis=2), 0), -neg)
    bottom = np.where(neg < 0, -top, neg)
    none = (bottom == 0) & (top == 0)
    bottom[none], top[none] = -1, 1
    scales = ((top - bottom) / GPTQ_LEVELS).astype(np.float16)
    codes = np.clip(np.rint(g / scales.astype(np.float32)[..., None]) + GPTQ_SYM_ZERO, 0, GPTQ_LEVELS)
    return (codes - GPTQ_SYM_ZERO).astype(np.int8).reshape(w.shape), scales


def pack_nibbles(values: np.ndarray, offset: int = 8) -> np.ndarray:
    """int values (code - offset) [rows, cols] -> uint8 [rows, cols/2], even column low."""
    u = (np.asarray(values).astype(np.int16) + offset).astype(np.uint8)
    return (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)


def unpack_nibbles(packed: np.ndarray) -> np.ndarray:
    """uint8 [rows, half] -> raw codes 0..15 [rows, 2*half] (uint8)."""
    rows, half = packed.shape
    codes = np.empty((rows, 2 * half), dtype=np.uint8)
    codes[:, 0::2] = packed & 0x0F
    codes[:, 1::2] = packed >> 4
    return codes


def dequant_int8(q: np.ndarray, scales: np.ndarray) -> np.ndarray:
    return q.astype(np.float32) * scales.astype(np.float32)[:, None]


def dequant_int4(packed: np.ndarray, scales: np.ndarray, group: int, zeros: np.ndarray | None = None) -> np.ndarray:
    """(code - zero) * float32(scale); zero = 8 for the store's symmetric encoding."""
    codes = unpack_nibbles(packed).astype(np.float32)
    zero = np.float32(8.0) if zeros is None else np.repeat(zeros.astype(np.float32), group, axis=1)
    return (codes - zero) * np.repeat(scales.astype(np.float32), group, axis=1)


# ---- GPTQ v1 tensors -------------------------------------------------------


def pack_int32_nibbles(codes: np.ndarray, axis: int) -> np.ndarray:
    """uint codes 0..15 -> int32 with 8 codes per word along `axis`, the first
    in the lowest 4 bits (AutoGPTQ v1 packing)."""
    c = np.moveaxis(np.asarray(codes, dtype=np.uint32), axis, 0)
    if c.shape[0] % 8:
        raise ValueError(f"axis length {c.shape[0]} is not a multiple of 8")
    c = c.reshape(c.shape[0] // 8, 8, *c.shape[1:])
    word = np.zeros((c.shape[0], *c.shape[2:]), dtype=np.uint32)
    for b in range(8):
        word |= c[:, b] << np.uint32(4 * b)
    return np.moveaxis(word, 0, axis).view(np.int32)


def unpack_int32_nibbles(packed: np.ndarray, axis: int) -> np.ndarray:
    """Inverse of pack_int32_nibbles -> uint8 codes, 8x longer along `axis`."""
    u = np.moveaxis(np.ascontiguousarray(packed).view(np.uint32), axis, 0)
    out = np.empty((u.shape[0], 8, *u.shape[1:]), dtype=np.uint8)
    for b in range(8):
        out[:, b] = (u >> np.uint32(4 * b)) & 0xF
    return np.moveaxis(out.reshape(u.shape[0] * 8, *u.shape[1:]), 0, axis)


def gptq_asym_rtn(w: np.ndarray, group: int) -> dict[str, np.ndarray]:
    """Asymmetric 4-bit round-to-nearest in GPTQ v1 checkpoint form, no act-order.

    Per group (GPTQ's Quantizer.find_params with sym=False, Frantar et al.,
    arXiv:2210.17323): lo = min(w, 0), hi = max(w, 0), (-1, 1) for an all-zero
    group; scale = (hi - lo) / 15 stored as float16; zero = clamp(rint(-lo /
    scale), 0, 15); code = clamp(rint(w / scale) + zero, 0, 15), rounded with
    the stored float16 scale. W_hat = (code - zero) * scale.
    Returns qweight [I/8, O], qzeros [I/G, O/8] (zero - 1), scales [I/G, O]
    float16, g_idx [I] (i // G) and a zero float16 bias [O], for W [O, I]."""
    g = _groups(w, group)
    lo = np.minimum(g.min(axis=2), 0)
    hi = np.maximum(g.max(axis=2), 0)
    empty = (lo == 0) & (hi == 0)
    lo[empty], hi[empty] = -1, 1
    scales = ((hi - lo) / GPTQ_LEVELS).astype(np.float16)
    s32 = scales.astype(np.float32)
    zero = np.clip(np.rint(-lo / s32), 0, GPTQ_LEVELS)
    if (zero < 1).any():
        # v1 stores zero - 1 in 4 bits: a zero point of 0 would wrap to 16 on read
        raise ValueError("a group has no negative weight (zero point 0): not representable in GPTQ v1")
    codes = np.clip(np.rint(g / s32[..., None]) + zero[..., None], 0, GPTQ_LEVELS).astype(np.uint8)
    rows, cols = w.shape
    codes = codes.reshape(rows, cols)  # [O, I]
    return {
        "qweight": pack_int32_nibbles(codes.T, axis=0),
        "qzeros": pack_int32_nibbles((zero.astype(np.uint8) - 1).T, axis=1),
        "scales": np.ascontiguousarray(scales.T),
        "g_idx": (np.arange(cols) // group).astype(np.int32),
        "bias": np.zeros(rows, dtype=np.float16),
    }


def gptq_to_zp_matrix(t: dict[str, np.ndarray], group: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """GPTQ v1 tensors -> (packed [O, I/2], float16 scales [O, I/G], uint8 zeros
    [O, I/G] in 1..16), the ER_FMT_INT4_ZP matrix encoding. Lossless: the
    dequantized weights equal the GPTQ formula bit for bit. Refuses act-order
    (g_idx != i // G) and a nonzero bias, as store/gptq.py:65-71 does."""
    codes = unpack_int32_nibbles(t["qweight"], axis=0)  # [I, O]
    in_dim, out_dim = codes.shape
    if t["qzeros"].shape != (in_dim // group, out_dim // 8) or t["scales"].shape != (in_dim // group, out_dim):
        raise ValueError(f"shapes don't match group size {group}: {t['qzeros'].shape}, {t['scales'].shape}")
    if not np.array_equal(np.asarray(t["g_idx"]), np.arange(in_dim) // group):
        raise ValueError("g_idx is not i // group (desc_act?): not supported")
    if t.get("bias") is not None and np.any(t["bias"]):
        raise ValueError("non-zero bias: not supported")
    zeros = unpack_int32_nibbles(t["qzeros"], axis=1).astype(np.uint8) + 1  # [I/G, O]
    cT = np.ascontiguousarray(codes.T)
    packed = (cT[:, 0::2] | (cT[:, 1::2] << 4)).astype(np.uint8)
    return packed, np.ascontiguousarray(t["scales"].T, dtype=np.float16), np.ascontiguousarray(zeros.T)
