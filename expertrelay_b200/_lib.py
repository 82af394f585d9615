"""ctypes binding of libexpertrelay_b200.so (declared in include/expertrelay_b200.h).

The library is loaded on first use. A missing library raises ImportError:
there is no fallback implementation. Status codes map to the exceptions the
reference raises for the same situations: bad arguments -> ValueError
(runtime/backends.py:99-100, store/layout.py:125-126), CUDA failures and
device-side timeouts -> RuntimeError.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).with_name("libexpertrelay_b200.so")

ER_OK, ER_EINVAL, ER_ECUDA, ER_ETIMEOUT, ER_ENOSPACE, ER_EIO = 0, 1, 2, 3, 4, 5
DTYPE_F32, DTYPE_BF16 = 0, 1
FMT_INT8, FMT_INT4, FMT_INT4_ZP = 0, 1, 2
PATH_AUTO, PATH_GEMV, PATH_GEMM, PATH_TC = 0, 1, 2, 3

_vp = C.c_void_p
_i = C.c_int


class MoeWeights(C.Structure):
    """struct er_moe_weights."""

    _fields_ = [
        ("hidden", _i),
        ("num_experts", _i),
        ("top_k", _i),
        ("inter", _i),
        ("shared_inter", _i),
        ("expert_fmt", _i),
        ("group", _i),
        ("norm_topk_prob", _i),
        ("router_w", _vp),
        ("shared_gate_w", _vp),
        ("expert_records", _vp),
        ("shared_record", _vp),
        ("record_arena", _vp),
        ("arena_slots", _i),
    ]


class MoeIO(C.Structure):
    """struct er_moe_io."""

    _fields_ = [
        ("h", _vp),
        ("h_dtype", _i),
        ("n", _i),
        ("logits_in", _vp),
        ("y", _vp),
        ("logits_out", _vp),
        ("topk_idx_out", _vp),
        ("topk_w_out", _vp),
        ("path", _i),
        ("stage_events", C.POINTER(C.c_void_p)),
        ("launch_count", C.POINTER(_i)),
    ]


class MoeRowsIO(C.Structure):
    """struct er_moe_rows_io."""

    _fields_ = [
        ("x", _vp),
        ("x_dtype", _i),
        ("m", _i),
        ("expert", _vp),
        ("weight", _vp),
        ("y", _vp),
        ("path", _i),
        ("launch_count", C.POINTER(_i)),
        ("y_dtype", _i),
    ]


MOE_STAGES = ("router", "plan", "gate_up", "down", "combine")

CACHE_DRY = 1
SLOT_FREE, SLOT_LOADING, SLOT_READY = 0, 1, 2


class CacheStats(C.Structure):
    """struct er_cache_stats (the counters of SourceStats, runtime/weights.py:170-193)."""

    _fields_ = [
        (name, C.c_longlong)
        for name in (
            "loads",
            "bytes_read",
            "demand_reads",
            "cache_hits",
            "prefetch_hits",
            "prefetch_waits",
            "prefetches_issued",
            "prefetch_reads",
            "prefetch_bytes",
            "prefetches_wasted",
            "prefetches_cancelled",
            "prefetches_skipped_full",
            "prefetches_skipped_budget",
        )
    ]


# name -> (restype, argtypes); every function declared in include/expertrelay_b200.h
SIGNATURES: dict[str, tuple] = {
    "er_version": (_i, []),
    "er_last_error": (C.c_char_p, []),
    "er_device_sm_count": (_i, [C.POINTER(_i)]),
    "er_record_bytes": (C.c_size_t, [_i, _i, _i, _i]),
    "er_record_offset": (C.c_size_t, [_i, _i, _i, _i, _i, _i]),
    "er_linear_f32": (_i, [_vp, C.c_longlong, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "er_int8_linear": (_i, [_vp, C.c_longlong, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "er_int4_linear": (_i, [_vp, C.c_longlong, _vp, _vp, _vp, _i, _vp, _vp, _i, _i, _i, _vp]),
    "er_attention": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "er_dequant_int8": (_i, [_vp, _vp, _vp, _i, _i, _vp]),
    "er_dequant_int4": (_i, [_vp, _vp, _vp, _i, _vp, _i, _i, _vp]),
    "er_router_topk": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "er_moe_workspace_bytes": (C.c_size_t, [C.POINTER(MoeWeights), _i, _i]),
    "er_moe_block": (_i, [C.POINTER(MoeWeights), C.POINTER(MoeIO), _vp, C.c_size_t, _vp]),
    "er_moe_block_noalloc": (_i, [C.POINTER(MoeWeights), C.POINTER(MoeIO), _vp]),
    "er_tc_test_stall": (_i, [C.c_ulonglong, _i]),
    "er_moe_error_bits": (_i, [C.POINTER(MoeWeights), _i, _i, _vp, C.POINTER(_i), _vp]),
    "er_moe_rows_workspace_bytes": (C.c_size_t, [C.POINTER(MoeWeights), _i, _i]),
    "er_moe_rows": (_i, [C.POINTER(MoeWeights), C.POINTER(MoeRowsIO), _vp, C.c_size_t, _vp]),
    "er_moe_shared_workspace_bytes": (C.c_size_t, [C.POINTER(MoeWeights), _i, _i]),
    "er_moe_shared": (_i, [C.POINTER(MoeWeights), _vp, _i, _i, _vp, _i, _vp, C.c_size_t, _vp]),
    "er_moe_combine": (_i, [_vp, _i, _vp, _vp, _vp, _i, _i, _i, _vp, _vp]),
    "er_route_scratch_bytes": (C.c_size_t, [_i, _i]),
    "er_route": (_i, [_vp, _i, _i, _i, _vp, _i, _i, _i, _vp, C.c_size_t, _vp, _vp, _vp, _vp]),
    "er_ep_count": (_i, [_vp, _i, _i, _vp, _i, _i, _vp, _vp]),
    "er_ep_pack": (_i, [_vp, _i, _i, _vp, _vp, _i, _i, _vp, _vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _i, _vp, _vp]),
    "er_cache_create": (_i, [_i, C.c_size_t, _i, _vp, _i, C.POINTER(_vp)]),
    "er_cache_destroy": (_i, [_vp]),
    "er_cache_info": (_i, [_vp, C.POINTER(_vp), C.POINTER(_i), C.POINTER(C.c_size_t), C.POINTER(_vp)]),
    "er_cache_set_source": (_i, [_vp, _i, _i, C.POINTER(_vp)]),
    "er_cache_pin": (_i, [_vp, _i, _i]),
    "er_cache_acquire": (_i, [_vp, _i, C.POINTER(_i), _i, _vp, C.POINTER(C.c_uint64)]),
    "er_cache_prefetch": (_i, [_vp, _i, C.POINTER(_i), _i, C.POINTER(_i), _i, _i]),
    "er_cache_end_layer": (_i, [_vp, _i, _vp]),
    "er_cache_resize": (_i, [_vp, _i, _vp, C.POINTER(_i)]),
    "er_cache_lookup": (_i, [_vp, _i, _i, C.POINTER(_i), C.POINTER(_i)]),
    "er_cache_stats_get": (_i, [_vp, C.POINTER(CacheStats)]),
    "er_trace_record_bytes": (C.c_size_t, [_i, _i]),
    "er_rms_norm": (_i, [_vp, _vp, _vp, C.c_float, _i, _i, _vp, _vp, _vp]),
    "er_rope_kv": (_i, [_vp, C.c_longlong, _vp, _i, _i, _i, _i, _i, C.c_float, _vp, _vp, _i, _vp]),
    "er_embed_int8": (_i, [_vp, _vp, C.c_longlong, _i, _vp, _i, _vp, _vp, _vp]),
    "er_store_open": (_i, [C.c_char_p, _i, C.POINTER(_vp)]),
    "er_store_close": (_i, [_vp]),
    "er_store_info": (_i, [_vp, C.POINTER(C.c_uint64), C.POINTER(_i)]),
    "er_store_read": (_i, [_vp, C.c_uint64, C.c_uint64, _vp]),
    "er_store_read_many": (_i, [_vp, _i, _vp, C.c_uint64, _vp, _i, _vp]),
    "er_trace_pack_layer": (_i, [_vp, _i, _i, _i, _vp, _vp, _i, _vp, _vp, _i, _vp, _vp, _vp, _vp, _i, _i, _vp]),
}

_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """The loaded library with every signature set."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing; build it with `python -m expertrelay_b200.build`")
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().er_last_error()
    return msg.decode(errors="replace") if msg else ""


def check(rc: int, what: str) -> None:
    """Raise for a nonzero status: ValueError for bad arguments or too little
    workspace, OSError for failed or short file reads, RuntimeError for CUDA
    errors and device-side timeouts."""
    if rc == ER_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc in (ER_EINVAL, ER_ENOSPACE):
        raise ValueError(msg)
    if rc == ER_EIO:
        raise OSError(msg)
    raise RuntimeError(msg)
