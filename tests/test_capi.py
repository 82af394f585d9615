"""The C-ABI library without a GPU: it loads, exports every function the
header declares with the signatures the binding sets, answers the pure
queries, and rejects bad arguments before touching the device."""

from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

from expertrelay_b200 import _lib
from expertrelay_b200.store import FMT_INT4, FMT_INT4_ZP, FMT_INT8, RecordLayout

HEADERS = sorted((Path(__file__).resolve().parents[1] / "include").glob("*.h"))


def declared_functions() -> list[str]:
    names = []
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"^ER_API\s+[\w\s\*]+?\b(er_\w+)\s*\(", text, flags=re.M)
    return names


def test_library_exports_every_declared_function():
    names = declared_functions()
    assert len(names) >= 14
    L = _lib.lib()
    for n in names:
        assert hasattr(L, n), f"{n} declared in include/ but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(names)
    assert L.er_version() == 100


def declared_arities() -> dict[str, int]:
    out = {}
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for name, params in re.findall(r"^ER_API\s+[\w\s\*]+?\b(er_\w+)\s*\(([^)]*)\)\s*;", text, flags=re.M):
            params = " ".join(params.split())
            out[name] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_binding_arities_match_the_header():
    """Each ctypes signature takes as many arguments as the header's
    declaration: a parameter added on one side only fails here, not on a GPU."""
    arities = declared_arities()
    assert set(arities) == set(declared_functions())
    for name, n in arities.items():
        assert len(_lib.SIGNATURES[name][1]) == n, f"{name}: header {n} parameters, binding {len(_lib.SIGNATURES[name][1])}"


@pytest.mark.parametrize(
    "lay",
    [RecordLayout(FMT_INT8, 2048, 1408), RecordLayout(FMT_INT4, 2048, 1408, 128),
     RecordLayout(FMT_INT4_ZP, 2048, 1408, 128), RecordLayout(FMT_INT8, 2048, 5632), RecordLayout(FMT_INT4, 64, 32, 16)],
)
def test_record_queries_match_the_python_layout(lay):
    L = _lib.lib()
    assert L.er_record_bytes(lay.fmt, lay.hidden, lay.inter, lay.group) == lay.record_size
    for which, m in enumerate(("gate_proj", "up_proj", "down_proj")):
        assert L.er_record_offset(lay.fmt, lay.hidden, lay.inter, lay.group, which, 0) == lay.weight_offset(m)
        assert L.er_record_offset(lay.fmt, lay.hidden, lay.inter, lay.group, which, 1) == lay.scale_offset(m)
        if lay.fmt == FMT_INT4_ZP:
            assert L.er_record_offset(lay.fmt, lay.hidden, lay.inter, lay.group, which, 2) == lay.zero_offset(m)


def test_bad_arguments_are_rejected_without_a_device():
    L = _lib.lib()
    dummy = C.c_void_p(16)
    assert L.er_router_topk(dummy, 4, 0, 4, None, None, None, None) == _lib.ER_EINVAL
    assert "num_experts" in _lib.last_error()
    assert L.er_router_topk(dummy, 4, 60, 9, None, None, None, None) == _lib.ER_EINVAL
    assert L.er_int4_linear(dummy, 30, dummy, dummy, None, 8, None, dummy, 1, 4, 30, None) == _lib.ER_EINVAL
    assert "groups" in _lib.last_error()
    with pytest.raises(ValueError, match="er_int4_linear"):
        _lib.check(_lib.ER_EINVAL, "er_int4_linear")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.ER_ECUDA, "x")


def test_moe_weights_validation_and_workspace_query():
    L = _lib.lib()
    w = _lib.MoeWeights(hidden=2048, num_experts=60, top_k=4, inter=1408, shared_inter=5632, expert_fmt=0, group=0,
                        norm_topk_prob=0, router_w=16, shared_gate_w=16, expert_records=16, shared_record=256)
    ws = L.er_moe_workspace_bytes(C.byref(w), 8, 0)
    # logits, gate, top-k, plan, permutation, activations [8*4, 1408] + [8, 5632], outputs
    assert ws > 32 * 1408 * 4 + 8 * 5632 * 4 + 32 * 2048 * 4
    assert L.er_moe_workspace_bytes(C.byref(w), 4096, 0) > ws
    bad = _lib.MoeWeights.from_buffer_copy(w)
    bad.hidden = 2047
    assert L.er_moe_workspace_bytes(C.byref(bad), 8, 0) == 0
    io = _lib.MoeIO(h=16, h_dtype=0, n=8, y=16, path=0)
    assert L.er_moe_block(C.byref(bad), C.byref(io), None, 0, None) == _lib.ER_EINVAL
    assert "hidden" in _lib.last_error()
    assert L.er_moe_block(C.byref(w), C.byref(io), None, 0, None) == _lib.ER_ENOSPACE
    bad4 = _lib.MoeWeights.from_buffer_copy(w)
    bad4.expert_fmt, bad4.group = 1, 100
    assert L.er_moe_block(C.byref(bad4), C.byref(io), None, 0, None) == _lib.ER_EINVAL


# fixed device scratch of er_moe_block_noalloc (csrc/er_moe_noalloc.cu)
NOALLOC_SCRATCH_BYTES = 8 << 20


def _noalloc_limit(w, path: int) -> int:
    L = _lib.lib()
    n = 0
    while L.er_moe_workspace_bytes(C.byref(w), n + 1, path) <= NOALLOC_SCRATCH_BYTES:
        n += 1
    return n


def test_noalloc_token_limit_at_qwen_shapes():
    """er_moe_block_noalloc serves a batch when its er_moe_workspace_bytes
    fits the fixed 8 MiB scratch. At Qwen1.5-MoE-A2.7B shapes (60 experts,
    top-4) the limits its header states: 96 tokens on the GEMV / SIMT GEMM
    paths (the default without a record arena), 64 on the tensor-core path
    (the default for int8 records in an arena)."""
    w = _lib.MoeWeights(hidden=2048, num_experts=60, top_k=4, inter=1408, shared_inter=5632, expert_fmt=0, group=0,
                        norm_topk_prob=0, router_w=16, shared_gate_w=16, expert_records=16, shared_record=256)
    assert _noalloc_limit(w, _lib.PATH_AUTO) == 96
    assert _noalloc_limit(w, _lib.PATH_GEMV) == 96 and _noalloc_limit(w, _lib.PATH_GEMM) == 96
    arena = _lib.MoeWeights.from_buffer_copy(w)
    arena.record_arena, arena.arena_slots = 4096, 60
    assert _noalloc_limit(arena, _lib.PATH_TC) == 64
    assert _noalloc_limit(arena, _lib.PATH_AUTO) == 64
