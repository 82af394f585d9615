"""Generate the golden fixtures in tests/golden/ by running the reference.

    python tests/golden/make_golden.py --reference <path of the ExpertRelay checkout>

(or set EXPERTRELAY_REFERENCE to that path instead of passing --reference)

Imports ExpertRelay from <reference>/src (read only: no bytecode is written
and numba's cache goes to a temporary directory) and records its outputs on
seeded inputs: the quantizers and packers, the GPTQ conversion and formula,
the int8/int4 linear kernels (blocked and numba-fused), the record layouts,
and QwenMoe._moe on a small block and on full Qwen1.5-MoE-A2.7B-shaped
blocks built by expertrelay_b200.synth. Needs the reference, so it runs
where the reference is mounted; the fixtures it writes are committed and
are all the tests need.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]


def _import_reference(ref: Path):
    sys.dont_write_bytecode = True
    os.environ.setdefault("NUMBA_CACHE_DIR", tempfile.mkdtemp(prefix="numba-ref-"))
    sys.path.insert(0, str(ref / "src"))
    sys.path.insert(0, str(ROOT))


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def quantizer_fixtures() -> dict:
    from expertrelay.store.int4 import pack_int4, quantize_groupwise_int4, quantize_groupwise_int4_gptq_grid
    from expertrelay.store.quantize import quantize_rowwise_int8

    out = {}
    rng = np.random.default_rng(0)
    w = rng.normal(0, 0.02, (64, 128)).astype(np.float32)
    w[3] *= 50
    w[7] = 0  # all-zero row
    out["i8_w"] = w
    out["i8_q"], out["i8_s"] = quantize_rowwise_int8(w)

    w4 = (np.random.default_rng(1).standard_t(3, (64, 256)) * 0.02).astype(np.float32)
    w4[5, :32] = 0  # all-zero group
    out["i4_w"] = w4
    out["i4_q"], out["i4_s"] = quantize_groupwise_int4(w4, 32)
    bump = np.zeros((1, 8), dtype=np.float32)
    bump[0, 0] = 0.100006  # float16 rounding would shrink this group's scale
    out["i4_bump_w"] = bump
    out["i4_bump_q"], out["i4_bump_s"] = quantize_groupwise_int4(bump, 8)

    wg = (np.random.default_rng(2).standard_t(3, (6, 64)) * 0.02).astype(np.float32)
    wg[1, :16] = np.abs(wg[1, :16])
    wg[2, 16:32] = 0
    out["gg_w"] = wg
    out["gg_q"], out["gg_s"] = quantize_groupwise_int4_gptq_grid(wg, 16)

    pq = np.random.default_rng(3).integers(-8, 8, (5, 12)).astype(np.int8)
    out["pack_q"] = pq
    out["pack_p"] = pack_int4(pq)
    return out


def _pack_gptq_int32(codes: np.ndarray, axis: int) -> np.ndarray:
    # element-by-element packer, independent of both implementations under test
    codes = np.moveaxis(codes, axis, 0)
    out = np.zeros((codes.shape[0] // 8, *codes.shape[1:]), dtype=np.uint32)
    for i in range(codes.shape[0]):
        out[i // 8] |= codes[i].astype(np.uint32) << np.uint32(4 * (i % 8))
    return np.moveaxis(out, 0, axis).view(np.int32)


def _gptq_layer(out_dim, in_dim, group, seed, zero=8):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 16, (in_dim, out_dim))
    codes[0, 0], codes[1, 0] = 0, 15
    return {
        "qweight": _pack_gptq_int32(codes, axis=0),
        "qzeros": _pack_gptq_int32(np.full((in_dim // group, out_dim), zero - 1), axis=1),
        "scales": rng.uniform(0.001, 0.05, (in_dim // group, out_dim)).astype(np.float16),
        "g_idx": (np.arange(in_dim) // group).astype(np.int32),
        "bias": np.zeros(out_dim, dtype=np.float16),
    }


def gptq_fixtures() -> dict:
    from expertrelay.bench.gptq_conversion_check import reference_dequantize
    from expertrelay.store.gptq import gptq_to_int4

    out = {}
    t = _gptq_layer(48, 64, 16, seed=0)
    for k, v in t.items():
        out[f"sym_{k}"] = v
    out["sym_store_packed"], out["sym_store_scales"] = gptq_to_int4(*t.values(), group=16)
    out["sym_ref_w"] = reference_dequantize(t["qweight"], t["qzeros"], t["scales"], t["g_idx"])
    a = _gptq_layer(8, 16, 8, seed=1, zero=3)
    a["g_idx"] = a["g_idx"][::-1].copy()
    for k, v in a.items():
        out[f"asym_{k}"] = v
    out["asym_ref_w"] = reference_dequantize(a["qweight"], a["qzeros"], a["scales"], a["g_idx"])
    b = _gptq_layer(304, 128, 32, seed=3)
    for k, v in b.items():
        out[f"k_{k}"] = v
    out["k_ref_w"] = reference_dequantize(b["qweight"], b["qzeros"], b["scales"], b["g_idx"])
    return out


def linear_fixtures() -> dict:
    from expertrelay.runtime.int4_linear import int4_linear
    from expertrelay.runtime.int8_linear import int8_linear
    from expertrelay.store.int4 import pack_int4, quantize_groupwise_int4
    from expertrelay.store.quantize import quantize_rowwise_int8

    out = {}
    rng = np.random.default_rng(0)
    q, s = quantize_rowwise_int8(rng.normal(0, 0.05, (300, 96)).astype(np.float32))
    out["i8_q"], out["i8_s"] = q, s
    out["i8_bias"] = rng.normal(0, 1, 300).astype(np.float32)
    for n in (1, 3, 40):
        x = rng.normal(0, 1, (n, 96)).astype(np.float32)
        out[f"i8_x{n}"] = x
        out[f"i8_y{n}_blocked"] = int8_linear(x, q, s, kernel="blocked")
        out[f"i8_y{n}_fused"] = int8_linear(x, q, s, kernel="fused")
        out[f"i8_y{n}_bias"] = int8_linear(x, q, s, out["i8_bias"], kernel="blocked")
    rng = np.random.default_rng(3)
    v, s4 = quantize_groupwise_int4(rng.normal(0, 0.05, (300, 128)).astype(np.float32), 32)
    p = pack_int4(v)
    out["i4_p"], out["i4_s"] = p, s4
    for n in (1, 4, 20):
        x = rng.normal(0, 1, (n, 128)).astype(np.float32)
        out[f"i4_x{n}"] = x
        out[f"i4_y{n}_blocked"] = int4_linear(x, p, s4, 32, kernel="blocked")
        out[f"i4_y{n}_fused"] = int4_linear(x, p, s4, 32, kernel="fused")
    return out


def layout_fixtures(ref: Path) -> dict:
    from expertrelay.store.int4 import Int4RecordLayout, pack_int4, quantize_groupwise_int4, serialize_int4_record
    from expertrelay.store.layout import ExpertRecordLayout, serialize_expert_record
    from expertrelay.store.quantize import quantize_rowwise_int8

    cfg = {"moe_intermediate_size": 16, "hidden_size": 32}
    rng = np.random.default_rng(4)
    l8 = ExpertRecordLayout.from_config(cfg)
    q8 = {
        n: quantize_rowwise_int8(rng.normal(0, 0.1, s).astype(np.float32)) for n, s in l8.matrices
    }
    rec8 = np.frombuffer(bytes(serialize_expert_record(l8, q8)), dtype=np.uint8)
    l4 = Int4RecordLayout.from_config(cfg, 8)
    q4 = {}
    for n, s in l4.matrices:
        v, sc = quantize_groupwise_int4(rng.normal(0, 0.1, s).astype(np.float32), 8)
        q4[n] = (pack_int4(v), sc)
    rec4 = np.frombuffer(bytes(serialize_int4_record(l4, q4)), dtype=np.uint8)
    out = {"rec8": rec8, "rec4": rec4}
    for n, (qq, ss) in q8.items():
        out[f"rec8_{n}_q"], out[f"rec8_{n}_s"] = qq, ss
    for n, (pp, ss) in q4.items():
        out[f"rec4_{n}_p"], out[f"rec4_{n}_s"] = pp, ss
    manifests = {}
    for d in sorted((ref / "benchmarks" / "stores").glob("*/store.json")):
        manifests[d.parent.name] = json.loads(d.read_text())["expert_layout"]
    return out, manifests


def _run_moe(block, x, kernel="blocked"):
    from expertrelay.runtime import int8_linear as i8mod
    from expertrelay.runtime.qwen_moe import ForwardTrace, ModelConfig, QwenMoe, StepTimings
    from expertrelay.runtime.weights import ExpertSource, Int4Matrix, Int8Matrix, ResidentWeights, SourceStats

    class MemSource(ExpertSource):
        def __init__(self, experts):
            self._experts = experts
            self.stats = SourceStats()

        def load(self, layer, expert):
            return self._experts[expert]

    experts = []
    for mats in block.experts:
        d = {}
        for name, t in mats.items():
            if block.fmt == "int8":
                d[name] = Int8Matrix(t[0], t[1])
            elif block.fmt == "int4":
                d[name] = Int4Matrix(t[0], t[1], t[0].shape[1] * 2 // t[1].shape[1])
            else:
                raise ValueError("the reference path has no zero-point int4 (store/gptq.py:67-69)")
        experts.append(d)
    p = "model.layers.0.mlp."
    resident = ResidentWeights(
        {
            p + "gate.weight": block.router,
            p + "shared_expert_gate.weight": block.shared_gate,
            **{p + f"shared_expert.{m}.weight": Int8Matrix(*block.shared[m]) for m in block.shared},
        },
        0,
    )
    cfg = ModelConfig(151936, block.hidden, 1, 16, 16, block.num_experts, block.top_k, False, 1e-6, 1e6)
    model = QwenMoe(cfg, resident, MemSource(experts))
    before = i8mod.current_kernel()
    i8mod.set_kernel(kernel)
    try:
        trace = ForwardTrace()
        lg = model._linear(p + "gate.weight", x)
        y = model._moe(0, x, StepTimings(), trace, None)
    finally:
        i8mod.set_kernel(before)
    return y, lg, trace.selected_experts[0]


def moe_fixtures() -> dict:
    from expertrelay_b200 import synth

    out = {}
    # small block: every shape path of the kernels at a size the oracle runs in milliseconds
    for fmt, group in (("int8", 0), ("int4", 16)):
        blk = synth.make_block(11, hidden=64, inter=32, shared_inter=48, num_experts=8, top_k=4, fmt=fmt,
                               group=group or 128, sigma=0.1)
        x = synth.make_tokens(11, 5, 64)
        y, lg, sel = _run_moe(blk, x)
        tag = f"mini_{fmt}"
        out[f"{tag}_x"], out[f"{tag}_y"], out[f"{tag}_logits"], out[f"{tag}_sel"] = x, y, lg, sel
        out[f"{tag}_records"] = blk.records()
        out[f"{tag}_shared_record"] = blk.shared_record()
        out[f"{tag}_router"], out[f"{tag}_shared_gate"] = blk.router, blk.shared_gate
    return out


def full_fixtures() -> dict:
    """Qwen-shaped blocks: outputs of the reference on the synth workloads.
    The weights are regenerated from the seed; their digests pin them."""
    from expertrelay_b200 import synth

    out = {}
    blk, x = synth.make_workload("decode8_int8", seed=0)
    for kernel in ("blocked", "fused"):
        y, lg, sel = _run_moe(blk, x, kernel=kernel)
        out[f"decode8_y_{kernel}"] = y
    out["decode8_x"], out["decode8_logits"], out["decode8_sel"] = x, lg, sel
    out["decode8_records_sha"] = np.frombuffer(sha(blk.records()).encode(), dtype=np.uint8)
    out["decode8_shared_sha"] = np.frombuffer(sha(blk.shared_record()).encode(), dtype=np.uint8)
    out["decode8_router_sha"] = np.frombuffer(sha(blk.router).encode(), dtype=np.uint8)

    blk, x = synth.make_workload("prefill4096_int8_zipf", seed=0)
    y, lg, sel = _run_moe(blk, x)
    out["prefill_sel"] = sel.astype(np.int8)
    out["prefill_logits"] = lg.astype(np.float32)
    out["prefill_y_head"] = y[:32]
    # every row of the output projected on PREFILL_SKETCH_COLS seeded
    # directions: catches a wrong direction that the row norms cannot
    out["prefill_y_sketch"] = y.astype(np.float64) @ prefill_sketch_matrix(y.shape[1])
    out["prefill_y_rownorm"] = np.linalg.norm(y.astype(np.float64), axis=1)
    out["prefill_y_sum"] = np.array([y.astype(np.float64).sum()])
    out["prefill_router_sha"] = np.frombuffer(sha(blk.router).encode(), dtype=np.uint8)
    out["prefill_zipf_realised"] = np.array(blk.meta["zipf"]["realised"])
    return out


PREFILL_SKETCH_SEED, PREFILL_SKETCH_COLS = 7, 8


def prefill_sketch_matrix(hidden: int) -> np.ndarray:
    """[hidden, PREFILL_SKETCH_COLS] float64 directions (the GPU test rebuilds them)."""
    return np.random.default_rng(PREFILL_SKETCH_SEED).standard_normal((hidden, PREFILL_SKETCH_COLS))


def prefetch_fixtures() -> tuple[dict, dict]:
    """The reference's prefetch policy (predictor/prefetch_policy.py:41-54)
    and calibration maps (predictor/offline.py:87-200) on seeded router
    logits: the experts each policy picks, the low-confidence skips, and
    the calibrated probabilities; plus the maps' JSON form."""
    from expertrelay.predictor.offline import IsotonicCalibrator, RankedIsotonicCalibrator
    from expertrelay.predictor.prefetch_policy import PrefetchPolicy

    rng = np.random.default_rng(21)
    # fitted maps: scores with labels that grow more likely with the score
    scores = rng.uniform(0, 1, 4000)
    labels = (rng.uniform(0, 1, 4000) < scores ** 2).astype(np.float64)
    single = IsotonicCalibrator(num_bins=40).fit(scores, labels)
    probs = rng.dirichlet(np.full(16, 0.3), 600)
    picked = np.zeros_like(probs)
    np.put_along_axis(picked, np.argsort(-probs + rng.normal(0, 0.05, probs.shape), axis=1)[:, :4], 1.0, axis=1)
    ranked = RankedIsotonicCalibrator(max_rank=6, num_bins=20).fit(probs, picked)
    cases = []
    for n, e, scale in ((1, 60, 2.0), (1, 16, 0.5), (7, 60, 1.5), (3, 16, 3.0), (32, 60, 1.0)):
        cases.append(rng.normal(0, scale, (n, e)).astype(np.float32))
    tie = np.zeros((2, 16), dtype=np.float32)
    tie[0, [9, 4, 12]] = 2.0  # equal best scores: ascending id
    cases.append(tie)
    out = {}
    policies = (("plain", None, 0.0), ("single", single, 0.3), ("ranked", ranked, 0.3), ("ranked_hi", ranked, 0.7))
    for c, logits in enumerate(cases):
        out[f"logits{c}"] = logits
        for name, cal, pmin in policies:
            for k in (1, 4, 8):
                choice = PrefetchPolicy(top_k=k, min_probability=pmin, calibrator=cal).choose(logits)
                out[f"experts{c}_{name}_k{k}"] = np.array(choice.experts, dtype=np.int64)
                out[f"skipped{c}_{name}_k{k}"] = np.array([choice.skipped_low_confidence])
        out[f"single_pred{c}"] = single.predict(logits.ravel())
        out[f"ranked_pred{c}"] = ranked.predict(np.exp(logits) / np.exp(logits).sum(axis=-1, keepdims=True))
    maps = {"calibrator": single.to_dict(), "rank_calibrator": ranked.to_dict(), "cases": len(cases)}
    return out, maps


# (num_layers, num_experts, top_k, prefill tokens) of the trace fixtures
TRACE_CASES = ((3, 8, 2, 5), (2, 60, 4, 3))


def trace_inputs(case: int) -> list[dict]:
    """Seeded writer calls for trace case `case`: a prefill call, then two
    one-token decode calls. Logits hold values that float16 rounds to
    infinity, to subnormals and to zero, and a tie inside the top-k."""
    layers, experts, k, n0 = TRACE_CASES[case]
    rng = np.random.default_rng(100 + case)
    calls, pos = [], 0
    for n, phase in ((n0, 0), (1, 1), (1, 1)):
        call = {"positions": np.arange(pos, pos + n, dtype=np.int64),
                "tokens": rng.integers(0, 151936, n).astype(np.int64), "phase": phase, "layers": []}
        pos += n
        for layer in range(layers):
            logits = rng.normal(0, 3, (n, experts)).astype(np.float32)
            logits[0, 0] = 70000.0  # float16 overflow
            logits[0, 1] = 3e-6     # float16 subnormal
            logits[-1, 2] = -1e-9   # rounds to -0
            sel = np.argsort(-logits, axis=1, kind="stable")[:, :k].astype(np.int64)
            p = np.exp(logits - logits.max(axis=1, keepdims=True))
            p /= p.sum(axis=1, keepdims=True)
            weights = np.take_along_axis(p, sel, axis=1).astype(np.float32)
            fate = None
            if layer + 1 < layers:
                fate = rng.normal(0, 2, (n, experts)).astype(np.float32)
                fate[0, 3] = fate[0, 5] = fate[0].max() + 1.0  # an exact tie at the top (lower id first)
            call["layers"].append({"logits": logits, "selected": sel, "weights": weights, "fate": fate})
        calls.append(call)
    return calls


def trace_fixtures(tmp: Path) -> dict:
    """The reference ExpertTraceWriter's file for each trace case."""
    from expertrelay.runtime.expert_trace import ExpertTraceWriter

    out = {}
    for case, (layers, experts, k, _) in enumerate(TRACE_CASES):
        path = tmp / f"trace{case}.ert"
        w = ExpertTraceWriter(path, num_layers=layers, num_experts=experts, top_k=k,
                              metadata={"prompt_id": f"case{case}", "model": "synthetic"})
        for call in trace_inputs(case):
            w.begin(call["positions"], call["tokens"], call["phase"])
            for layer, lc in enumerate(call["layers"]):
                w.layer(layer, lc["logits"], lc["selected"], lc["weights"], lc["fate"])
            w.end()
        out[f"file{case}"] = np.frombuffer(path.read_bytes(), dtype=np.uint8)
    return out


# a small Qwen2-MoE decoder for the whole-model fixtures (the reference's
# QwenMoe.forward on it, numpy backend)
TINY_MODEL = {
    "vocab_size": 96,
    "hidden_size": 256,
    "num_hidden_layers": 3,
    "num_attention_heads": 4,
    "num_key_value_heads": 4,
    "num_experts": 16,
    "num_experts_per_tok": 4,
    "moe_intermediate_size": 128,
    "shared_expert_intermediate_size": 384,
    "norm_topk_prob": False,
    "rms_norm_eps": 1e-6,
    "rope_theta": 1e6,
}
TINY_MODEL_GQA = {**TINY_MODEL, "num_key_value_heads": 2, "norm_topk_prob": True}
MODEL_CASES = ((TINY_MODEL, 11), (TINY_MODEL_GQA, 12))
MODEL_PROMPT, MODEL_NEW = 9, 4


def model_fixtures() -> dict:
    """The reference forward pass (runtime/qwen_moe.py:376-432) on seeded
    synthetic decoders (expertrelay_b200.synth.make_model, regenerated by
    the tests from the same seeds): all-position logits of a prompt, then
    greedy decoding one token per call, with each call's logits."""
    from expertrelay.runtime.qwen_moe import KVCache, ModelConfig, QwenMoe
    from expertrelay.runtime.weights import ExpertSource, Int8Matrix, ResidentWeights, SourceStats

    from expertrelay_b200 import synth

    out = {}
    for case, (cfg, seed) in enumerate(MODEL_CASES):
        host = synth.make_model(cfg, seed=seed)
        tensors = {k: (Int8Matrix(*v) if isinstance(v, tuple) else v) for k, v in host.tensors().items()}

        class MemSource(ExpertSource):
            def __init__(self):
                self.stats = SourceStats()

            def load(self, layer, expert):
                self.stats.loads += 1
                return {m: Int8Matrix(*qs) for m, qs in host.blocks[layer].experts[expert].items()}

        model = QwenMoe(ModelConfig.from_hf(cfg), ResidentWeights(tensors, 0), MemSource())
        kv = KVCache(model.c, MODEL_PROMPT + MODEL_NEW)
        prompt = np.random.default_rng(seed).integers(0, cfg["vocab_size"], MODEL_PROMPT)
        logits, _ = model.forward(prompt, kv, all_logits=True)
        out[f"prompt{case}"] = prompt
        out[f"prompt_logits{case}"] = logits.astype(np.float32)
        tok, toks, steps = int(np.argmax(logits[-1])), [], []
        for _ in range(MODEL_NEW):
            toks.append(tok)
            step, _ = model.forward(np.array([tok]), kv)
            steps.append(step.astype(np.float32))
            tok = int(np.argmax(step))
        out[f"tokens{case}"] = np.array(toks, dtype=np.int64)
        out[f"step_logits{case}"] = np.stack(steps)
    return out


STORE_SHAPE = {"hidden_size": 64, "moe_intermediate_size": 32, "num_layers": 2, "num_experts": 3}


def store_fixture(out_dir: Path) -> None:
    """A tiny int8 expert store (experts.bin + experts_index.json) written
    with the reference's record and index writers (store/layout.py:117-133,
    179-188) at the offsets its builder uses (expert_offset, :152-153)."""
    from expertrelay.store.layout import (
        ExpertIndexEntry,
        ExpertRecordLayout,
        expert_offset,
        serialize_expert_record,
        write_expert_index,
    )
    from expertrelay.store.quantize import quantize_rowwise_int8

    cfg = STORE_SHAPE
    layout = ExpertRecordLayout.from_config(cfg)
    rng = np.random.default_rng(42)
    out_dir.mkdir(parents=True, exist_ok=True)
    entries, blob = [], bytearray()
    for layer in range(cfg["num_layers"]):
        for expert in range(cfg["num_experts"]):
            quantized = {m: quantize_rowwise_int8(rng.normal(0, 0.02, s).astype(np.float32)) for m, s in layout.matrices}
            record = serialize_expert_record(layout, quantized)
            offset = expert_offset(layer, expert, cfg["num_experts"], layout.record_size)
            blob[len(blob):offset + layout.record_size] = bytes(offset + layout.record_size - len(blob))
            blob[offset:offset + layout.record_size] = record
            entries.append(ExpertIndexEntry(layer=layer, expert=expert, offset=offset, size=layout.record_size,
                                            shapes={m: list(sh) for m, sh in layout.matrices},
                                            sha256=hashlib.sha256(record).hexdigest(), quant_error={}))
    (out_dir / "experts.bin").write_bytes(bytes(blob))
    write_expert_index(out_dir / "experts_index.json", layout, entries)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("EXPERTRELAY_REFERENCE"),
                    help="the ExpertRelay checkout (default: $EXPERTRELAY_REFERENCE)")
    ap.add_argument("--skip-full", action="store_true")
    ap.add_argument("--only", choices=("trace", "store", "model", "prefetch", "qwen"),
                    help="regenerate one fixture only")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set EXPERTRELAY_REFERENCE")
    ref = Path(args.reference)
    _import_reference(ref)
    if args.only == "qwen":
        np.savez_compressed(HERE / "moe_qwen.npz", **full_fixtures())
        return
    if args.only in (None, "prefetch"):
        arrays, maps = prefetch_fixtures()
        np.savez_compressed(HERE / "prefetch.npz", **arrays)
        (HERE / "prefetch_maps.json").write_text(json.dumps(maps, indent=1))
    if args.only in (None, "trace"):
        with tempfile.TemporaryDirectory() as tmp:
            np.savez_compressed(HERE / "trace.npz", **trace_fixtures(Path(tmp)))
    if args.only in (None, "store"):
        store_fixture(HERE / "store_small")
    if args.only in (None, "model"):
        np.savez_compressed(HERE / "model.npz", **model_fixtures())
    if args.only is not None:
        return
    np.savez_compressed(HERE / "quant.npz", **quantizer_fixtures())
    np.savez_compressed(HERE / "gptq.npz", **gptq_fixtures())
    np.savez_compressed(HERE / "linear.npz", **linear_fixtures())
    lay, manifests = layout_fixtures(ref)
    np.savez_compressed(HERE / "layout.npz", **lay)
    (HERE / "store_manifests.json").write_text(json.dumps(manifests, indent=1, sort_keys=True))
    np.savez_compressed(HERE / "moe_mini.npz", **moe_fixtures())
    if not args.skip_full:
        np.savez_compressed(HERE / "moe_qwen.npz", **full_fixtures())
    for f in sorted(HERE.glob("*.npz")):
        print(f"{f.name}: {f.stat().st_size / 1024:.1f} KiB")


if __name__ == "__main__":
    main()
