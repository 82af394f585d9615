#!/usr/bin/env python
"""Benchmark of the MoE-block hot path (QwenMoe._moe at Qwen1.5-MoE-A2.7B shapes).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload prefill4096_int8_zipf|decode8_int8|gptq_asym_decode1|gptq_asym_prefill512]

One step = one MoE block forward over one batch of seeded synthetic tokens
(router -> top-4 -> routed experts -> combine + gated shared expert). Rank 0
prints one JSON line. `value` is whole-job tokens/s with inputs resident in
HBM; `e2e` is the same through the public API from pinned host buffers, with
the host->device copy of the tokens and the device->host copy of the output
inside the timed region (HostPipeline: the copies of neighbouring steps
overlap each step's compute; `e2e.serial_value` runs one step at a time).
Each step is timed with CUDA events on the
launching stream after an L2 flush (a 256 MiB write), and the dominant
kernel is timed live through the block's stage events.

On one GPU the line also carries `decode` (the same block at 8 decode
tokens) and `full_model`: greedy decoding through the whole 24-layer
Qwen1.5-MoE-A2.7B-shaped decoder (random init, a 512-token seeded prompt,
128 tokens, batch 1) with a quarter of the routed experts in the HBM cache
and the rest paged from pinned host memory with the Fate prefetch
(--no-full-model skips it; --model-layers, --prompt-tokens, --new-tokens,
--cache-frac size it).

On one GPU the line also carries `gptq`: the block with int4 GPTQ-style
experts (asymmetric, group 128) at 1 and 512 tokens (--no-gptq skips it).

On every N the line carries `expert_parallel`: the MoE layer of the
expert-parallel prefill (32 x 2048 tokens split over the N ranks, the 60
experts spread over the GPUs, NCCL all-to-all of rows and results), timed
as max over ranks (--no-ep skips it). On N > 1 GPUs that layer is the
headline `value` (strong scaling) and the independent per-GPU replicas of
the block move to `replicas`.

--impl reference times the CPU implementation of the path (the oracle, a
restatement of the reference's numpy/BLAS code) on this host's cores on the
same workload; under torchrun only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import sys
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
FLUSH_BYTES = 256 << 20


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default="prefill4096_int8_zipf")
    ap.add_argument("--path", choices=("auto", "gemv", "gemm", "tc"), default="tc")
    ap.add_argument("--act-dtype", choices=("f32", "bf16"), default="f32")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode-shape side measurement")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="CPU-baseline sample budget")
    ap.add_argument("--no-full-model", action="store_true", help="skip the whole-model decode measurement")
    ap.add_argument("--model-layers", type=int, default=24, help="decoder layers of the whole-model measurement")
    ap.add_argument("--prompt-tokens", type=int, default=512)
    ap.add_argument("--new-tokens", type=int, default=128)
    ap.add_argument("--cache-frac", type=float, default=0.25, help="HBM expert-cache share of the routed records")
    ap.add_argument("--no-gptq", action="store_true", help="skip the int4 GPTQ block measurement")
    ap.add_argument("--no-ep", action="store_true", help="skip the expert-parallel layer measurement")
    ap.add_argument("--ep-tokens", type=int, default=65536, help="tokens of the expert-parallel layer (all ranks)")
    ap.add_argument("--ep-microbatch", type=int, default=0,
                    help="tokens per expert-parallel microbatch (0: half a rank's tokens, 4096 to 16384)")
    ap.add_argument("--ep-steps", type=int, default=10)
    return ap.parse_args()


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return {k: float(d[k]) for k in FALLBACK_PEAKS if k in d}, "measured"
        except (ValueError, KeyError):
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def traffic_from_profiles(workload: str, stage: str) -> tuple[float | None, str | None]:
    """DRAM bytes per launch recorded from an ncu capture in profiles/*.md, as a
    line `traffic_per_launch_bytes[<workload>/<stage>] = <bytes>`, and the file
    it came from. The figure is from that capture, not from this run."""
    key = f"traffic_per_launch_bytes[{workload}/{stage}]"
    for f in sorted((ROOT / "profiles").glob("*.md")):
        for line in f.read_text().splitlines():
            if key in line and "=" in line:
                try:
                    return float(line.split("=", 1)[1].strip().strip("`").split()[0]), f"profiles/{f.name}"
                except ValueError:
                    return None, None
    return None, None


class ClockSampler:
    """SM clock, power and clock-event reasons sampled through NVML every
    5 ms while the timed region runs (the data nvidia-smi's clocks query
    reports), for the GPU behind `device`."""

    REASONS = {
        "hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
        "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
        "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
        "sw_power_cap": "nvmlClocksEventReasonSwPowerCap",
        "hw_power_brake": "nvmlClocksEventReasonHwPowerBrakeSlowdown",
    }

    def __init__(self, device):
        self.device = device
        self.samples: list[tuple[float, float, int]] = []
        self.max_mhz = None
        self.error = None
        self._stop = None
        self._thread = None

    def _handle(self, nv):
        import torch

        p = torch.cuda.get_device_properties(self.device)
        try:
            return nv.nvmlDeviceGetHandleByPciBusId(f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0")
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.device.index or 0)

    def __enter__(self):
        import threading

        try:
            import pynvml as nv

            nv.nvmlInit()
            h = self._handle(nv)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        except Exception as e:  # no NVML: report unsampled
            self.error = f"{type(e).__name__}: {e}"
            return self
        self._stop = threading.Event()

        def run():
            while not self._stop.is_set():
                try:
                    self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                         nv.nvmlDeviceGetPowerUsage(h) / 1000.0,
                                         int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))))
                except Exception as e:
                    self.error = f"{type(e).__name__}: {e}"
                    return
                self._stop.wait(0.005)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"], "samples": 0,
                    "error": self.error}
        import pynvml as nv

        reasons = sorted(name for name, attr in self.REASONS.items()
                         if any(r & getattr(nv, attr) for _, _, r in self.samples))
        return {
            "sm_mhz": statistics.median(c for c, _, _ in self.samples),
            "sm_max_mhz": self.max_mhz,
            "power_w_max": max(p for _, p, _ in self.samples),
            "reasons": reasons,
            "samples": len(self.samples),
            "source": "NVML, 5 ms period, during the timed steps",
        }


# the MoE layer of the expert-parallel prefill (32 sequences x 2048 tokens)
EP_WORKLOAD = "ep_prefill65536_int8"


def arm_workload(args, world: int) -> str:
    """The workload the headline `value` measures at this GPU count: the
    block of --workload on one GPU, the expert-parallel layer on several."""
    return EP_WORKLOAD if world > 1 and not args.no_ep else args.workload


def blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        info = [i for i in threadpool_info() if i.get("user_api") == "blas"]
        if info:
            return int(max(i.get("num_threads", 1) for i in info))
    except Exception:
        pass
    return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ---------------------------------------------------------------------------
# workload accounting (algorithmic bytes and FLOPs)
# ---------------------------------------------------------------------------


def accounting(block, n: int, idx: np.ndarray, act_bytes: int) -> dict:
    H, I, Is, E, k = block.hidden, block.inter, block.shared_inter, block.num_experts, block.top_k
    lay, sh = block.layout, block.shared_layout
    uniq = np.unique(idx)
    U = len(uniq)
    nk = n * k
    # weight bytes each kernel must read once: gate+up (codes + scales (+ zeros)) and down
    gu_w = sum(lay._weight_bytes(m) + lay._scale_bytes(m) + lay._zero_bytes(m) for m in ("gate_proj", "up_proj"))
    dn_w = lay._weight_bytes("down_proj") + lay._scale_bytes("down_proj") + lay._zero_bytes("down_proj")
    sh_gu = sum(sh._weight_bytes(m) + sh._scale_bytes(m) for m in ("gate_proj", "up_proj"))
    sh_dn = sh._weight_bytes("down_proj") + sh._scale_bytes("down_proj")
    gate_up_bytes = U * gu_w + sh_gu + n * H * act_bytes + (nk * I + n * Is) * 4
    down_bytes = U * dn_w + sh_dn + (nk * I + n * Is) * 4 + (nk + n) * H * 4
    block_weight_bytes = U * (gu_w + dn_w) + sh_gu + sh_dn + E * H * 4 + H * 4
    return {
        "unique_experts": int(U),
        "gate_up_bytes": int(gate_up_bytes),
        "down_bytes": int(down_bytes),
        "block_weight_bytes": int(block_weight_bytes),
        "gate_up_flops": int(2 * (nk * 2 * I * H + n * 2 * Is * H)),
        "down_flops": int(2 * (nk * I * H + n * Is * H)),
        "router_flops": int(2 * n * (E + 1) * H),
        "block_flops": int(2 * (nk * 3 * I * H + n * 3 * Is * H + n * (E + 1) * H)),
    }


# ---------------------------------------------------------------------------
# CPU side: the reference's own QwenMoe._moe (installed in baseline/_ref), and
# the oracle port of it
# ---------------------------------------------------------------------------

REF_DIR = ROOT / "baseline" / "_ref"


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def pin_cpu_threads(cores: int) -> dict:
    """Give the reference's BLAS and numba pools every host core, whatever
    the launcher set (torchrun sets OMP_NUM_THREADS=1 on every rank); returns
    the thread counts actually in effect."""
    os.environ["NUMBA_NUM_THREADS"] = str(cores)
    got = {"blas": None, "numba": None}
    try:
        from threadpoolctl import threadpool_info, threadpool_limits

        threadpool_limits(limits=cores)
        blas = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        got["blas"] = int(max(blas)) if blas else None
    except Exception as e:  # reported, not fatal
        got["blas_error"] = f"{type(e).__name__}: {e}"[:120]
    try:
        import numba

        numba.set_num_threads(min(cores, numba.config.NUMBA_NUM_THREADS))
        got["numba"] = int(numba.get_num_threads())
    except Exception as e:
        got["numba_error"] = f"{type(e).__name__}: {e}"[:120]
    return got


class ReferenceBlock:
    """The reference's QwenMoe._moe (runtime/qwen_moe.py:293-359) from the
    unmodified package in baseline/_ref, driven in memory: the router, the
    shared expert and its gate as ResidentWeights, the routed experts from
    an ExpertSource that hands out Int8Matrix / Int4Matrix views of the
    block's store encodings (runtime/weights.py:51-80, 196-235). `kernel`
    is the reference's int8 kernel choice (runtime/int8_linear.py:78-93;
    "fused" is its runtime default, runtime/generate.py:110)."""

    def __init__(self, block, kernel: str = "fused"):
        if not (REF_DIR / "expertrelay").is_dir():
            raise ImportError(f"the reference is not installed in {REF_DIR}")
        sys.dont_write_bytecode = True
        import tempfile

        os.environ.setdefault("NUMBA_CACHE_DIR", tempfile.mkdtemp(prefix="numba-ref-"))
        if str(REF_DIR) not in sys.path:
            sys.path.insert(0, str(REF_DIR))
        from expertrelay.runtime import int8_linear as i8mod
        from expertrelay.runtime.qwen_moe import ModelConfig, QwenMoe, StepTimings
        from expertrelay.runtime.weights import ExpertSource, Int4Matrix, Int8Matrix, ResidentWeights, SourceStats

        if block.fmt not in ("int8", "int4"):
            raise ValueError(f"the reference's block path has no {block.fmt} experts (store/gptq.py:67-69)")
        experts = []
        for mats in block.experts:
            if block.fmt == "int8":
                experts.append({m: Int8Matrix(t[0], t[1]) for m, t in mats.items()})
            else:
                experts.append({m: Int4Matrix(t[0], t[1], t[0].shape[1] * 2 // t[1].shape[1]) for m, t in mats.items()})

        class MemorySource(ExpertSource):
            def __init__(self):
                self.stats = SourceStats()

            def load(self, layer, expert):
                return experts[expert]

        p = "model.layers.0.mlp."
        resident = ResidentWeights({
            p + "gate.weight": block.router,
            p + "shared_expert_gate.weight": block.shared_gate,
            **{p + f"shared_expert.{m}.weight": Int8Matrix(*block.shared[m]) for m in block.shared},
        }, 0)
        cfg = ModelConfig(151936, block.hidden, 1, 16, 16, block.num_experts, block.top_k, False, 1e-6, 1e6)
        self.model = QwenMoe(cfg, resident, MemorySource())
        self.kernel = kernel
        self._i8 = i8mod
        self._timings = StepTimings
        i8mod.set_kernel(kernel)  # the fused kernel compiles here (numba)

    def __call__(self, x: np.ndarray) -> np.ndarray:
        self._i8.set_kernel(self.kernel)
        return self.model._moe(0, np.ascontiguousarray(x, dtype=np.float32), self._timings(), None, None)


def _time_calls(fn, x, budget_s: float, max_calls: int = 5) -> list[float]:
    times = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        fn(x)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s or len(times) >= max_calls:
            return times


def _sample_tokens(fn, x: np.ndarray, per_call_s: float) -> int:
    """Tokens per call so that one call takes about per_call_s (at least
    256, at most all of x), from a timed call on 256 tokens."""
    n = x.shape[0]
    probe = min(n, 256)
    t0 = time.perf_counter()
    fn(x[:probe])
    dt = max(time.perf_counter() - t0, 1e-6)
    return int(min(n, max(probe, probe * per_call_s / dt)))


def cpu_baseline(block, x: np.ndarray, budget_s: float) -> dict:
    """The reference's own block (both int8 kernels) and the oracle port,
    timed on this host's cores on a bounded sample of the workload's tokens;
    `value` is the reference with its default kernel."""
    cores = host_cores()
    threads = pin_cpu_threads(cores)
    out = {"unit": "tokens/s", "cores": cores, "threads": threads, "host": cpu_model()}
    kernels = {}
    try:
        # one sample size for both kernels (per-token cost depends on rows per expert)
        n = None
        for kernel in ("blocked", "fused"):
            ref = ReferenceBlock(block, kernel)
            if n is None:
                n = _sample_tokens(ref, x, budget_s / 5)
            times = _time_calls(ref, x[:n], budget_s / 3, max_calls=3)
            med = statistics.median(times)
            kernels[kernel] = {"value": n / med, "tokens": n, "calls": len(times), "median_ms": med * 1e3}
        out.update({"value": kernels["fused"]["value"], "kind": "reference", "kernels": kernels,
                    "sample": (f"{kernels['fused']['calls']} x {kernels['fused']['tokens']} tokens of the same "
                               f"workload through the reference's QwenMoe._moe (baseline/_ref, unmodified), int8 "
                               f"kernel 'fused' (its runtime default); 'blocked' in kernels; {cores} host threads")})
    except (ImportError, ValueError) as e:
        out["reference_unavailable"] = f"{type(e).__name__}: {e}"[:200]
    from oracle import moe_oracle as O
    from oracle.blocks import oracle_weights

    w = oracle_weights(block)

    def port(xs):
        return O.moe_block(xs, w)

    n = _sample_tokens(port, x, budget_s / 5)
    times = _time_calls(port, x[:n], budget_s / 3, max_calls=3)
    med = statistics.median(times)
    out["port"] = {"value": n / med, "tokens": n, "calls": len(times), "median_ms": med * 1e3,
                   "what": "oracle/moe_oracle.py: numpy/BLAS restatement of QwenMoe._moe, blocked int8 kernel"}
    if "value" not in out:
        out.update({"value": out["port"]["value"], "kind": "port",
                    "sample": f"{len(times)} x {n} tokens through the oracle port; {cores} host threads"})
    return out


# ---------------------------------------------------------------------------
# the reference arm
# ---------------------------------------------------------------------------


def run_reference_arm(args) -> None:
    """--impl reference: the reference's own QwenMoe._moe (baseline/_ref,
    its default int8 kernel) on this host's cores, on the workload our arm
    measures at this GPU count, each step a bounded sample of its tokens.
    Under torchrun only rank 0 runs; the other ranks exit at once."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from expertrelay_b200 import synth

    world = args.gpus
    workload = arm_workload(args, world)
    if workload == EP_WORKLOAD:
        # the expert-parallel layer: the same block and near-uniform routing
        # (the router without the Zipf scaling), tokens of that layer
        import dataclasses

        block, _ = synth.make_workload("prefill4096_int8_zipf", seed=args.seed)
        block = dataclasses.replace(block, router=block.meta.get("router_base", block.router), meta={})
        x = synth.make_tokens(args.seed * 1000 + 577, 4096, block.hidden)
        tokens_total = args.ep_tokens
    else:
        block, x = synth.make_workload(workload, seed=args.seed)
        tokens_total = x.shape[0]
    cores = host_cores()
    threads = pin_cpu_threads(cores)
    try:
        fn = ReferenceBlock(block, "fused")
        kind, what = "reference", "the reference's QwenMoe._moe (baseline/_ref, unmodified), int8 kernel 'fused'"
    except (ImportError, ValueError) as e:
        from oracle import moe_oracle as O
        from oracle.blocks import oracle_weights

        w = oracle_weights(block)

        def fn(xs):
            return O.moe_block(xs, w)

        kind, what = "port", f"the oracle port of QwenMoe._moe (reference unavailable: {e})"[:200]
    # each step at most about 120 s / (steps + warm-up) of CPU work (the whole
    # batch when that fits), so the run ends within a few minutes
    sample = _sample_tokens(fn, x, 120.0 / max(args.steps + args.warmup, 1))
    xs = x[:sample]
    for _ in range(args.warmup):
        fn(xs)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        fn(xs)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = sample * args.steps / total
    line = {
        "impl": "reference",
        "metric": "MoE-block tokens/s",
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": total / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic: seeded N(0,0.02) weights in store encodings, N(0,1) activations",
        "config": {"workload": workload, "tokens": tokens_total, "tokens_per_step": sample,
                   "hidden": block.hidden, "experts": block.num_experts, "top_k": block.top_k,
                   "expert_format": block.fmt},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": kind, "threads": threads,
                         "sample": f"{sample} of the workload's tokens per step through {what}; {cores} host "
                                   f"threads on {cpu_model()}"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference_arm(args)
        return

    import torch
    import torch.distributed as dist

    from expertrelay_b200 import _lib, synth
    from expertrelay_b200.moe import HostPipeline, MoeBlock

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    path = {"auto": _lib.PATH_AUTO, "gemv": _lib.PATH_GEMV, "gemm": _lib.PATH_GEMM, "tc": _lib.PATH_TC}[args.path]
    act_dtype = torch.bfloat16 if args.act_dtype == "bf16" else torch.float32
    act_bytes = 2 if args.act_dtype == "bf16" else 4

    # weights are identical on every rank (same seed); each rank has its own tokens
    block, x = synth.make_workload(args.workload, seed=args.seed)
    if rank:
        x = synth.make_tokens(args.seed + 7919 * rank, x.shape[0], block.hidden)
    n = x.shape[0]
    mb = MoeBlock.from_host_block(block, device=dev)
    h_dev = torch.from_numpy(x).to(dev).to(act_dtype)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stage_ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(_lib.MOE_STAGES) + 1)]
    for ev in stage_ev:
        ev.record()
    torch.cuda.synchronize()

    # routing of this batch (for the accounting) and warm-up
    _, _, idx, _ = mb.forward(h_dev, path=path, return_routing=True)
    acct = accounting(block, n, idx.cpu().numpy(), act_bytes)
    for _ in range(max(args.warmup, 3)):
        mb.forward(h_dev, path=path)
    torch.cuda.synchronize()

    # the forward captured once as a CUDA graph (no host work per step); a
    # second capture carries CUDA events between the stages, for the live
    # per-stage times (event nodes between kernels would break the kernels'
    # chained launches, so the step time comes from the first)
    cap = mb.capture(n, dtype=act_dtype, path=path)
    cap_st = mb.capture(n, dtype=act_dtype, path=path, stage_events=stage_ev)
    cap.h.copy_(h_dev)
    cap_st.h.copy_(h_dev)
    for _ in range(max(args.warmup, 3)):
        cap.replay()
        cap_st.replay()
    torch.cuda.synchronize()

    # timed region: K steps, each after an L2 flush, bracketed by barrier + sync
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    stage_ms = {s: 0.0 for s in _lib.MOE_STAGES}
    launches = C.c_int(0)
    launches_per_forward = C.c_int(0)
    mb.forward(h_dev, path=path, launch_counter=launches_per_forward)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev) as clocks:
        for i in range(args.steps):
            flush.zero_()
            starts[i].record()
            cap.replay()
            ends[i].record()
            launches.value += launches_per_forward.value
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    # the stage pass: the same steps through the capture with stage events
    for i in range(args.steps):
        flush.zero_()
        cap_st.replay()
        stage_ev[-1].synchronize()
        for j, s in enumerate(_lib.MOE_STAGES):
            stage_ms[s] += stage_ev[j].elapsed_time(stage_ev[j + 1])
    torch.cuda.synchronize()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = sum(step_ms)
    t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms_max = float(t.item())
    value = world * n * args.steps / (total_ms_max / 1e3)
    stage_avg = {s: v / args.steps for s, v in stage_ms.items()}

    # the same steps without the graph: one ctypes call and its launches per step
    eager_ms = 0.0
    for i in range(args.steps):
        flush.zero_()
        starts[i].record()
        mb.forward(h_dev, path=path)
        ends[i].record()
    torch.cuda.synchronize()
    eager_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps

    # end to end through the public API: pinned host tokens in, host output back
    x_host = torch.from_numpy(x).to(act_dtype).pin_memory()
    y_host = torch.empty((n, block.hidden), dtype=torch.float32).pin_memory()
    e_start = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    e_end = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for _ in range(2):
        cap.run_host(x_host, y_host)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    for i in range(args.steps):
        flush.zero_()
        e_start[i].record()
        cap.run_host(x_host, y_host)
        e_end[i].record()
    torch.cuda.synchronize()
    e2e_ms = sum(s.elapsed_time(e) for s, e in zip(e_start, e_end))
    t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
    e2e_serial_value = world * n * args.steps / (float(t.item()) / 1e3)

    # the same host-to-host steps through HostPipeline: step i + 1's input copy
    # and step i - 1's output copy overlap step i's compute (two graph slots,
    # copy-in / compute / copy-out streams); every step's copies stay inside
    # the timed region, from the first input copy to the last output copy
    pipe = HostPipeline(mb, n, dtype=act_dtype, path=path, depth=2)
    y_hosts = [y_host, torch.empty((n, block.hidden), dtype=torch.float32).pin_memory()]
    for i in range(max(args.warmup, 3)):
        pipe.submit(x_host, y_hosts[i % 2])
    pipe.sync()
    if world > 1:
        dist.barrier()
    p_start, p_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p_start.record(pipe.s_in)
    for i in range(args.steps):
        pipe.submit(x_host, y_hosts[i % 2])
    p_end.record(pipe.s_out)
    pipe.sync()
    t = torch.tensor([p_start.elapsed_time(p_end)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
    e2e_pipe_ms = float(t.item())
    e2e_pipe_value = world * n * args.steps / (e2e_pipe_ms / 1e3)
    # the line's e2e is the faster of the two ways a caller runs host batches
    # (the pipeline's three streams and events cost more than they hide on
    # small decode batches); both are reported
    e2e_mode = "pipelined" if e2e_pipe_value >= e2e_serial_value else "serial"
    e2e_value = max(e2e_pipe_value, e2e_serial_value)
    del pipe

    # roofline of the dominant stage
    peaks, peak_src = load_peaks()
    dom = max(("gate_up", "down"), key=lambda s: stage_avg[s])
    tensor_bound = n >= 256
    if tensor_bound:
        # the timed region is a few ms of short steps: the burst GEMM peak is
        # the denominator; the sustained (power-capped) one rides beside it
        work = acct["gate_up_flops"] if dom == "gate_up" else acct["down_flops"]
        achieved = work / (stage_avg[dom] / 1e3) / 1e12
        peak = peaks["bf16_tflops"]
        roof = {"bound": "tensor", "unit": "TFLOP/s", "kernel": dom, "algorithmic_flops_per_launch": work,
                "peak_kind": "burst bf16 GEMM", "frac_of_sustained": achieved / peaks["bf16_tflops_sustained"]}
    else:
        work = acct["gate_up_bytes"] if dom == "gate_up" else acct["down_bytes"]
        achieved = work / (stage_avg[dom] / 1e3) / 1e9
        peak = peaks["hbm_gbs"]
        roof = {"bound": "hbm", "unit": "GB/s", "kernel": dom, "algorithmic_bytes_per_launch": work,
                "peak_kind": "copy bandwidth"}
    traffic, traffic_src = traffic_from_profiles(args.workload, dom)
    roof.update({"achieved": achieved, "peak": peak, "frac": achieved / peak, "peak_source": f"of {peak_src}",
                 "traffic": traffic,
                 "traffic_source": f"ncu capture summarised in {traffic_src}, not this run" if traffic_src else None})

    line = {
        "metric": "MoE-block tokens/s",
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": total_ms_max / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        # arithmetic: fp32 FMA (GEMV / SIMT GEMM) or int8 tensor-core MMA on int8 weights and two
        # int8 activation slices with exact int32 accumulation (tcgen05 path)
        "dtype": "i8" if path == _lib.PATH_TC else "f32",
        "data": "synthetic: seeded N(0,0.02) weights in store encodings, N(0,1) activations",
        "config": {
            "workload": args.workload,
            "tokens": n,
            "hidden": block.hidden,
            "experts": block.num_experts,
            "top_k": block.top_k,
            "expert_format": block.fmt,
            "activations": args.act_dtype,
            "path": args.path,
            "parallelism": f"replicas{world}" if world > 1 else "single",
            "l2": "flushed before every timed step (256 MiB write)",
        },
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": int(n * block.hidden * act_bytes),
                "d2h_bytes_per_step": int(n * block.hidden * 4), "mode": e2e_mode,
                "ms_per_step": world * n / e2e_value * 1e3,
                "pipelined_value": e2e_pipe_value,
                "how": "HostPipeline: pinned host tokens in, pinned host output back every step; step i+1's "
                       "input copy and step i-1's output copy overlap step i's graph; timed from the first "
                       "input copy to the last output copy; no flush (each step streams the expert weights, "
                       "larger than L2)",
                "serial_value": e2e_serial_value,
                "serial_how": "one step at a time on one stream: copy in, graph, copy out; L2 flushed between steps"},
        "gpu_launches": int(launches.value),
        "roofline": roof,
        "stages_ms": stage_avg,
        "graph": "each step replays the forward captured as one CUDA graph (MoeBlock.capture)",
        "eager_ms_per_step": eager_ms,
        "block": {"weight_bytes": acct["block_weight_bytes"], "flops": acct["block_flops"],
                  "unique_experts": acct["unique_experts"],
                  "weight_GBps": acct["block_weight_bytes"] / (total_ms_max / args.steps / 1e3) / 1e9,
                  "TFLOPs": acct["block_flops"] / (total_ms_max / args.steps / 1e3) / 1e12},
        "clocks": clocks.summary(),
    }
    if block.meta.get("zipf"):
        line["config"]["zipf_histogram"] = block.meta["zipf"]["realised"]

    if rank == 0 and world == 1 and not args.no_decode and args.workload != "decode8_int8":
        line["decode"] = decode_side(args, dev, mb, block, peaks, peak_src)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(block, x, args.cpu_seconds)
    if rank == 0 and world == 1 and not args.no_gptq:
        try:
            line["gptq"] = gptq_side(args, dev, peaks, peak_src)
        except (RuntimeError, ValueError, MemoryError) as e:  # reported, the main line still prints
            line["gptq"] = {"error": f"{type(e).__name__}: {e}"[:400]}
    if not args.no_ep:
        ep_line = expert_parallel_side(args, dev, block, world, rank, flush)
        line["expert_parallel"] = ep_line
        if world > 1 and "error" not in ep_line:
            # several GPUs: the headline is the sharded layer; the independent
            # replicas of the block stay beside it
            line["replicas"] = {"value": line["value"], "ms_per_step": line["ms_per_step"], "e2e": line["e2e"],
                                "workload": f"{args.workload} on every GPU independently (no collective)"}
            line["metric"] = "MoE-layer tokens/s (expert-parallel)"
            line["value"] = ep_line["value"]
            line["ms_per_step"] = ep_line["ms_per_step"]
            line["steps"] = ep_line["steps"]
            line["scaling"] = "strong"
            line["e2e"] = {k: ep_line["e2e"][k] for k in ("value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step")}
            line["gpu_launches"] = ep_line["gpu_launches_per_step"] * ep_line["steps"]
            line["dtype"] = "i8"
            line["config"] = {"workload": EP_WORKLOAD, "tokens": args.ep_tokens, "hidden": block.hidden,
                              "experts": block.num_experts, "top_k": block.top_k, "expert_format": block.fmt,
                              "activations": "bf16", "results": "bf16", "path": "tc",
                              "parallelism": f"ep{world}", "microbatch": ep_microbatch(args, world),
                              "l2": "flushed before every timed step (256 MiB write)"}
            line["clocks"] = ep_line["clocks"]
    if rank == 0 and world == 1 and not args.no_full_model:
        del mb
        torch.cuda.empty_cache()
        try:
            line["full_model"] = full_model_side(args, dev)
        except (RuntimeError, ValueError, OSError, MemoryError) as e:  # reported, the main line still prints
            line["full_model"] = {"error": f"{type(e).__name__}: {e}"[:400]}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        line["summary"] = summary_of(line)  # last, so a tail of the output keeps it
        print(json.dumps(line), flush=True)


def summary_of(line: dict) -> dict:
    """The side measurements' key figures in a few short keys."""

    def pick(d, *keys):
        for k in keys:
            if not isinstance(d, dict) or k not in d:
                return None
            d = d[k]
        return round(d, 4) if isinstance(d, float) else d

    out = {"value": pick(line, "value"), "frac": pick(line, "roofline", "frac"),
           "e2e": pick(line, "e2e", "value"), "cpu": pick(line, "cpu_baseline", "value")}
    if "decode" in line:
        out["decode8"] = {"path": pick(line, "decode", "best_path"), "ms": pick(line, "decode", "ms_per_block"),
                          "gate_up_hbm_frac": pick(line, "decode", "roofline", "frac"),
                          "block_GBps": pick(line, "decode", "block_weight_GBps")}
    if "gptq" in line:
        for k in ("decode1", "prefill512"):
            out[f"gptq_{k}"] = {"path": pick(line, "gptq", k, "path"), "ms": pick(line, "gptq", k, "ms_per_block"),
                                "hbm_frac": pick(line, "gptq", k, "hbm", "frac"),
                                "tensor_frac": pick(line, "gptq", k, "tensor", "frac"),
                                "gate_up_hbm_frac": pick(line, "gptq", k, "expert_kernels", "gate_up", "hbm_frac"),
                                "gate_up_tensor_frac": pick(line, "gptq", k, "expert_kernels", "gate_up",
                                                            "tensor_frac")}
    if "expert_parallel" in line:
        out["ep"] = {"value": pick(line, "expert_parallel", "value"), "ms": pick(line, "expert_parallel", "ms_per_step"),
                     "nvlink_GBps": pick(line, "expert_parallel", "nvlink", "GBps"),
                     "phases_ms": {k: round(v, 3) for k, v in (line["expert_parallel"].get("phases_ms") or {}).items()}}
    if "full_model" in line:
        out["full_model_tok_s"] = pick(line, "full_model", "decode_tokens_per_s")
    return out


def ep_microbatch(args, world: int) -> int:
    """Tokens per microbatch of the expert-parallel layer: --ep-microbatch, or
    half a rank's tokens (two microbatches, so one's exchange overlaps the
    other's experts) kept within 4096..16384 (measured at 2 GPUs: 8.0, 8.9
    and 9.5 M tokens/s at 4096, 8192 and 16384)."""
    if args.ep_microbatch > 0:
        return args.ep_microbatch
    per = max(1, args.ep_tokens // world)
    mb = 4096
    while mb * 2 <= min(16384, per // 2) and per % (mb * 2) == 0:
        mb *= 2
    return mb


def expert_parallel_side(args, dev, block, world: int, rank: int, flush) -> dict:
    """The MoE layer of the expert-parallel prefill workload: 32 sequences x
    2048 tokens (65,536, --ep-tokens) split evenly over the ranks (the total
    is fixed: strong scaling), bf16 activations, the block's router without
    the Zipf scaling (a random-init model routes near-uniformly). The 60
    experts are spread contiguously over the ranks (30/30, 15 x 4,
    8,8,8,8,7,7,7,7); each rank runs ExpertParallelMoe on the tensor-core
    path in microbatches of --ep-microbatch: one exchange of counts, then the
    rows (bf16) with their expert ids and weights out and the results (bf16)
    back, asynchronously so that the transfers overlap the expert GEMMs, the
    gated shared expert on a side stream, and the ordered combine. On one GPU
    there is nothing to exchange and the layer runs as the block.

    Timed: `value` from CUDA events around each step (max over ranks);
    `e2e` the same steps with each rank's tokens copied in from pinned host
    memory and its output copied back inside the timed region; `phases`
    one extra step with the steps run one after another and timed apart
    (max over ranks). Every rank takes the same collective steps; a failure
    while building is agreed on first, so that no rank waits in a collective
    for one that gave up."""
    import dataclasses

    import torch
    import torch.distributed as dist

    from expertrelay_b200 import _lib
    from expertrelay_b200.ep import EpCudaOps, ExpertParallelMoe, expert_partition

    total, mbatch = args.ep_tokens, ep_microbatch(args, world)
    per = total // world
    chunks = max(1, per // mbatch)
    err = None
    try:
        if per % mbatch:
            raise ValueError(f"{per} tokens per rank are not a multiple of the {mbatch}-token microbatch")
        ep_block = dataclasses.replace(block, router=block.meta.get("router_base", block.router), meta={})
        ops = EpCudaOps(ep_block, rank, world, dev, _lib.PATH_TC, return_bf16=True)
        ep = ExpertParallelMoe(ops)
        gen = torch.Generator(device=dev)
        gen.manual_seed(args.seed * 1000 + 577 + rank)
        h = torch.randn((per, block.hidden), generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)
    except (RuntimeError, ValueError, MemoryError) as e:
        err = f"{type(e).__name__}: {e}"[:300]
    bad = torch.tensor([1 if err else 0], dtype=torch.int32, device=dev)
    if world > 1:
        dist.all_reduce(bad, op=dist.ReduceOp.MAX)
    if int(bad.item()):
        return {"error": err or "another rank failed to set up"}

    parts = [h[c * mbatch:(c + 1) * mbatch] for c in range(chunks)]

    def step(stats=None):
        out = ep.forward_many(parts)
        if stats is not None:
            send, recv = ep.last_counts
            stats[0] += sum(v for r, v in enumerate(send) if r != rank)
            stats[1] += sum(v for r, v in enumerate(recv) if r != rank)
            stats[2] += sum(recv)
        return out

    for _ in range(max(args.warmup, 3)):
        step()
    steps = max(3, min(args.steps, args.ep_steps))
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    stats = [0, 0, 0]  # rows this rank sent to other ranks, got from them, computed
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    with ClockSampler(dev) as clocks:
        for i in range(steps):
            flush.zero_()
            starts[i].record()
            step(stats if i == 0 else None)
            ends[i].record()
        torch.cuda.synchronize()
    step_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / steps

    # end to end: this rank's tokens in from pinned host memory, its output back
    h_host = h.cpu().pin_memory()
    y_host = torch.empty((per, block.hidden), dtype=torch.float32).pin_memory()

    def step_e2e():
        h.copy_(h_host, non_blocking=True)
        out = step()
        for c, y in enumerate(out):
            y_host[c * mbatch:(c + 1) * mbatch].copy_(y, non_blocking=True)

    step_e2e()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    for i in range(steps):
        flush.zero_()
        starts[i].record()
        step_e2e()
        ends[i].record()
    torch.cuda.synchronize()
    e2e_serial_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / steps

    # the same, pipelined over steps: step i+1's tokens are copied in (copy
    # stream, second device buffer) and step i-1's output copied out (another
    # stream) while step i runs; timed from the first input copy to the last
    # output copy
    cur = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    h_bufs = [h, torch.empty_like(h)]
    in_done = [torch.cuda.Event() for _ in range(2)]
    run_done = [torch.cuda.Event() for _ in range(2)]
    for s_ in (s_in, s_out):
        s_.wait_stream(cur)

    def copy_in(i):
        b = i % 2
        if i >= 2:
            s_in.wait_event(run_done[b])  # step i-2 read this buffer
        with torch.cuda.stream(s_in):
            h_bufs[b].copy_(h_host, non_blocking=True)
            in_done[b].record(s_in)

    def run_pipelined(n_steps, start=None, end=None):
        if start is not None:
            start.record(s_in)
        copy_in(0)
        for i in range(n_steps):
            if i + 1 < n_steps:
                copy_in(i + 1)
            b = i % 2
            cur.wait_event(in_done[b])
            out = ep.forward_many([h_bufs[b][c * mbatch:(c + 1) * mbatch] for c in range(chunks)])
            run_done[b].record(cur)
            s_out.wait_event(run_done[b])
            with torch.cuda.stream(s_out):
                for c, y in enumerate(out):
                    y.record_stream(s_out)
                    y_host[c * mbatch:(c + 1) * mbatch].copy_(y, non_blocking=True)
        if end is not None:
            end.record(s_out)
        for s_ in (s_in, s_out):
            cur.wait_stream(s_)

    run_pipelined(2)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    p_start, p_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    run_pipelined(steps, p_start, p_end)
    torch.cuda.synchronize()
    e2e_ms = p_start.elapsed_time(p_end) / steps

    # one more step with its steps timed apart
    phases: dict = {}
    if world > 1:
        dist.barrier()
    ep.forward_many(parts, phases=phases)
    torch.cuda.synchronize()
    keys = ["route", "counts", "shared", "pack", "dispatch", "rows", "return", "combine"]
    t = torch.tensor([step_ms, e2e_ms, stats[2], stats[0], stats[1], e2e_serial_ms]
                     + [phases.get(k, 0.0) for k in keys], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_max, rows_max, sent_max, got_max, e2e_serial_max = (float(v) for v in t[:6].tolist())
    row_out = block.hidden * 2 + 8  # bf16 row + expert id + weight
    row_back = block.hidden * 2  # bf16 result
    link_bytes = sent_max * row_out + got_max * row_back  # bytes one rank pushes out over NVLink per step (max)
    # kernels per step: router, top-k, count, pack, rows (dispatch, gate/up, slices, down, combine, plus its
    # tally), shared expert (gate logit, sigmoid, dispatch, gate/up, slices, down, combine), combine
    launches = chunks * (2 + 1 + 1 + 6 + 7 + 1) if world > 1 else chunks * 7
    return {
        "workload": (f"MoE layer of the expert-parallel prefill: {total} tokens (32 x 2048) over {world} GPU(s), "
                     f"{per} per rank in {chunks} microbatch(es) of {mbatch}; int8 experts, bf16 activations and "
                     f"results, near-uniform routing"),
        "value": total / (ms / 1e3),
        "unit": "tokens/s",
        "ms_per_step": ms,
        "steps": steps,
        "scaling": "strong",
        "e2e": {"value": total / (e2e_max / 1e3), "unit": "tokens/s", "ms_per_step": e2e_max,
                "h2d_bytes_per_step": int(per * block.hidden * 2), "d2h_bytes_per_step": int(per * block.hidden * 4),
                "how": "each rank's tokens in from pinned host memory and its output back every step, step i+1's "
                       "input copy and step i-1's output copy overlapping step i; first input copy to last "
                       "output copy, max over ranks; no flush (each step streams the expert weights)",
                "serial_value": total / (e2e_serial_max / 1e3),
                "serial_how": "one step at a time, copies on the compute stream, L2 flushed between steps"},
        "phases_ms": {k: float(v) for k, v in zip(keys, t[6:].tolist())},
        "phases_timing": "one step with its steps run one after another (not overlapped), max over ranks",
        "experts_per_rank": [hi - lo for lo, hi in expert_partition(block.num_experts, world)],
        "rows_computed_max_rank": int(rows_max),
        "nvlink": {"bytes_out_per_step_max_rank": int(link_bytes),
                   "GBps": link_bytes / (ms / 1e3) / 1e9 if world > 1 else 0.0,
                   "peak_GBps": 770.0, "peak_source": "measured peer copy per direction on this pool"},
        "gpu_launches_per_step": launches,
        "collectives": ("NCCL all_to_all_single: counts, rows, ids + weights (one int32 buffer), results; "
                        "asynchronous, overlapping the expert GEMMs") if world > 1 else "none (the block)",
        "timing": "CUDA events around each step (host waits for the counts included), max over ranks, L2 flushed",
        "clocks": clocks.summary(),
    }


def full_model_side(args, dev) -> dict:
    """Whole-model greedy decoding (Qwen1.5-MoE-A2.7B shapes, random init):
    a seeded uniform prompt in one call, then one token per call; routed
    experts paged through an HBM cache of cache_frac of the records from
    pinned host memory, with the Fate prefetch. Decode tokens/s counts the
    one-token calls (each a full forward: embedding, 24 layers, lm_head)."""
    import torch

    from expertrelay_b200 import synth
    from expertrelay_b200.model import QwenMoeModel

    cfg = dict(synth.QWEN_MODEL, num_hidden_layers=args.model_layers)
    t0 = time.perf_counter()
    host, records = synth.make_model_gpu(cfg, seed=args.seed + 17, device=dev)
    t_build = time.perf_counter() - t0
    n_records = records.shape[0] * records.shape[1]
    slots = max(cfg["num_experts"] + 1, int(round(args.cache_frac * n_records)))
    model = QwenMoeModel(host, records=records, cache_records=slots, prefetch=True, device=dev)
    prompt = np.random.default_rng(args.seed + 4242).integers(0, cfg["vocab_size"], args.prompt_tokens)
    model.generate(prompt[:16], 4)  # warm-up: kernels, allocator, cache bookkeeping
    keys = ("loads", "demand_reads", "cache_hits", "prefetch_hits", "prefetch_waits", "prefetches_issued",
            "prefetch_reads", "prefetches_wasted", "prefetches_skipped_budget")

    def run():
        s0 = model.cache.stats
        out = model.generate(prompt, args.new_tokens)
        s1 = model.cache.stats
        return out, {k: getattr(s1, k) - getattr(s0, k) for k in keys}

    (tokens, t_prompt, steps), delta = run()
    # the same generation with the adaptive read budget (prefetch copies capped per layer window)
    model.stack.prefetch_adaptive = True
    (tokens_a, _, steps_a), delta_a = run()
    win = model.stack.window[:-1]
    adaptive = {
        "decode_tokens_per_s": (len(steps_a) / float(np.sum(steps_a))) if steps_a else None,
        "ms_per_decode_token": float(np.sum(steps_a)) / max(len(steps_a), 1) * 1e3,
        "same_tokens": tokens_a == tokens,
        "record_copy_ms": model.stack.read_seconds * 1e3 if model.stack.read_seconds else None,
        "window_ms_median": float(np.median(win[np.isfinite(win)])) * 1e3 if np.isfinite(win).any() else None,
        "cache": delta_a,
    }
    rs = model.records.layout.record_size
    dec_s = float(np.sum(steps))
    model.close()
    return {
        "workload": (f"Qwen1.5-MoE-A2.7B shapes, random init, {cfg['num_hidden_layers']} layers, int8 experts; "
                     f"{args.prompt_tokens}-token seeded uniform prompt, {args.new_tokens} greedy tokens, batch 1; "
                     f"HBM expert cache {slots} of {n_records} records, the rest in pinned host RAM, Fate prefetch"),
        "decode_tokens_per_s": (len(steps) / dec_s) if steps else None,
        "ms_per_decode_token": dec_s / max(len(steps), 1) * 1e3,
        "decode_ms_p50": float(np.median(steps)) * 1e3 if steps else None,
        "prompt_ms": t_prompt * 1e3,
        "prompt_tokens_per_s": args.prompt_tokens / t_prompt,
        "expert_bytes_copied_GB": (delta["demand_reads"] + delta["prefetch_reads"]) * rs / 1e9,
        "cache": delta,
        "adaptive_budget": adaptive,
        "build_s": t_build,
        "timing": "host wall clock around each generate() call (synchronous: argmax read back per token)",
    }


def gptq_side(args, dev, peaks, peak_src) -> dict:
    """The MoE block with int4 GPTQ-style routed experts (asymmetric 4-bit,
    group 128 along the input, fp16 scales, 4-bit zero points; the shared
    expert int8), at 1 decode token and at 512 tokens, on the tcgen05 path
    (the default for these records) and, for comparison, on the exact-fp32
    weight-streaming GEMV (1 token) / SIMT GEMM (512 tokens). Each step
    replays the captured forward after an L2 flush. Both report the block's
    algorithmic weight bytes against HBM and its FLOPs against dense bf16
    (512 tokens sits near the ridge between the two); the gate/up and down
    kernels are also timed alone (stage events in a second capture)."""
    import torch

    from expertrelay_b200 import _lib, synth
    from expertrelay_b200.moe import MoeBlock

    block, _ = synth.make_workload("gptq_asym_decode1", seed=args.seed)
    mb = MoeBlock.from_host_block(block, device=dev)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(_lib.MOE_STAGES) + 1)]
    for e in ev:
        e.record()
    steps = max(args.steps, 20)
    out = {}
    cases = (("decode1", 1, (("tc", _lib.PATH_TC), ("gemv", _lib.PATH_GEMV))),
             ("prefill512", 512, (("tc", _lib.PATH_TC), ("gemm", _lib.PATH_GEMM))))
    for name, n, paths in cases:
        h = torch.from_numpy(synth.make_tokens(args.seed, n, block.hidden)).to(dev)
        _, _, idx, _ = mb.forward(h, path=_lib.PATH_TC, return_routing=True)
        acct = accounting(block, n, idx.cpu().numpy(), 4)
        res = {}
        for pname, path in paths:
            cap = mb.capture(n, path=path)
            cap_st = mb.capture(n, path=path, stage_events=ev)
            cap.h.copy_(h)
            cap_st.h.copy_(h)
            for _ in range(max(args.warmup, 3)):
                cap.replay()
                cap_st.replay()
            torch.cuda.synchronize()
            tot = 0.0
            stage = {s: 0.0 for s in _lib.MOE_STAGES}
            for _ in range(steps):
                flush.zero_()
                t0.record()
                cap.replay()
                t1.record()
                t1.synchronize()
                tot += t0.elapsed_time(t1)
                flush.zero_()
                cap_st.replay()
                ev[-1].synchronize()
                for j, s in enumerate(_lib.MOE_STAGES):
                    stage[s] += ev[j].elapsed_time(ev[j + 1])
            sec = tot / steps / 1e3
            stage = {s: v / steps for s, v in stage.items()}
            gbs = acct["block_weight_bytes"] / sec / 1e9
            tfs = acct["block_flops"] / sec / 1e12
            kern = {
                "gate_up": {"ms": stage["gate_up"],
                            "GBps": acct["gate_up_bytes"] / (stage["gate_up"] / 1e3) / 1e9,
                            "TFLOPs": acct["gate_up_flops"] / (stage["gate_up"] / 1e3) / 1e12},
                "down": {"ms": stage["down"],
                         "GBps": acct["down_bytes"] / (stage["down"] / 1e3) / 1e9,
                         "TFLOPs": acct["down_flops"] / (stage["down"] / 1e3) / 1e12},
            }
            for k in kern.values():
                k["hbm_frac"] = k["GBps"] / peaks["hbm_gbs"]
                k["tensor_frac"] = k["TFLOPs"] / peaks["bf16_tflops"]
            res[pname] = {
                "tokens": n, "path": pname, "ms_per_block": sec * 1e3, "tokens_per_s": n / sec,
                "unique_experts": acct["unique_experts"],
                "hbm": {"achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": gbs / peaks["hbm_gbs"],
                        "algorithmic_bytes": acct["block_weight_bytes"], "peak_source": f"of {peak_src}"},
                "tensor": {"achieved": tfs, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                           "frac": tfs / peaks["bf16_tflops"], "algorithmic_flops": acct["block_flops"],
                           "peak_kind": "burst bf16 GEMM", "peak_source": f"of {peak_src}"},
                "stages_ms": stage,
                "expert_kernels": kern,
            }
            del cap, cap_st
        best = min(res, key=lambda k: res[k]["ms_per_block"])
        out[name] = {**res[best], "best_path": best,
                     "other_paths": {k: {"ms_per_block": v["ms_per_block"], "hbm_frac": v["hbm"]["frac"],
                                         "tensor_frac": v["tensor"]["frac"]} for k, v in res.items() if k != best}}
    del mb
    torch.cuda.empty_cache()
    return {"workload": "int4 GPTQ-style experts (asymmetric, group 128, fp16 scales, 4-bit zero points), "
                        "int8 shared expert; 1 and 512 tokens", "steps": steps, **out}


def decode_side(args, dev, mb, block, peaks, peak_src) -> dict:
    """Decode shape on the same experts (8 tokens, router without the Zipf
    scaling): block tokens/s and the expert-weight streaming rate of the
    gate/up launch, for the weight-streaming GEMV and the tensor-core path;
    the faster one is the decode result."""
    import torch

    from expertrelay_b200 import _lib, synth

    base_router = block.meta.get("router_base")
    if base_router is not None:
        mb.router.copy_(torch.from_numpy(base_router).to(dev))
    x = synth.make_tokens(args.seed, 8, block.hidden)
    h = torch.from_numpy(x).to(dev)
    _, _, idx, _ = mb.forward(h, path=_lib.PATH_GEMV, return_routing=True)
    acct = accounting(block, 8, idx.cpu().numpy(), 4)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(_lib.MOE_STAGES) + 1)]
    for e in ev:
        e.record()
    steps = max(args.steps, 20)
    results = {}
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for name, path in (("gemv", _lib.PATH_GEMV), ("tc", _lib.PATH_TC)):
        # block time from a capture without events between the stages; stage
        # times from a second capture with them
        cap = mb.capture(8, path=path)
        cap_st = mb.capture(8, path=path, stage_events=ev)
        cap.h.copy_(h)
        cap_st.h.copy_(h)
        for _ in range(5):
            cap.replay()
            cap_st.replay()
        torch.cuda.synchronize()
        tot = 0.0
        stage = {s: 0.0 for s in _lib.MOE_STAGES}
        for _ in range(steps):
            flush.zero_()
            t0.record()
            cap.replay()
            t1.record()
            t1.synchronize()
            tot += t0.elapsed_time(t1)
            flush.zero_()
            cap_st.replay()
            ev[-1].synchronize()
            for j, s in enumerate(_lib.MOE_STAGES):
                stage[s] += ev[j].elapsed_time(ev[j + 1])
        ms = tot / steps
        stage = {s: v / steps for s, v in stage.items()}
        gu_gbs = acct["gate_up_bytes"] / (stage["gate_up"] / 1e3) / 1e9
        results[name] = {
            "tokens_per_s": 8 / (ms / 1e3),
            "ms_per_block": ms,
            "block_weight_GBps": acct["block_weight_bytes"] / (ms / 1e3) / 1e9,
            "roofline": {"bound": "hbm", "kernel": "gate_up", "achieved": gu_gbs, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": gu_gbs / peaks["hbm_gbs"], "peak_source": f"of {peak_src}",
                         "algorithmic_bytes_per_launch": acct["gate_up_bytes"],
                         "traffic": traffic_from_profiles("decode8_int8", "gate_up")[0] if name == "tc" else None,
                         "traffic_source": "ncu capture summarised in profiles/, not this run" if name == "tc" else None},
            "stages_ms": stage,
        }
    if base_router is not None:
        mb.router.copy_(torch.from_numpy(block.router).to(dev))
    best = min(results, key=lambda k: results[k]["ms_per_block"])
    return {"workload": "8 decode tokens, same int8 experts, unscaled router",
            "unique_experts": acct["unique_experts"], "best_path": best, **results[best], "paths": results}


if __name__ == "__main__":
    main()
