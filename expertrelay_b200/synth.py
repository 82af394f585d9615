"""Seeded synthetic MoE blocks and activations with Qwen1.5-MoE-A2.7B shapes.

There are no real checkpoints here, so every benchmark and parity case is
built from a seed: weights ~ N(0, sigma) in float32, then encoded exactly as
the expert store encodes them (expertrelay_b200.quant); activations ~ N(0, 1).

Workloads (hidden 2048, 60 routed experts with intermediate 1408, top-4,
shared expert with intermediate 5632):
  decode8_int8          8 decode tokens, int8 per-channel experts
  prefill4096_int8_zipf 4096 tokens, int8 experts, router rows scaled so the
                        per-expert token counts follow Zipf(s = 1.1)
  gptq_asym_decode1     1 token, asymmetric 4-bit GPTQ-style experts (group 128)
  gptq_asym_prefill512  512 tokens, same experts
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import quant
from .store import FMT_INT4, FMT_INT4_ZP, FMT_INT8, RecordLayout, serialize_record

QWEN = dict(hidden=2048, inter=1408, shared_inter=5632, num_experts=60, top_k=4)

WORKLOADS = {
    "decode8_int8": dict(n=8, fmt="int8", zipf=None),
    "prefill4096_int8_zipf": dict(n=4096, fmt="int8", zipf=1.1),
    "gptq_asym_decode1": dict(n=1, fmt="gptq_asym", zipf=None),
    "gptq_asym_prefill512": dict(n=512, fmt="gptq_asym", zipf=None),
}

FORMATS = {"int8": FMT_INT8, "int4": FMT_INT4, "gptq_asym": FMT_INT4_ZP}


@dataclass
class HostBlock:
    """One MoE layer's weights on the host, in store encodings."""

    hidden: int
    inter: int
    shared_inter: int
    num_experts: int
    top_k: int
    fmt: str  # "int8" | "int4" (store symmetric) | "gptq_asym"
    group: int
    router: np.ndarray  # [E, H] float32 (mlp.gate.weight)
    shared_gate: np.ndarray  # [1, H] float32 (mlp.shared_expert_gate.weight)
    shared: dict  # name -> (int8 q, float32 scales)
    experts: list  # per expert: name -> tuple in the record encoding
    gptq: list | None = None  # per expert: name -> GPTQ v1 tensors (gptq_asym only)
    meta: dict = field(default_factory=dict)

    @property
    def layout(self) -> RecordLayout:
        return RecordLayout(FORMATS[self.fmt], self.hidden, self.inter, self.group if self.fmt != "int8" else 0,
                            "gptq_asym_rtn" if self.fmt == "gptq_asym" else "rtn_absmax7")

    @property
    def shared_layout(self) -> RecordLayout:
        return RecordLayout(FMT_INT8, self.hidden, self.shared_inter)

    def records(self) -> np.ndarray:
        """All routed experts as store records, [E, record_size] uint8."""
        lay = self.layout
        out = np.empty((self.num_experts, lay.record_size), dtype=np.uint8)
        for e, mats in enumerate(self.experts):
            out[e] = serialize_record(lay, mats)
        return out

    def shared_record(self) -> np.ndarray:
        return serialize_record(self.shared_layout, self.shared)

    def weight_bytes_per_expert(self) -> int:
        """Bytes the kernels must read for one routed expert (weights + scales (+ zeros))."""
        lay = self.layout
        return lay.weights_bytes + lay.scales_bytes + lay.zeros_bytes

    def shared_bytes(self) -> int:
        lay = self.shared_layout
        return lay.weights_bytes + lay.scales_bytes


def _normal(rng: np.random.Generator, shape, sigma: float) -> np.ndarray:
    return rng.standard_normal(shape, dtype=np.float32) * np.float32(sigma)


def make_block(
    seed: int = 0,
    *,
    hidden: int = QWEN["hidden"],
    inter: int = QWEN["inter"],
    shared_inter: int = QWEN["shared_inter"],
    num_experts: int = QWEN["num_experts"],
    top_k: int = QWEN["top_k"],
    fmt: str = "int8",
    group: int = 128,
    sigma: float = 0.02,
) -> HostBlock:
    """Seeded weights ~ N(0, sigma), router and shared gate kept float32, the
    shared expert int8, routed experts in `fmt`. Generation order (one
    generator): router, shared gate, shared gate/up/down, then per expert
    gate/up/down."""
    if fmt not in FORMATS:
        raise ValueError(f"unknown format {fmt!r}")
    rng = np.random.default_rng(seed)
    router = _normal(rng, (num_experts, hidden), sigma)
    shared_gate = _normal(rng, (1, hidden), sigma)
    shapes = {"gate_proj": (inter, hidden), "up_proj": (inter, hidden), "down_proj": (hidden, inter)}
    sh_shapes = {"gate_proj": (shared_inter, hidden), "up_proj": (shared_inter, hidden), "down_proj": (hidden, shared_inter)}
    shared = {m: quant.int8_rowwise(_normal(rng, s, sigma)) for m, s in sh_shapes.items()}
    experts, gptq = [], ([] if fmt == "gptq_asym" else None)
    for _ in range(num_experts):
        mats, gt = {}, {}
        for m, s in shapes.items():
            w = _normal(rng, s, sigma)
            if fmt == "int8":
                mats[m] = quant.int8_rowwise(w)
            elif fmt == "int4":
                v, sc = quant.int4_rtn_absmax7(w, group)
                mats[m] = (quant.pack_nibbles(v), sc)
            else:
                t = quant.gptq_asym_rtn(w, group)
                gt[m] = t
                mats[m] = quant.gptq_to_zp_matrix(t, group)
        experts.append(mats)
        if gptq is not None:
            gptq.append(gt)
    return HostBlock(hidden, inter, shared_inter, num_experts, top_k, fmt, group if fmt != "int8" else 0, router,
                     shared_gate, shared, experts, gptq, {"seed": seed, "sigma": sigma})


def make_tokens(seed: int, n: int, hidden: int = QWEN["hidden"]) -> np.ndarray:
    """Activations ~ N(0, 1), float32 [n, hidden], from their own generator."""
    return np.random.default_rng(seed + 1_000_003).standard_normal((n, hidden), dtype=np.float32)


def zipf_targets(num_experts: int, total: int, n: int, s: float, seed: int, cap_frac: float = 0.45) -> np.ndarray:
    """Per-expert target counts proportional to rank^-s over a seeded ranking,
    summing to `total`, each capped at cap_frac * n (a router over zero-mean
    inputs picks an expert for at most about half of the tokens; the excess
    is spread over the others in proportion)."""
    rank = np.random.default_rng(seed + 7).permutation(num_experts)  # expert -> rank (0 = most popular)
    t = (rank + 1.0) ** (-s)
    t = t / t.sum() * total
    cap = cap_frac * n
    for _ in range(num_experts):
        over = t > cap + 1e-9
        if not over.any():
            break
        excess = float((t[over] - cap).sum())
        t[over] = cap
        free = ~over & (t < cap)
        t[free] += excess * t[free] / t[free].sum()
    return t


def apply_zipf_routing(block: HostBlock, x: np.ndarray, s: float = 1.1, seed: int = 0, iters: int = 120) -> dict:
    """Scale router rows W_r[e] *= c_e so the top-k counts over `x` follow
    Zipf(s). Deterministic (fixed-step multiplicative fit on the logits).
    Modifies block.router in place; returns the realised histogram."""
    n, E, k = x.shape[0], block.num_experts, block.top_k
    base = x @ block.router.T  # scaling a row scales that expert's logits
    target = zipf_targets(E, n * k, n, s, seed)
    c = np.ones(E, dtype=np.float64)
    for _ in range(iters):
        sel = np.argpartition(-(base * c.astype(np.float32)), k - 1, axis=1)[:, :k]
        counts = np.bincount(sel.ravel(), minlength=E)
        c *= (target / np.maximum(counts, 0.5)) ** 0.3
        np.clip(c, 1e-3, 1e3, out=c)
    block.meta["router_base"] = block.router
    block.router = (block.router * c.astype(np.float32)[:, None]).astype(np.float32)
    sel = np.argpartition(-(x @ block.router.T), k - 1, axis=1)[:, :k]
    counts = np.bincount(sel.ravel(), minlength=E)
    block.meta["zipf"] = {"s": s, "target": np.round(target).astype(int).tolist(), "realised": counts.tolist()}
    return block.meta["zipf"]


def make_workload(name: str, seed: int = 0, **overrides) -> tuple[HostBlock, np.ndarray]:
    """(block, activations) for one of WORKLOADS at Qwen shapes (or overridden sizes)."""
    spec = dict(WORKLOADS[name])
    n = overrides.pop("n", spec["n"])
    shape = {k: overrides.pop(k, v) for k, v in QWEN.items()}
    block = make_block(seed, fmt=spec["fmt"], **shape, **overrides)
    x = make_tokens(seed, n, shape["hidden"])
    if spec["zipf"]:
        apply_zipf_routing(block, x, spec["zipf"], seed)
    return block, x


# ---------------------------------------------------------------------------
# the whole decoder (runtime/qwen_moe.py:376-432)
# ---------------------------------------------------------------------------

# Qwen1.5-MoE-A2.7B's config.json fields the forward pass reads
QWEN_MODEL = {
    "vocab_size": 151936,
    "hidden_size": 2048,
    "num_hidden_layers": 24,
    "num_attention_heads": 16,
    "num_key_value_heads": 16,
    "num_experts": 60,
    "num_experts_per_tok": 4,
    "moe_intermediate_size": 1408,
    "shared_expert_intermediate_size": 5632,
    "norm_topk_prob": False,
    "rms_norm_eps": 1e-6,
    "rope_theta": 1e6,
}


@dataclass
class HostLayer:
    """A decoder layer's non-MoE weights: int8 (q, scales) projections, fp32
    q/k/v biases and RMSNorm weights."""

    input_norm: np.ndarray
    post_norm: np.ndarray
    proj: dict  # "q_proj" | "k_proj" | "v_proj" | "o_proj" -> (int8 q, float32 scales)
    bias: dict  # "q_proj" | "k_proj" | "v_proj" -> float32


@dataclass
class HostModel:
    """A whole Qwen2-MoE decoder on the host: config (config.json fields),
    embedding and lm_head as int8 rows, final norm, per-layer weights and
    MoE blocks (routed records included)."""

    config: dict
    embed: tuple
    lm_head: tuple
    final_norm: np.ndarray
    layers: list
    blocks: list

    def tensors(self) -> dict:
        """Checkpoint-named tensors, as the reference's ResidentWeights holds
        them: (q, scales) for int8 matrices, arrays for fp32 ones."""
        out = {"model.embed_tokens.weight": self.embed, "lm_head.weight": self.lm_head,
               "model.norm.weight": self.final_norm}
        for i, (lay, blk) in enumerate(zip(self.layers, self.blocks)):
            p = f"model.layers.{i}."
            out[p + "input_layernorm.weight"] = lay.input_norm
            out[p + "post_attention_layernorm.weight"] = lay.post_norm
            for m, qs in lay.proj.items():
                out[p + f"self_attn.{m}.weight"] = qs
            for m, b in lay.bias.items():
                out[p + f"self_attn.{m}.bias"] = b
            out[p + "mlp.gate.weight"] = blk.router
            out[p + "mlp.shared_expert_gate.weight"] = blk.shared_gate
            for m, qs in blk.shared.items():
                out[p + f"mlp.shared_expert.{m}.weight"] = qs
        return out


def make_model(config: dict | None = None, seed: int = 0, sigma: float = 0.02) -> HostModel:
    """Seeded random-init decoder (numpy; for models small enough to build on
    the host): projections ~ N(0, sigma) then int8 per row, biases ~ N(0,
    sigma), norm weights 1 + N(0, 0.1), embedding and lm_head rows ~ N(0, 1)
    and N(0, sigma) then int8, MoE blocks from make_block(seed * 1000 + layer)."""
    c = dict(QWEN_MODEL if config is None else config)
    H, V, L = c["hidden_size"], c["vocab_size"], c["num_hidden_layers"]
    heads, kvh = c["num_attention_heads"], c["num_key_value_heads"]
    d = H // heads
    rng = np.random.default_rng(seed)
    embed = quant.int8_rowwise(_normal(rng, (V, H), 1.0))
    lm_head = quant.int8_rowwise(_normal(rng, (V, H), sigma))
    final_norm = (1.0 + _normal(rng, (H,), 0.1)).astype(np.float32)
    layers, blocks = [], []
    for i in range(L):
        lr = np.random.default_rng([seed, 1, i])
        shapes = {"q_proj": (heads * d, H), "k_proj": (kvh * d, H), "v_proj": (kvh * d, H), "o_proj": (H, heads * d)}
        proj = {m: quant.int8_rowwise(_normal(lr, s, sigma)) for m, s in shapes.items()}
        bias = {m: _normal(lr, (shapes[m][0],), sigma) for m in ("q_proj", "k_proj", "v_proj")}
        layers.append(HostLayer((1.0 + _normal(lr, (H,), 0.1)).astype(np.float32),
                                (1.0 + _normal(lr, (H,), 0.1)).astype(np.float32), proj, bias))
        blocks.append(make_block(seed * 1000 + i, hidden=H, inter=c["moe_intermediate_size"],
                                 shared_inter=c["shared_expert_intermediate_size"], num_experts=c["num_experts"],
                                 top_k=c["num_experts_per_tok"], sigma=sigma))
    return HostModel(c, embed, lm_head, final_norm, layers, blocks)


def make_model_gpu(config: dict | None = None, seed: int = 0, sigma: float = 0.02, device="cuda"):
    """The same kind of random-init decoder at full size, generated on the
    GPU (torch's seeded generator) and quantized there, so a 24-layer model's
    12.5 GB of routed-expert records take seconds rather than the minutes
    numpy would: returns (HostModel whose blocks carry no routed records,
    pinned [layers, experts, record_size] uint8 records). Not bit-equal to
    make_model's weights (another generator)."""
    import torch

    c = dict(QWEN_MODEL if config is None else config)
    H, V, L = c["hidden_size"], c["vocab_size"], c["num_hidden_layers"]
    heads, kvh = c["num_attention_heads"], c["num_key_value_heads"]
    E, I, Is, k = c["num_experts"], c["moe_intermediate_size"], c["shared_expert_intermediate_size"], c["num_experts_per_tok"]
    d = H // heads
    dev = torch.device(device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)

    def normal(shape, s):
        return torch.randn(shape, generator=gen, device=dev, dtype=torch.float32) * s

    def q8(w):  # per-row int8, as quant.int8_rowwise
        sc = w.abs().amax(dim=-1) / 127.0
        sc = torch.where(sc > 0, sc, torch.ones_like(sc))
        q = torch.clamp(torch.round(w / sc.unsqueeze(-1)), -127, 127).to(torch.int8)
        return q, sc

    def host(qs):
        return qs[0].cpu().numpy(), qs[1].cpu().numpy()

    embed = host(q8(normal((V, H), 1.0)))
    lm_head = host(q8(normal((V, H), sigma)))
    final_norm = (1.0 + normal((H,), 0.1)).cpu().numpy()
    layout = RecordLayout(FMT_INT8, H, I)
    rs = layout.record_size
    records = torch.empty((L, E, rs), dtype=torch.uint8, pin_memory=True)
    layers, blocks = [], []
    for i in range(L):
        shapes = {"q_proj": (heads * d, H), "k_proj": (kvh * d, H), "v_proj": (kvh * d, H), "o_proj": (H, heads * d)}
        proj = {m: host(q8(normal(s, sigma))) for m, s in shapes.items()}
        bias = {m: normal((shapes[m][0],), sigma).cpu().numpy() for m in ("q_proj", "k_proj", "v_proj")}
        layers.append(HostLayer((1.0 + normal((H,), 0.1)).cpu().numpy(), (1.0 + normal((H,), 0.1)).cpu().numpy(),
                                proj, bias))
        router = normal((E, H), sigma).cpu().numpy()
        shared_gate = normal((1, H), sigma).cpu().numpy()
        sh_shapes = {"gate_proj": (Is, H), "up_proj": (Is, H), "down_proj": (H, Is)}
        shared = {m: host(q8(normal(s, sigma))) for m, s in sh_shapes.items()}
        # the layer's routed records, laid out on the GPU, then into pinned memory
        rec = torch.zeros((E, rs), dtype=torch.uint8, device=dev)
        mats = {m: q8(normal((E, *layout.shape(m)), sigma)) for m in ("gate_proj", "up_proj", "down_proj")}
        for m, (q, sc) in mats.items():
            wo, so = layout.weight_offset(m), layout.scale_offset(m)
            rec[:, wo : wo + q[0].numel()] = q.reshape(E, -1).view(torch.uint8)
            rec[:, so : so + sc.shape[1] * 4] = sc.contiguous().view(torch.uint8).reshape(E, -1)
        records[i].copy_(rec)
        del rec, mats
        blocks.append(HostBlock(H, I, Is, E, k, "int8", 0, router, shared_gate, shared, [], None,
                                {"seed": seed, "sigma": sigma, "generator": "torch.cuda"}))
    return HostModel(c, embed, lm_head, final_norm, layers, blocks), records
