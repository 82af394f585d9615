"""MoeBlock: one MoE layer resident in HBM, run by er_moe_block.

Drop-in for `QwenMoe._moe` (runtime/qwen_moe.py:293-359): given the
post-attention RMSNorm output h [n, 2048] it returns
routed + sigmoid(h @ w_g^T) * shared, with the router, top-4 selection,
expert dispatch and combine all on the GPU. Expert weights are store records
in HBM; the device pointer table `expert_table` says where each expert's
record is, so an HBM expert cache can remap experts between calls without
copying.

PyTorch provides device memory and the current stream; the arithmetic is
the CUDA library's.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from ._lib import MoeIO, MoeWeights
from .store import FMT_INT8, RecordLayout


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")


class MoeBlock:
    """One layer's MoE block on a CUDA device.

    router      [E, H] float32 (mlp.gate.weight)
    shared_gate [1, H] or [H] float32 (mlp.shared_expert_gate.weight)
    shared      {"gate_proj", "up_proj", "down_proj"} -> (int8 q, float32 scales)
    records     [E, record_size] uint8 routed-expert records (layout `layout`),
                host or device; or None when an expert table is set later
    """

    def __init__(
        self,
        *,
        router: np.ndarray,
        shared_gate: np.ndarray,
        shared: dict,
        layout: RecordLayout,
        shared_inter: int,
        records: np.ndarray | torch.Tensor | None = None,
        top_k: int = 4,
        norm_topk_prob: bool = False,
        device: str | torch.device = "cuda",
    ):
        if not torch.cuda.is_available():
            raise RuntimeError("MoeBlock needs a CUDA device (the B200 path has no CPU fallback)")
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.layout = layout
        self.num_experts, self.hidden = int(router.shape[0]), int(router.shape[1])
        self.inter, self.shared_inter, self.top_k = layout.inter, int(shared_inter), int(top_k)
        dev = self.device
        self.router = torch.as_tensor(np.ascontiguousarray(router, dtype=np.float32)).to(dev)
        self.shared_gate = torch.as_tensor(np.ascontiguousarray(shared_gate, dtype=np.float32).reshape(-1)).to(dev)
        from .store import serialize_record

        sh_layout = RecordLayout(FMT_INT8, self.hidden, self.shared_inter)
        self.shared_record = torch.as_tensor(serialize_record(sh_layout, shared)).to(dev)
        self.records: torch.Tensor | None = None
        self.expert_table = torch.zeros(self.num_experts, dtype=torch.int64, device=dev)
        if records is not None:
            self.set_records(records)
        self._w = MoeWeights(
            hidden=self.hidden,
            num_experts=self.num_experts,
            top_k=self.top_k,
            inter=self.inter,
            shared_inter=self.shared_inter,
            expert_fmt=layout.fmt,
            group=layout.group,
            norm_topk_prob=int(norm_topk_prob),
            router_w=self.router.data_ptr(),
            shared_gate_w=self.shared_gate.data_ptr(),
            expert_records=self.expert_table.data_ptr(),
            shared_record=self.shared_record.data_ptr(),
        )
        self._set_arena()
        self._ws: torch.Tensor | None = None

    @classmethod
    def from_host_block(cls, block, device: str | torch.device = "cuda") -> MoeBlock:
        """From an expertrelay_b200.synth.HostBlock."""
        return cls(
            router=block.router,
            shared_gate=block.shared_gate,
            shared=block.shared,
            layout=block.layout,
            shared_inter=block.shared_inter,
            records=block.records(),
            top_k=block.top_k,
            device=device,
        )

    def set_records(self, records: np.ndarray | torch.Tensor) -> None:
        """Upload (or adopt) all E records back to back and point the table at them."""
        rs = self.layout.record_size
        t = torch.as_tensor(records)
        if t.dtype != torch.uint8 or t.numel() != self.num_experts * rs:
            raise ValueError(f"records: expected {self.num_experts} x {rs} uint8, got {tuple(t.shape)} {t.dtype}")
        self.records = t.reshape(self.num_experts, rs).to(self.device).contiguous()
        base = self.records.data_ptr()
        self.set_expert_table(torch.arange(self.num_experts, dtype=torch.int64, device=self.device) * rs + base)
        if hasattr(self, "_w"):
            self._set_arena()

    def _set_arena(self, base: int | None = None, slots: int | None = None) -> None:
        """Declare the array the routed records live in (the tensor-core path
        addresses records as slots of one arena)."""
        if base is None and self.records is not None:
            base, slots = self.records.data_ptr(), self.num_experts
        self._w.record_arena = base
        self._w.arena_slots = int(slots or 0)

    def use_arena(self, base: int, slots: int) -> None:
        """Serve the routed records from an external arena of `slots` records
        starting at device address `base` (an HbmExpertCache's); the expert
        table must then point into it."""
        self.records = None
        self._set_arena(int(base), int(slots))

    def router_logits(self, h: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """h @ router^T in fp32 ([n, E]); also what the next layer's router on
        this layer's input gives for a Fate-style prefetch guess."""
        _require_cuda(h, "h")
        if h.dtype != torch.float32 or not h.is_contiguous():
            h = h.float().contiguous()
        n = h.shape[0]
        if out is None:
            out = torch.empty((n, self.num_experts), dtype=torch.float32, device=h.device)
        stream = torch.cuda.current_stream(h.device).cuda_stream
        rc = _lib.lib().er_linear_f32(h.data_ptr(), self.hidden, self.router.data_ptr(), None, out.data_ptr(), n,
                                      self.num_experts, self.hidden, stream)
        _lib.check(rc, "er_linear_f32")
        return out

    def set_expert_table(self, addresses: torch.Tensor) -> None:
        """Device addresses of each expert's record (e.g. HBM cache slots)."""
        if addresses.numel() != self.num_experts:
            raise ValueError("one address per expert")
        if addresses.device.type == "cpu" and addresses.dtype == torch.int64:
            # straight from host memory: asynchronous when the source is pinned
            self.expert_table.copy_(addresses, non_blocking=addresses.is_pinned())
        else:
            self.expert_table.copy_(addresses.to(self.device, torch.int64), non_blocking=True)

    def error_bits(self, n: int, path: int = _lib.PATH_AUTO, workspace: torch.Tensor | None = None) -> int:
        """The plan's error bits after the last forward of n tokens on this
        path (0: clean; see er_moe_error_bits). Synchronises the stream."""
        ws = workspace if workspace is not None else self._ws
        if ws is None:
            return 0
        bits = C.c_int(0)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(_lib.lib().er_moe_error_bits(C.byref(self._w), int(n), int(path), ws.data_ptr(), C.byref(bits),
                                                stream), "er_moe_error_bits")
        return int(bits.value)

    def workspace_bytes(self, n: int, path: int = _lib.PATH_AUTO) -> int:
        return int(_lib.lib().er_moe_workspace_bytes(C.byref(self._w), int(n), int(path)))

    def _workspace(self, n: int, path: int) -> torch.Tensor:
        need = self.workspace_bytes(n, path)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 256), dtype=torch.uint8, device=self.device)
        return self._ws

    def forward(
        self,
        h: torch.Tensor,
        *,
        logits: torch.Tensor | None = None,
        out: torch.Tensor | None = None,
        path: int = _lib.PATH_AUTO,
        return_routing: bool = False,
        stage_events: list | None = None,
        launch_counter: C.c_int | None = None,
        workspace: torch.Tensor | None = None,
    ):
        """h [n, H] float32 or bfloat16 CUDA tensor -> y [n, H] float32. With
        `logits` ([n, E] float32) the routing uses those router logits. With
        return_routing, also returns (logits [n, E], top-k ids [n, k] int64,
        top-k weights [n, k] float32). `stage_events` (len(MOE_STAGES) + 1
        timing-enabled torch.cuda.Event, already recorded once) are recorded
        around each stage; `launch_counter` accumulates the kernel launches."""
        _require_cuda(h, "h")
        if h.dim() != 2 or h.shape[1] != self.hidden:
            raise ValueError(f"h: expected [n, {self.hidden}], got {tuple(h.shape)}")
        if h.dtype not in (torch.float32, torch.bfloat16):
            raise ValueError(f"h: float32 or bfloat16, got {h.dtype}")
        h = h.contiguous()
        n = h.shape[0]
        y = out if out is not None else torch.empty((n, self.hidden), dtype=torch.float32, device=self.device)
        lg_out = idx_out = w_out = None
        if return_routing:
            lg_out = torch.empty((n, self.num_experts), dtype=torch.float32, device=self.device)
            idx_out = torch.empty((n, self.top_k), dtype=torch.int64, device=self.device)
            w_out = torch.empty((n, self.top_k), dtype=torch.float32, device=self.device)
        if logits is not None:
            _require_cuda(logits, "logits")
            logits = logits.to(torch.float32).contiguous()
            if tuple(logits.shape) != (n, self.num_experts):
                raise ValueError(f"logits: expected [{n}, {self.num_experts}], got {tuple(logits.shape)}")
        if workspace is None:
            ws = self._workspace(n, path)
        else:
            if workspace.numel() < self.workspace_bytes(n, path):
                raise ValueError("workspace too small for this batch")
            ws = workspace
        io = MoeIO(
            h=h.data_ptr(),
            h_dtype=_lib.DTYPE_BF16 if h.dtype == torch.bfloat16 else _lib.DTYPE_F32,
            n=n,
            logits_in=_ptr(logits),
            y=y.data_ptr(),
            logits_out=_ptr(lg_out),
            topk_idx_out=_ptr(idx_out),
            topk_w_out=_ptr(w_out),
            path=int(path),
        )
        if stage_events is not None:
            if len(stage_events) != len(_lib.MOE_STAGES) + 1:
                raise ValueError(f"stage_events: need {len(_lib.MOE_STAGES) + 1} events")
            for ev in stage_events:
                if not ev.cuda_event:  # torch creates the CUDA event on its first record
                    ev.record()
            handles = (C.c_void_p * len(stage_events))(*[ev.cuda_event for ev in stage_events])
            io.stage_events = C.cast(handles, C.POINTER(C.c_void_p))
        if launch_counter is not None:
            io.launch_count = C.pointer(launch_counter)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        rc = _lib.lib().er_moe_block(C.byref(self._w), C.byref(io), ws.data_ptr(), ws.numel(), stream)
        _lib.check(rc, "er_moe_block")
        if return_routing:
            return y, lg_out, idx_out, w_out
        return y

    __call__ = forward

    def capture(
        self,
        n: int,
        *,
        dtype: torch.dtype = torch.float32,
        path: int = _lib.PATH_AUTO,
        stage_events: list | None = None,
    ) -> CapturedBlock:
        """Record one forward over a fixed [n, H] input buffer into a CUDA graph.
        The graph owns its workspace, input and output; replays re-read the
        expert table, so remapped experts are picked up without re-capture."""
        h = torch.zeros((n, self.hidden), dtype=dtype, device=self.device)
        y = torch.empty((n, self.hidden), dtype=torch.float32, device=self.device)
        ws = torch.empty(max(self.workspace_bytes(n, path), 256), dtype=torch.uint8, device=self.device)
        self.forward(h, out=y, path=path, workspace=ws)  # first-use setup happens outside the capture
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self.forward(h, out=y, path=path, workspace=ws, stage_events=stage_events)
        return CapturedBlock(graph, h, y, ws)

    def moe_numpy(self, h: np.ndarray) -> np.ndarray:
        """The reference's calling convention: numpy float32 in, new numpy float32 out."""
        hd = torch.from_numpy(np.ascontiguousarray(h, dtype=np.float32)).to(self.device, non_blocking=False)
        return self.forward(hd).cpu().numpy()


class CapturedBlock:
    """A MoeBlock forward captured as a CUDA graph over fixed buffers `h` -> `y`."""

    def __init__(self, graph, h: torch.Tensor, y: torch.Tensor, workspace: torch.Tensor):
        self.graph, self.h, self.y, self._ws = graph, h, y, workspace

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.y

    def __call__(self, h: torch.Tensor) -> torch.Tensor:
        """Copy `h` (device or pinned host) into the graph's input and replay."""
        self.h.copy_(h, non_blocking=True)
        return self.replay()

    def run_host(self, h_host: torch.Tensor, y_host: torch.Tensor) -> torch.Tensor:
        """Host tokens in, host output back, all ordered on the current stream
        (pinned buffers make both copies asynchronous)."""
        self.h.copy_(h_host, non_blocking=True)
        self.graph.replay()
        y_host.copy_(self.y, non_blocking=True)
        return y_host


class HostPipeline:
    """The MoE block over a stream of host batches (the serving loop of
    `QwenMoe.forward` calls with numpy in and out, runtime/qwen_moe.py:293),
    with the copies overlapped: `depth` captured graphs, each with its own
    device input, output and workspace, and three streams, so the
    host->device copy of batch i + 1 and the device->host copy of batch i - 1
    run while batch i computes. Every batch's inputs are copied from the
    caller's pinned host buffer and its result copied back into the caller's
    pinned host buffer; `sync()` waits for all of them.

    Ordering per slot b = i % depth: the input copy of batch i waits for the
    compute of batch i - depth (which read the slot's input); the compute of
    batch i waits for its input copy and for the output copy of batch
    i - depth (which read the slot's output)."""

    def __init__(self, block: MoeBlock, n: int, *, dtype: torch.dtype = torch.float32,
                 path: int = _lib.PATH_AUTO, depth: int = 2):
        if depth < 1:
            raise ValueError("depth: at least one slot")
        self.n, self.hidden, self.device = n, block.hidden, block.device
        self.slots = [block.capture(n, dtype=dtype, path=path) for _ in range(depth)]
        self.s_in, self.s_run, self.s_out = (torch.cuda.Stream(self.device) for _ in range(3))
        self.ev_in = [torch.cuda.Event() for _ in range(depth)]
        self.ev_run = [torch.cuda.Event() for _ in range(depth)]
        self.ev_out = [torch.cuda.Event() for _ in range(depth)]
        self.count = 0
        # the slots' buffers were written on the capturing stream
        for s in (self.s_in, self.s_run, self.s_out):
            s.wait_stream(torch.cuda.current_stream(self.device))

    def submit(self, h_host: torch.Tensor, y_host: torch.Tensor, before_run=None) -> torch.Tensor:
        """Queue one batch: `h_host` [n, H] (pinned, the capture's dtype) in,
        `y_host` [n, H] float32 (pinned) out. `before_run`, if given, is
        called on the compute stream just before the graph replays (bench
        hook: an L2 flush). Returns `y_host`, valid after `sync()`."""
        if tuple(h_host.shape) != (self.n, self.hidden) or tuple(y_host.shape) != (self.n, self.hidden):
            raise ValueError(f"host buffers must be [{self.n}, {self.hidden}]")
        if h_host.is_cuda or y_host.is_cuda or not (h_host.is_pinned() and y_host.is_pinned()):
            raise ValueError("host buffers must be pinned host memory")
        depth = len(self.slots)
        b = self.count % depth
        slot = self.slots[b]
        reuse = self.count >= depth
        if reuse:
            self.s_in.wait_event(self.ev_run[b])
        with torch.cuda.stream(self.s_in):
            slot.h.copy_(h_host, non_blocking=True)
            self.ev_in[b].record(self.s_in)
        self.s_run.wait_event(self.ev_in[b])
        if reuse:
            self.s_run.wait_event(self.ev_out[b])
        with torch.cuda.stream(self.s_run):
            if before_run is not None:
                before_run()
            slot.graph.replay()
            self.ev_run[b].record(self.s_run)
        self.s_out.wait_event(self.ev_run[b])
        with torch.cuda.stream(self.s_out):
            y_host.copy_(slot.y, non_blocking=True)
            self.ev_out[b].record(self.s_out)
        self.count += 1
        return y_host

    def join(self, stream: torch.cuda.Stream | None = None) -> None:
        """Make `stream` (default: the current one) wait for every queued batch."""
        st = stream if stream is not None else torch.cuda.current_stream(self.device)
        for s in (self.s_in, self.s_run, self.s_out):
            st.wait_stream(s)

    def sync(self) -> None:
        """Wait on the host until every queued batch's output is in its host buffer."""
        for s in (self.s_in, self.s_run, self.s_out):
            s.synchronize()
