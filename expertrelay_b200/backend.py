"""B200Backend: the reference's compute-backend protocol on the GPU.

Implements `runtime.backends.Backend` (runtime/backends.py:44-67) with the
same calling convention as NumpyBackend (:75-95): numpy arrays in, a new
numpy float32 array out. Each call copies its operands to the device, runs
one CUDA kernel of libexpertrelay_b200 and copies the result back, so it is
a drop-in for any caller of the protocol; the fused, HBM-resident path for
the MoE block is expertrelay_b200.moe.MoeBlock.

Registered under the name "b200" with the same lookup rules as the
reference's make_backend (backends.py:98-103): an unknown name raises
ValueError.
"""

from __future__ import annotations

import importlib

import numpy as np
import torch

from . import _lib

_BACKENDS = {"b200": "expertrelay_b200.backend:B200Backend"}
BACKEND_NAMES = tuple(_BACKENDS)


def _dev(a: np.ndarray, dtype, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=dtype)).to(device)


class B200Backend:
    name = "b200"

    def __init__(self, device: str | None = None):
        if not torch.cuda.is_available():
            raise RuntimeError("the b200 backend needs a CUDA device (there is no CPU fallback)")
        self.device = torch.device(device or "cuda")
        _lib.lib()  # fail now, not mid-run, if the library is missing

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def int8_linear(
        self, x: np.ndarray, q: np.ndarray, scales: np.ndarray, bias: np.ndarray | None = None
    ) -> np.ndarray:
        """x [n, in] f32, q [out, in] int8, scales [out] f32 -> [n, out] f32."""
        x = np.asarray(x)
        n, in_dim = x.shape
        out_dim = q.shape[0]
        if q.shape[1] != in_dim or scales.shape != (out_dim,):
            raise ValueError(f"int8_linear: x {x.shape}, q {q.shape}, scales {scales.shape}")
        xd, qd = _dev(x, np.float32, self.device), _dev(q, np.int8, self.device)
        sd = _dev(scales, np.float32, self.device)
        bd = None if bias is None else _dev(bias, np.float32, self.device)
        y = torch.empty((n, out_dim), dtype=torch.float32, device=self.device)
        rc = _lib.lib().er_int8_linear(xd.data_ptr(), in_dim, qd.data_ptr(), sd.data_ptr(),
                                       None if bd is None else bd.data_ptr(), y.data_ptr(), n, out_dim, in_dim,
                                       self._stream())
        _lib.check(rc, "er_int8_linear")
        return y.cpu().numpy()

    def int4_linear(self, x: np.ndarray, packed: np.ndarray, scales: np.ndarray, group: int) -> np.ndarray:
        """x [n, in] f32, packed [out, in/2] uint8 (store.int4), scales [out, in/group] f16 -> [n, out] f32."""
        x = np.asarray(x)
        n, in_dim = x.shape
        out_dim = packed.shape[0]
        if packed.shape[1] * 2 != in_dim:
            raise ValueError(f"int4_linear: x {x.shape} vs packed {packed.shape}")
        xd, pd = _dev(x, np.float32, self.device), _dev(packed, np.uint8, self.device)
        sd = torch.from_numpy(np.ascontiguousarray(scales, dtype=np.float16).view(np.uint16)).to(self.device)
        y = torch.empty((n, out_dim), dtype=torch.float32, device=self.device)
        rc = _lib.lib().er_int4_linear(xd.data_ptr(), in_dim, pd.data_ptr(), sd.data_ptr(), None, int(group), None,
                                       y.data_ptr(), n, out_dim, in_dim, self._stream())
        _lib.check(rc, "er_int4_linear")
        return y.cpu().numpy()

    def linear(self, x: np.ndarray, w: np.ndarray, bias: np.ndarray | None = None) -> np.ndarray:
        """x [n, in] f32, w [out, in] f32 -> [n, out] f32."""
        x = np.asarray(x)
        n, in_dim = x.shape
        out_dim = w.shape[0]
        xd, wd = _dev(x, np.float32, self.device), _dev(w, np.float32, self.device)
        bd = None if bias is None else _dev(bias, np.float32, self.device)
        y = torch.empty((n, out_dim), dtype=torch.float32, device=self.device)
        rc = _lib.lib().er_linear_f32(xd.data_ptr(), in_dim, wd.data_ptr(), None if bd is None else bd.data_ptr(),
                                      y.data_ptr(), n, out_dim, in_dim, self._stream())
        _lib.check(rc, "er_linear_f32")
        return y.cpu().numpy()

    def attention(self, q: np.ndarray, keys: np.ndarray, values: np.ndarray, allowed: np.ndarray) -> np.ndarray:
        """q [n, heads, d], keys/values [k, heads, d], allowed [n, k] bool -> [n, heads, d]."""
        n, heads, d = q.shape
        kv = keys.shape[0]
        qd, kd = _dev(q, np.float32, self.device), _dev(keys, np.float32, self.device)
        vd = _dev(values, np.float32, self.device)
        ad = _dev(np.asarray(allowed, dtype=bool).astype(np.uint8), np.uint8, self.device)
        out = torch.empty((n, heads, d), dtype=torch.float32, device=self.device)
        rc = _lib.lib().er_attention(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), ad.data_ptr(), out.data_ptr(), n,
                                     kv, heads, d, self._stream())
        _lib.check(rc, "er_attention")
        return out.cpu().numpy()


def make_backend(name: str, device: str | None = None):
    if name not in _BACKENDS:
        raise ValueError(f"unknown backend {name!r}; available: {', '.join(BACKEND_NAMES)}")
    module, cls = _BACKENDS[name].split(":")
    backend_cls = getattr(importlib.import_module(module), cls)
    return backend_cls(device) if device is not None else backend_cls()
