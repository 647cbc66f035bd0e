"""Device context and weight handles over the C ABI (replaces GpuDevice / KernelContext,
crates/v2/core/src/gpu.rs:21-170 and crates/v2/core/src/kernel.rs:666-733).

Device memory is plain torch tensors; every compute call goes through libshardlm_cuda.so on the
context's stream (torch's current stream of the device).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from ._lib import ShdError, check, lib


def ptr(t) -> int | None:
    """Device (or host) address of a contiguous tensor, None for None."""
    if t is None:
        return None
    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    return t.data_ptr()


class Context:
    """One libshardlm_cuda context on one CUDA device."""

    def __init__(self, device: int = 0):
        if not torch.cuda.is_available():
            raise RuntimeError("shardlm_b200 needs a CUDA device (sm_100); there is no CPU path")
        self.device = int(device)
        self.torch_device = torch.device("cuda", self.device)
        handle = C.c_void_p()
        rc = lib().shd_init(self.device, C.byref(handle))
        if rc != _lib.SHD_OK:
            raise ShdError(rc, f"shd_init(device={self.device}) failed (needs an sm_100 GPU)")
        self.ptr = handle
        self._bound_stream = None
        self.bind_stream()

    # -- plumbing ------------------------------------------------------------------------------
    def bind_stream(self, stream: torch.cuda.Stream | None = None) -> None:
        s = stream if stream is not None else torch.cuda.current_stream(self.torch_device)
        raw = s.cuda_stream
        if raw != self._bound_stream:
            check(lib().shd_set_stream(self.ptr, raw), self.ptr)
            self._bound_stream = raw

    def call(self, name: str, *args) -> None:
        self.bind_stream()
        rc = getattr(lib(), name)(self.ptr, *args)
        check(rc, self.ptr)

    def sync(self) -> None:
        check(lib().shd_sync(self.ptr), self.ptr)

    @property
    def launch_count(self) -> int:
        return int(lib().shd_launch_count(self.ptr))

    def close(self) -> None:
        if getattr(self, "ptr", None):
            lib().shd_destroy(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- helpers -------------------------------------------------------------------------------
    def empty(self, *shape, dtype=torch.float32) -> torch.Tensor:
        return torch.empty(*shape, dtype=dtype, device=self.torch_device)

    def to_device(self, a, dtype=None) -> torch.Tensor:
        t = torch.as_tensor(np.ascontiguousarray(a) if isinstance(a, np.ndarray) else a)
        if dtype is not None:
            t = t.to(dtype)
        return t.to(self.torch_device).contiguous()


class Weight:
    """A weight matrix in the library's tiled device format."""

    def __init__(self, ctx: Context, handle: C.c_void_p, in_features: int, out_features: int, kind: str):
        self.ctx = ctx
        self.handle = handle
        self.in_features = in_features
        self.out_features = out_features
        self.kind = kind

    @property
    def device_bytes(self) -> int:
        return int(lib().shd_weight_device_bytes(self.handle))

    @classmethod
    def from_f32_in_out(cls, ctx: Context, w_in_out: np.ndarray, in_features: int, out_features: int):
        w = np.ascontiguousarray(np.asarray(w_in_out, dtype=np.float32).reshape(-1))
        if w.size != in_features * out_features:
            raise ValueError("weight size mismatch")
        h = C.c_void_p()
        ctx.bind_stream()
        check(lib().shd_weight_upload_f32_as_bf16(ctx.ptr, w.ctypes.data, in_features, out_features,
                                                  C.byref(h)), ctx.ptr)
        return cls(ctx, h, in_features, out_features, "bf16")

    @classmethod
    def from_bf16_out_in(cls, ctx: Context, w: torch.Tensor, bias: torch.Tensor | None = None,
                         rows: int = _lib.ROWS_PLAIN, head_dim: int = 0):
        """w: device bf16 [out][in] (the safetensors layout)."""
        if w.dtype != torch.bfloat16 or not w.is_cuda or w.dim() != 2:
            raise ValueError("expected a 2-D bf16 CUDA tensor [out][in]")
        w = w.contiguous()
        b = None if bias is None else bias.to(torch.float32).contiguous()
        h = C.c_void_p()
        ctx.bind_stream()
        check(lib().shd_weight_from_bf16(ctx.ptr, ptr(w), ptr(b), w.shape[1], w.shape[0], rows,
                                         head_dim, C.byref(h)), ctx.ptr)
        return cls(ctx, h, w.shape[1], w.shape[0], "bf16")

    @classmethod
    def from_i32_in_out(cls, ctx: Context, w_in_out: np.ndarray, bias: np.ndarray | None,
                        in_features: int, out_features: int):
        w = np.ascontiguousarray(np.asarray(w_in_out, dtype=np.int32).reshape(-1))
        if w.size != in_features * out_features:
            raise ValueError("weight size mismatch")
        b = None if bias is None else np.ascontiguousarray(np.asarray(bias, dtype=np.int32))
        h = C.c_void_p()
        ctx.bind_stream()
        check(lib().shd_weight_upload_i32(ctx.ptr, w.ctypes.data, None if b is None else b.ctypes.data,
                                          in_features, out_features, C.byref(h)), ctx.ptr)
        return cls(ctx, h, in_features, out_features, "i32")

    def close(self) -> None:
        if getattr(self, "handle", None):
            lib().shd_weight_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
