"""Scalar-gated scan on the GPU: a drop-in for the third-party ``assoc_scan.AssocScan``.

The reference imports ``from assoc_scan import AssocScan`` (rnn_memory.py:34) and calls
``AssocScan(use_accelerated=...)(gates, inputs, prev=...)`` (rnn_memory.py:189,363-379) and,
in the legacy OmegaNeuralMemory, with ``remove_prev=False`` (omega.py:315). Over dim 1,

    h_t = gates[b, t] * h_{t-1} + inputs[b, t, ...],   h_0 = prev (or 0),

returning h_1..h_T, with ``prev`` prepended (T + 1 outputs) when it is given and
``remove_prev`` is false. Forward and backward run as the C-ABI kernels
``atlas_scan_forward`` / ``atlas_scan_backward`` (fp32 accumulation; fp32 or bf16 io).
"""
from __future__ import annotations

import ctypes
import math

import torch
from torch import Tensor

from . import _lib
from .ops import _stream


def _io_dtype(t: Tensor):
    return (torch.bfloat16, _lib.BF16) if t.dtype == torch.bfloat16 else (torch.float32, _lib.F32)


class AssocScanFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gates: Tensor, inputs: Tensor, prev: Tensor | None, remove_prev: bool):
        if not inputs.is_cuda:
            raise RuntimeError("atlas_rnn_b200.AssocScan: tensors must be on a CUDA device (no CPU path)")
        B, T = inputs.shape[0], inputs.shape[1]
        trail = tuple(inputs.shape[2:])
        D = math.prod(trail) if trail else 1
        if gates.numel() != B * T:
            raise ValueError(f"gates must hold one scalar per (batch, step): {tuple(gates.shape)} vs {(B, T)}")
        io, io_code = _io_dtype(inputs)
        g32 = gates.reshape(B, T).to(torch.float32).contiguous()
        x = inputs.to(io).contiguous()
        p = prev.reshape(B, D).to(torch.float32).contiguous() if prev is not None else None
        off = 1 if (prev is not None and not remove_prev) else 0
        out = torch.empty((B, T + off) + trail, dtype=io, device=inputs.device)
        ptr = _lib.ptr
        _lib.check(_lib.lib().atlas_scan_forward(ptr(g32), ptr(x), ptr(p), ptr(out), B, T, D, io_code,
                                                 0 if off else 1, _stream(inputs.device)), "scan forward")
        ctx.save_for_backward(g32, out, p)
        ctx.meta = (B, T, D, trail, io, io_code, off, gates.dtype, gates.shape, inputs.dtype,
                    None if prev is None else (prev.dtype, prev.shape))
        return out.to(inputs.dtype)

    @staticmethod
    def backward(ctx, dout: Tensor):
        g32, out, p = ctx.saved_tensors
        B, T, D, trail, io, io_code, off, g_dtype, g_shape, x_dtype, prev_meta = ctx.meta
        dout = dout.to(io).contiguous()
        dg = torch.empty(B, T, dtype=torch.float32, device=out.device)
        dx = torch.empty((B, T) + trail, dtype=io, device=out.device)
        dp = torch.empty(B, D, dtype=torch.float32, device=out.device) if p is not None else None
        ptr = _lib.ptr
        _lib.check(_lib.lib().atlas_scan_backward(ptr(g32), ptr(out), ptr(p), ptr(dout), ptr(dg), ptr(dx),
                                                  ptr(dp), B, T, D, io_code, 0 if off else 1,
                                                  _stream(out.device)), "scan backward")
        d_prev = dp.reshape(prev_meta[1]).to(prev_meta[0]) if dp is not None else None
        return dg.reshape(g_shape).to(g_dtype), dx.to(x_dtype), d_prev, None


class AssocScan(torch.nn.Module):
    """Drop-in for ``assoc_scan.AssocScan``: ``use_accelerated`` is accepted and ignored
    (the scan always runs on the GPU kernels)."""

    def __init__(self, use_accelerated: bool = False):
        super().__init__()
        self.use_accelerated = use_accelerated

    def forward(self, gates: Tensor, inputs: Tensor, prev: Tensor | None = None,
                remove_prev: bool | None = None) -> Tensor:
        return AssocScanFn.apply(gates, inputs, prev, True if remove_prev is None else bool(remove_prev))


def assoc_scan(gates: Tensor, inputs: Tensor, prev: Tensor | None = None, remove_prev: bool = True) -> Tensor:
    """Functional form of :class:`AssocScan`."""
    return AssocScanFn.apply(gates, inputs, prev, remove_prev)
