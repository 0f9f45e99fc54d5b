"""Right-affine matrix scan on the GPU: the drop-in of the reference's
``affine_associative_scan`` (atlas_pytorch/affine_scan.py:36-160).

    H_t = H_{t-1} @ A_t + B_t,   H_{-1} = prev (or zeros)

A [N, T, D, D], B [N, T, R, D], prev [N, R, D]. Returns [N, T, R, D], or
[N, T + 1, R, D] with prev first when prev is given and remove_prev is False --
the reference's output convention. The reference composes transforms in a
log-depth tree (O(T D^3) products); the kernels (atlas_affine_scan_forward /
_backward, csrc/affine_scan.cuh) run the recurrence in order, one [R, D] x
[D, D] product per step, fp32, with autograd.
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import _lib
from .ops import _stream


class AffineScanFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, A, B, prev, remove_prev: bool):
        if not A.is_cuda:
            raise RuntimeError("atlas_rnn_b200.affine_associative_scan: tensors must be on a CUDA device "
                               "(no CPU path)")
        if A.ndim != 4 or B.ndim != 4:
            raise ValueError("Expected A=[N,T,D,D], B=[N,T,R,D]")
        N, T, D, D2 = A.shape
        nB, tB, R, dB = B.shape
        if D != D2 or (nB, tB, dB) != (N, T, D):
            raise ValueError(f"inconsistent shapes A {tuple(A.shape)}, B {tuple(B.shape)}")
        if prev is not None and tuple(prev.shape) != (N, R, D):
            raise ValueError(f"prev must be {(N, R, D)}, not {tuple(prev.shape)}")
        a, b = A.float().contiguous(), B.float().contiguous()
        p = prev.float().contiguous() if prev is not None else None
        off = 1 if (p is not None and not remove_prev) else 0
        out = torch.empty(N, T + off, R, D, dtype=torch.float32, device=A.device)
        ptr = _lib.ptr
        _lib.check(_lib.lib().atlas_affine_scan_forward(ptr(a), ptr(b), ptr(p), ptr(out), N, T, R, D,
                                                        int(bool(remove_prev)), _stream(A.device)),
                   "affine scan forward")
        ctx.save_for_backward(a, p, out)
        ctx.meta = (N, T, R, D, bool(remove_prev), A.dtype, B.dtype, None if prev is None else prev.dtype)
        return out.to(A.dtype)

    @staticmethod
    def backward(ctx, dout):
        a, p, out = ctx.saved_tensors
        N, T, R, D, remove_prev, a_dtype, b_dtype, p_dtype = ctx.meta
        dout = dout.float().contiguous()
        dA = torch.empty_like(a)
        dB = torch.empty(N, T, R, D, dtype=torch.float32, device=a.device)
        dp = torch.empty_like(p) if p is not None else None
        ptr = _lib.ptr
        _lib.check(_lib.lib().atlas_affine_scan_backward(ptr(a), ptr(p), ptr(out), ptr(dout), ptr(dA), ptr(dB),
                                                         ptr(dp), N, T, R, D, int(remove_prev),
                                                         _stream(a.device)), "affine scan backward")
        return dA.to(a_dtype), dB.to(b_dtype), (dp.to(p_dtype) if dp is not None else None), None


def affine_associative_scan(A: Tensor, B: Tensor, *, prev: Tensor | None = None,
                            remove_prev: bool = False) -> Tensor:
    """GPU form of ``affine_scan.affine_associative_scan`` (same arguments and output)."""
    return AffineScanFn.apply(A, B, prev, remove_prev)
