"""Head preparation of the memory cells as one GPU op (``atlas_head_prep_forward``).

Replaces, for q, k and v, the chain split_heads -> MultiheadRMSNorm (q, k;
rnn_memory.py:139-147) -> '(b h) n d' reshape copy -> cast -> zero-pad to the tensor-core
kernels' 128 columns: the projection output [B, T, H * d] becomes [B * H, T, d_out] in one
pass, and the backward (``atlas_head_prep_backward``) gives the input gradient and the
norm's gain gradient in one pass.
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import _lib
from .ops import _stream

HEAD_DIMS = (32, 64, 96, 128)


def _code(dt):
    return _lib.BF16 if dt == torch.bfloat16 else _lib.F32


class HeadPrepFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, t: Tensor, gamma: Tensor | None, heads: int, d_out: int, out_dtype: torch.dtype):
        B, T, HD = t.shape
        d = HD // heads
        td = torch.bfloat16 if t.dtype == torch.bfloat16 else torch.float32
        tc = t.to(td).contiguous()
        g = gamma.reshape(heads, d).to(torch.float32).contiguous() if gamma is not None else None
        out = torch.empty(B * heads, T, d_out, dtype=out_dtype, device=t.device)
        p = _lib.ptr
        _lib.check(_lib.lib().atlas_head_prep_forward(p(tc), _code(td), p(g), p(out), _code(out_dtype), B, T, heads,
                                                      d, d_out, _stream(t.device)), "head_prep forward")
        ctx.save_for_backward(tc, g)
        ctx.meta = (t.dtype, heads, d, d_out, out_dtype, None if gamma is None else (gamma.dtype, gamma.shape))
        return out

    @staticmethod
    def backward(ctx, grad_out):
        tc, g = ctx.saved_tensors
        t_dtype, heads, d, d_out, out_dtype, gmeta = ctx.meta
        B, T, _ = tc.shape
        go = grad_out.to(out_dtype).contiguous()
        dt = torch.empty_like(tc)
        dg = torch.empty(heads, d, dtype=torch.float32, device=tc.device) if g is not None else None
        p = _lib.ptr
        _lib.check(_lib.lib().atlas_head_prep_backward(p(tc), _code(tc.dtype), p(g), p(go), _code(out_dtype), p(dt),
                                                       p(dg), B, T, heads, d, d_out, _stream(tc.device)),
                   "head_prep backward")
        d_gamma = dg.reshape(gmeta[1]).to(gmeta[0]) if dg is not None else None
        return dt.to(t_dtype), d_gamma, None, None, None


def head_prep(t: Tensor, gamma: Tensor | None, heads: int, d_out: int, out_dtype: torch.dtype) -> Tensor:
    """[B, T, heads * d] -> [B * heads, T, d_out] (optionally RMS-normalised per head with gain
    gamma [heads, 1, d]; columns d .. d_out - 1 zero)."""
    if not t.is_cuda:
        raise RuntimeError("atlas_rnn_b200.head_prep: tensors must be on a CUDA device (no CPU path)")
    return HeadPrepFn.apply(t, gamma, heads, d_out, out_dtype)
