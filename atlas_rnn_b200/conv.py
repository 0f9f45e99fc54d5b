"""The q/k/v depthwise convolutions of the memory cells as one GPU op.

The reference cells apply three ``Conv1d(dim, dim, K, padding=K // 2, groups=dim,
bias=False)`` to the pre-normed input (rnn_memory.py:196-202, 334-340; :503-510,
643-649 in the omega cell) and keep the first T outputs. ``qkv_depthwise_conv`` computes
all three in one pass over x in its [B, T, C] layout (``atlas_dwconv3_forward``; no
transposes), and its backward gives dx and the three weight gradients in one pass
(``atlas_dwconv3_backward``). Outputs are bf16 under bf16 autocast (as autocast runs the
reference's convolution), else x's dtype; fp32 accumulation.
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import _lib
from .ops import _stream


def _code(dt: torch.dtype) -> int:
    return _lib.BF16 if dt == torch.bfloat16 else _lib.F32


class QKVDepthwiseConvFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, w_q: Tensor, w_k: Tensor, w_v: Tensor, out_dtype: torch.dtype):
        B, T, C = x.shape
        K = w_q.shape[-1]
        xd = torch.bfloat16 if x.dtype == torch.bfloat16 else torch.float32
        xc = x.to(xd).contiguous()
        ws = [w.reshape(C, K).to(torch.float32).contiguous() for w in (w_q, w_k, w_v)]
        ys = [torch.empty(B, T, C, dtype=out_dtype, device=x.device) for _ in range(3)]
        p = _lib.ptr
        _lib.check(_lib.lib().atlas_dwconv3_forward(p(xc), _code(xd), p(ws[0]), p(ws[1]), p(ws[2]), K, p(ys[0]),
                                                    p(ys[1]), p(ys[2]), _code(out_dtype), B, T, C,
                                                    _stream(x.device)), "dwconv3 forward")
        ctx.save_for_backward(xc, *ws)
        ctx.meta = (x.dtype, w_q.dtype, w_q.shape, out_dtype)
        return tuple(ys)

    @staticmethod
    def backward(ctx, dq, dk, dv):
        xc, wq, wk, wv = ctx.saved_tensors
        x_dtype, w_dtype, w_shape, out_dtype = ctx.meta
        B, T, C = xc.shape
        K = wq.shape[-1]
        zero = lambda: torch.zeros(B, T, C, dtype=out_dtype, device=xc.device)
        dys = [(d if d is not None else zero()).to(out_dtype).contiguous() for d in (dq, dk, dv)]
        dx = torch.empty_like(xc)
        dw = torch.empty(3, C, K, dtype=torch.float32, device=xc.device)
        p = _lib.ptr
        _lib.check(_lib.lib().atlas_dwconv3_backward(p(xc), _code(xc.dtype), p(wq), p(wk), p(wv), K, p(dys[0]),
                                                     p(dys[1]), p(dys[2]), _code(out_dtype), p(dx), p(dw), B, T, C,
                                                     _stream(xc.device)), "dwconv3 backward")
        g = lambda i: dw[i].reshape(w_shape).to(w_dtype)
        return dx.to(x_dtype), g(0), g(1), g(2), None


def qkv_depthwise_conv(x: Tensor, w_q: Tensor, w_k: Tensor, w_v: Tensor):
    """(conv_q(x), conv_k(x), conv_v(x)) for x [B, T, C] and Conv1d weights [C, 1, K]."""
    if not x.is_cuda:
        raise RuntimeError("atlas_rnn_b200.qkv_depthwise_conv: tensors must be on a CUDA device (no CPU path)")
    if torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16:
        out = torch.bfloat16
    else:
        out = torch.bfloat16 if x.dtype == torch.bfloat16 else torch.float32
    return QKVDepthwiseConvFn.apply(x, w_q, w_k, w_v, out)
