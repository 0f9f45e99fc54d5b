"""Legacy OmegaNeuralMemory per-parameter update on the GPU.

``OmegaNeuralMemory.store_memories`` (atlas_pytorch/omega.py:120-329) turns each
parameter's surprises [(bh), n, ...] into updates with a momentum scan
(omega.py:262-268), the omega gate (:276-283), a window sum over the last e
entries with a buffer carried across calls (:285-298, ``_sliding_sum_along_n``
:24-33) and a decay scan that keeps the previous update (:315). ``omega_store_update``
runs that chain as one fused kernel pass (``atlas_omega_store_forward`` /
``_backward``, csrc/omega_store.cuh) with autograd; the reference runs it as three
passes over [(bh), n, ...] plus concatenations.
"""
from __future__ import annotations

import math

import torch
from torch import Tensor

from . import _lib
from .ops import _stream


def _io(t: Tensor):
    return (torch.bfloat16, _lib.BF16) if t.dtype == torch.bfloat16 else (torch.float32, _lib.F32)


class OmegaStoreFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, surprise, keep, last_update, beta, last_momentum, gate, prev_buf, window: int):
        if not surprise.is_cuda:
            raise RuntimeError("atlas_rnn_b200.omega_store_update: tensors must be on a CUDA device (no CPU path)")
        B, T = surprise.shape[:2]
        trail = tuple(surprise.shape[2:])
        D = math.prod(trail) if trail else 1
        io, code = _io(surprise)
        f32 = lambda t, shape: None if t is None else t.reshape(shape).to(torch.float32).contiguous()
        s = surprise.to(io).contiguous()
        a, be, u = f32(keep, (B, T)), f32(beta, (B, T)), f32(gate, (B, T))
        m0, h0 = f32(last_momentum, (B, D)), f32(last_update, (B, D))
        buf = f32(prev_buf, (B, window - 1, D)) if window > 1 else None
        off = 1 if h0 is not None else 0
        dev = surprise.device
        out = torch.empty((B, T + off, D), dtype=io, device=dev)
        m_all = torch.empty((B, T, D), dtype=torch.float32, device=dev) if be is not None else None
        m_last = torch.empty((B, D), dtype=torch.float32, device=dev) if be is not None else None
        buf_out = torch.empty((B, window - 1, D), dtype=torch.float32, device=dev) if window > 1 else None
        p = _lib.ptr
        _lib.check(_lib.lib().atlas_omega_store_forward(p(be), p(s), p(m0), p(u), p(buf), p(a), p(h0), p(out),
                                                         p(m_all), p(m_last), p(buf_out), B, T, D, window, code,
                                                         _stream(dev)), "omega store forward")
        ctx.save_for_backward(s, a, be, u, m0, h0, out, m_all)
        ctx.meta = (B, T, D, trail, window, code, io, surprise.dtype,
                    [None if t is None else (t.shape, t.dtype) for t in
                     (keep, last_update, beta, last_momentum, gate, prev_buf)])
        ret_m = m_last.reshape((B,) + trail) if m_last is not None else None
        ret_b = buf_out.reshape((B, window - 1) + trail) if buf_out is not None else None
        return out.reshape((B, T + off) + trail).to(surprise.dtype), ret_m, ret_b

    @staticmethod
    def backward(ctx, d_out, d_mlast, d_buf):
        s, a, be, u, m0, h0, out, m_all = ctx.saved_tensors
        B, T, D, trail, window, code, io, s_dtype, metas = ctx.meta
        dev = s.device
        off = 1 if h0 is not None else 0
        d_out = (d_out if d_out is not None else torch.zeros((B, T + off) + trail, device=dev)).reshape(
            B, T + off, D).to(io).contiguous()
        dml = d_mlast.reshape(B, D).float().contiguous() if (d_mlast is not None and be is not None) else None
        dbo = d_buf.reshape(B, window - 1, D).float().contiguous() if (d_buf is not None and window > 1) else None
        ds = torch.empty((B, T, D), dtype=io, device=dev)
        dkeep = torch.empty((B, T), dtype=torch.float32, device=dev)
        dbeta = torch.empty((B, T), dtype=torch.float32, device=dev) if be is not None else None
        dgate = torch.empty((B, T), dtype=torch.float32, device=dev) if u is not None else None
        dm0 = torch.empty((B, D), dtype=torch.float32, device=dev) if m0 is not None else None
        dh0 = torch.empty((B, D), dtype=torch.float32, device=dev) if h0 is not None else None
        dbuf = torch.empty((B, window - 1, D), dtype=torch.float32, device=dev) if (
            window > 1 and metas[5] is not None) else None
        p = _lib.ptr
        _lib.check(_lib.lib().atlas_omega_store_backward(p(be), p(s), p(m0), p(u), p(a), p(h0), p(out), p(m_all),
                                                          p(d_out), p(dml), p(dbo), p(ds), p(dbeta), p(dgate),
                                                          p(dkeep), p(dm0), p(dh0), p(dbuf), B, T, D, window, code,
                                                          _stream(dev)), "omega store backward")
        back = lambda g, m: None if (g is None or m is None) else g.reshape(m[0]).to(m[1])
        return (ds.reshape((B, T) + trail).to(s_dtype), back(dkeep, metas[0]), back(dh0, metas[1]),
                back(dbeta, metas[2]), back(dm0, metas[3]), back(dgate, metas[4]), back(dbuf, metas[5]), None)


def omega_store_update(surprise: Tensor, decay_factor: Tensor, last_update: Tensor | None = None, *,
                       adaptive_momentum: Tensor | None = None, last_momentum: Tensor | None = None,
                       omega_gate: Tensor | None = None, prev_buf: Tensor | None = None, window: int = 1):
    """One parameter's update in ``OmegaNeuralMemory.store_memories`` (omega.py:262-315).

    surprise [(bh), n, ...]; decay_factor, adaptive_momentum, omega_gate one scalar per
    ((bh), n) (trailing singleton dims allowed); last_update, last_momentum [(bh), ...];
    prev_buf [(bh), window-1, ...] (the ``<name>__omega_buf`` entry, None = zeros).
    Returns (update [(bh), n+1, ...] with last_update first -- or [(bh), n, ...] without
    it --, the next last momentum or None, the next buffer or None). As in the reference,
    when every omega gate of the chunk is below 1e-3 the update is all zeros and not
    scanned (omega.py:306-309).
    """
    if window < 1:
        raise ValueError("window must be >= 1")
    keep = 1.0 - decay_factor
    update, m_last, buf = OmegaStoreFn.apply(surprise, keep, last_update, adaptive_momentum, last_momentum,
                                             omega_gate, prev_buf if window > 1 else None, window)
    if omega_gate is not None and bool(torch.all(omega_gate.reshape(surprise.shape[0], -1).amax(dim=1) < 1e-3)):
        n = surprise.shape[1]
        update = torch.zeros_like(update[:, -n:])
    return update, m_last, buf
