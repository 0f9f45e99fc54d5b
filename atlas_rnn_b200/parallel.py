"""Multi-GPU execution of the memory recurrence.

* Batch*head sharding (``shard_units``): units are independent (the reference's
  batch-independence test, tests/test_rnn_all.py:996-1027), so a rank simply runs
  its own slice of N; no collective on the data path.
* Sequence parallelism (``seq_parallel_memory``): rank r holds tokens
  [r*T/P, (r+1)*T/P) of every unit. Each rank runs its chunk pass from a zero
  carry and gets its segment transform
      forward:  (S, Z)   -> (a S + b Z + dS, c Z + dZ)
      backward: (FS, FZ) -> (a FS + dFS, b FS + c FZ + dFZ)
  The transforms compose associatively -- the split-scan identity of the
  reference (tests/test_titans.py:680-707) -- so ranks all-gather them over NCCL
  and each composes the ones before it (forward) or after it (backward) into
  its carry. The transforms travel as one packed record per rank in a single
  all-gather, and the composition runs on the device (``compose_carries_device``
  over ``atlas_mem_compose_carries``); ``compose_forward_carries`` /
  ``compose_backward_carries`` state the same composition in torch ops and are
  what the kernel is tested against. S_ref is the call-start state of the whole
  sequence on every rank (rnn_memory.py:284,298); its gradient is summed over ranks. Window e = 1 only
  (a wider window would need an (e-1)-token halo from the previous rank).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist
from torch import Tensor

from . import _lib
from .ops import Spec, _shape, _stream


def shard_units(N: int, rank: int, world: int) -> slice:
    """Contiguous batch*head slice of a rank (units are independent)."""
    per = (N + world - 1) // world
    return slice(min(N, rank * per), min(N, (rank + 1) * per))


# ---------------------------------------------------------------------------
# transform composition in torch ops (the specification of atlas_mem_compose_carries)
# ---------------------------------------------------------------------------
def _c(coef, i):
    return coef[:, i, None, None]


def compose_forward_carries(coefs, dSs, dZs, S0: Tensor, Z0: Tensor):
    """Incoming (S, Z) of every rank, and the state after the last rank."""
    S, Z = S0, Z0
    carries = []
    for a_b_c, dS, dZ in zip(coefs, dSs, dZs):
        carries.append((S, Z))
        S, Z = _c(a_b_c, 0) * S + _c(a_b_c, 1) * Z + dS, _c(a_b_c, 2) * Z + dZ
    return carries, (S, Z)


def compose_backward_carries(coefs, dFSs, dFZs, FS_end: Tensor, FZ_end: Tensor):
    """Adjoint arriving at the end of every rank's segment, and the adjoint at the
    start of the sequence (gradients of S0, Z0)."""
    P = len(coefs)
    FS, FZ = FS_end, FZ_end
    incoming = [None] * P
    for r in range(P - 1, -1, -1):
        incoming[r] = (FS, FZ)
        a_b_c = coefs[r]
        FS, FZ = _c(a_b_c, 0) * FS + dFSs[r], _c(a_b_c, 1) * FS + _c(a_b_c, 2) * FZ + dFZs[r]
    return incoming, (FS, FZ)


# ---------------------------------------------------------------------------
# one segment through the C ABI
# ---------------------------------------------------------------------------
class Segment:
    """A token segment of every unit, run through the *_local / *_finish entry points."""

    def __init__(self, spec: Spec, k, q, v, lr, decay, beta, S_ref):
        if spec.window != 1:
            raise ValueError("sequence parallelism needs window == 1")
        self.spec = spec
        self.k, self.q, self.v, self.lr, self.decay, self.beta, self.S_ref = k, q, v, lr, decay, beta, S_ref
        N, T, _ = k.shape
        self.N, self.T = N, T
        self.d_v, self.d_phi = v.shape[-1], S_ref.shape[-1]
        self.shape = _shape(spec, k, v, self.d_phi)
        saved_b, _, bwd_b = _lib.workspace_sizes(self.shape)
        dev = k.device
        self.saved = torch.empty(max(saved_b, 1), dtype=torch.uint8, device=dev)
        self.bwd_bytes = bwd_b
        self.dev = dev

    def _fwd_struct(self, S0=None, Z0=None, y=None, S_end=None, Z_end=None):
        p = _lib.ptr
        return _lib.Fwd(k=p(self.k), q=p(self.q), v=p(self.v), lr=p(self.lr), decay=p(self.decay),
                        beta=p(self.beta), gate=None, S_ref=p(self.S_ref),
                        S0=p(S0) if S0 is not None else p(self.S_ref), Z0=p(Z0), buf_in=None, proj=None,
                        y=p(y), S_end=p(S_end), Z_end=p(Z_end), buf_out=None,
                        status=p(_lib.status_word(self.dev)))

    def record_len(self) -> int:
        """Floats in one packed segment-transform record: coef [N,3] (padded to a
        multiple of 4), dS [N,d_v,d_phi], dZ [N,d_v,d_phi]."""
        return (self.N * 3 + 3) // 4 * 4 + 2 * self.N * self.d_v * self.d_phi

    def _seg_bufs(self):
        """A packed record and its three views, so one collective moves all of it."""
        rec = torch.empty(self.record_len(), device=self.dev)
        cl, nd2 = (self.N * 3 + 3) // 4 * 4, self.N * self.d_v * self.d_phi
        coef = rec[:self.N * 3].view(self.N, 3)
        dS = rec[cl:cl + nd2].view(self.N, self.d_v, self.d_phi)
        dZ = rec[cl + nd2:cl + 2 * nd2].view(self.N, self.d_v, self.d_phi)
        self.record = rec
        return coef, dS, dZ

    def forward_local(self):
        coef, dS, dZ = self._seg_bufs()
        f = self._fwd_struct()
        p = _lib.ptr
        _lib.check(_lib.lib().atlas_mem_forward_local(ctypes.byref(self.shape), ctypes.byref(f), p(self.saved),
                                                       self.saved.numel(), None, 0, p(coef), p(dS), p(dZ),
                                                       _stream(self.dev)), "forward_local")
        return coef, dS, dZ

    def forward_finish(self, S_in, Z_in):
        y = torch.empty(self.N, self.T, self.d_v, dtype=self.k.dtype, device=self.dev)
        S_end = torch.empty(self.N, self.d_v, self.d_phi, device=self.dev)
        Z_end = torch.empty_like(S_end) if self.spec.momentum else None
        self.S_in, self.Z_in = S_in.contiguous(), (Z_in.contiguous() if Z_in is not None else None)
        f = self._fwd_struct(self.S_in, self.Z_in, y, S_end, Z_end)
        _lib.check(_lib.lib().atlas_mem_forward_finish(ctypes.byref(self.shape), ctypes.byref(f),
                                                        _lib.ptr(self.saved), self.saved.numel(), None, 0,
                                                        _stream(self.dev)), "forward_finish")
        return y, S_end, Z_end

    def _bwd_struct(self, dy, FS=None, FZ=None, grads=None):
        p = _lib.ptr
        g = grads or {}
        return _lib.Bwd(dy=p(dy), dS_end=p(FS), dZ_end=p(FZ), dbuf_out=None, dk=p(g.get("k")), dq=p(g.get("q")),
                        dv=p(g.get("v")), dlr=p(g.get("lr")), ddecay=p(g.get("decay")), dbeta=p(g.get("beta")),
                        dgate=None, dS_ref=p(g.get("S_ref")), dS0=p(g.get("S0")), dZ0=p(g.get("Z0")),
                        dbuf_in=None, status=p(_lib.status_word(self.dev)))

    def backward_local(self, dy):
        self.scratch = torch.empty(max(self.bwd_bytes, 1), dtype=torch.uint8, device=self.dev)
        coef, dS, dZ = self._seg_bufs()
        f = self._fwd_struct(self.S_in, self.Z_in)
        b = self._bwd_struct(dy)
        p = _lib.ptr
        _lib.check(_lib.lib().atlas_mem_backward_local(ctypes.byref(self.shape), ctypes.byref(f), ctypes.byref(b),
                                                        p(self.saved), self.saved.numel(), p(self.scratch),
                                                        self.scratch.numel(), p(coef), p(dS), p(dZ),
                                                        _stream(self.dev)), "backward_local")
        return coef, dS, dZ

    def backward_finish(self, dy, FS, FZ, apply_mask: bool, need=None):
        """Input gradients of this segment; `need` names the ones to produce (default: all)."""
        names = [("k", self.k), ("q", self.q), ("v", self.v), ("lr", self.lr), ("decay", self.decay),
                 ("S_ref", self.S_ref), ("S0", self.S_ref)]
        if self.spec.momentum:
            names += [("beta", self.beta), ("Z0", self.S_ref)]
        g = {n: torch.empty_like(t) for n, t in names if need is None or n in need}
        f = self._fwd_struct(self.S_in, self.Z_in)
        b = self._bwd_struct(dy, FS.contiguous(), FZ.contiguous() if FZ is not None else None, g)
        p = _lib.ptr
        _lib.check(_lib.lib().atlas_mem_backward_finish(ctypes.byref(self.shape), ctypes.byref(f), ctypes.byref(b),
                                                         p(self.saved), self.saved.numel(), p(self.scratch),
                                                         self.scratch.numel(), int(apply_mask),
                                                         _stream(self.dev)), "backward_finish")
        return g


def _gather_records(seg: Segment, group) -> Tensor:
    """All ranks' packed segment-transform records, [world, record_len], in one all-gather."""
    P = dist.get_world_size(group)
    out = torch.empty(P, seg.record.numel(), device=seg.dev)
    dist.all_gather_into_tensor(out, seg.record, group=group)
    return out


def compose_carries_device(seg: Segment, records: Tensor, rank: int, backward: bool, S0, Z0, S_T=None,
                           clamped: bool = False):
    """The carry composition of compose_forward_carries / compose_backward_carries as one
    kernel (atlas_mem_compose_carries) over the gathered records.
    Returns (in_S, in_Z, out_S, out_S_clamped or None, out_Z)."""
    N, d2 = seg.N, seg.d_v * seg.d_phi
    shp = (N, seg.d_v, seg.d_phi)
    new = lambda: torch.empty(shp, device=seg.dev)
    in_S, in_Z, out_S, out_Z = new(), new(), new(), new()
    out_Sc = new() if clamped else None
    p = _lib.ptr
    c = lambda t: None if t is None else t.contiguous()
    S0, Z0, S_T = c(S0), c(Z0), c(S_T)
    _lib.check(_lib.lib().atlas_mem_compose_carries(p(records), records.shape[1], records.shape[0], rank, N, d2,
                                                    int(backward), p(S0), p(Z0), p(S_T), p(in_S), p(in_Z),
                                                    p(out_S), p(out_Sc), p(out_Z), _stream(seg.dev)),
               "compose_carries")
    return in_S, in_Z, out_S, out_Sc, out_Z


class SeqParallelMemoryFn(torch.autograd.Function):
    """Memory recurrence over a sequence split across the ranks of `group`."""

    @staticmethod
    def forward(ctx, spec: Spec, group, k, q, v, lr, decay, beta, S_ref, S0, Z0):
        seg = Segment(spec, k, q, v, lr, decay, beta, S_ref)
        seg.forward_local()
        r = dist.get_rank(group)
        records = _gather_records(seg, group)
        S_in, Z_in, S_T, S_end, Z_T = compose_carries_device(seg, records, r, False, S0, Z0, clamped=True)
        y, _, _ = seg.forward_finish(S_in, Z_in if spec.momentum else None)
        ctx.seg, ctx.group, ctx.spec, ctx.S_T = seg, group, spec, S_T
        ctx.set_materialize_grads(False)
        Z_end = Z_T if spec.momentum else S_T.new_empty(0)
        return y, S_end, Z_end

    @staticmethod
    def backward(ctx, dy, dS_end, dZ_end):
        seg, group, spec = ctx.seg, ctx.group, ctx.spec
        r = dist.get_rank(group)
        if dy is None:
            dy = torch.zeros(seg.N, seg.T, seg.d_v, dtype=seg.k.dtype, device=seg.dev)
        dy = dy.contiguous()
        seg.backward_local(dy)
        records = _gather_records(seg, group)
        # every rank returned the same S_end / Z_end: their upstream gradients add up
        # (one all-reduce of both; a fresh buffer, so the caller's tensors stay as they are)
        ends = torch.zeros((2,) + tuple(ctx.S_T.shape), device=seg.dev)
        if dS_end is not None:
            ends[0].copy_(dS_end)
        if dZ_end is not None and dZ_end.numel() != 0:
            ends[1].copy_(dZ_end)
        dist.all_reduce(ends, group=group)
        FS, FZ, dS0, _, dZ0 = compose_carries_device(seg, records, r, True, ends[0], ends[1], S_T=ctx.S_T)
        flags = ctx.needs_input_grad  # (spec, group, k, q, v, lr, decay, beta, S_ref, S0, Z0)
        need = {n for n, f in zip(("k", "q", "v", "lr", "decay", "beta", "S_ref"), flags[2:9]) if f}
        g = seg.backward_finish(dy, FS, FZ if spec.momentum else None, apply_mask=False, need=need)
        if "S_ref" in g:
            dist.all_reduce(g["S_ref"], group=group)
        return (None, None, g.get("k"), g.get("q"), g.get("v"), g.get("lr"), g.get("decay"), g.get("beta"),
                g.get("S_ref"), dS0 if flags[9] else None, dZ0 if (spec.momentum and flags[10]) else None)


def seq_parallel_memory(k, q, v, lr, decay, beta, *, S_ref, S0, Z0=None, group=None, fmap_mode="off",
                        fmap_degree=1):
    """Sequence-parallel memory recurrence (window 1, no omega gate). Every rank
    passes its own token slice of k, q, v, lr, decay, beta and the same S_ref, S0,
    Z0; returns this rank's y and the state after the whole sequence."""
    group = group or dist.group.WORLD
    io = torch.bfloat16 if k.dtype == torch.bfloat16 else torch.float32
    spec = Spec(window=1, gate_mode=_lib.GATE_NONE, fmap_mode=fmap_mode if fmap_degree > 1 else "off",
                fmap_degree=fmap_degree, momentum=beta is not None)
    cv = lambda t: None if t is None else t.to(io).contiguous()
    f32 = lambda t: None if t is None else t.float().contiguous()
    y, S_end, Z_end = SeqParallelMemoryFn.apply(spec, group, cv(k), cv(q), cv(v), cv(lr), cv(decay), cv(beta),
                                                f32(S_ref), f32(S0), f32(Z0))
    return y, S_end, (Z_end if beta is not None else None)
