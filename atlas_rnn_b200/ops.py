"""Autograd boundary of the memory recurrence over the C ABI.

``memory_recurrence`` is the functional form of the block the reference cells
run inside ``_forward_impl`` (rnn_memory.py:345-393 Titans, :655-717 Omega)
and of ``AtlasOmegaFunction.apply`` (cuda/atlas_omega_autograd.py:98-204),
taking the per-head raw q/k (the feature map is applied in the kernels).
All arithmetic happens in libatlas_mem.so on the caller's current CUDA stream;
this file only checks arguments, allocates outputs / workspaces with torch and
passes pointers.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import Tensor

from . import _lib


@dataclass(frozen=True)
class Spec:
    window: int = 1
    gate_mode: int = _lib.GATE_NONE
    fmap_mode: str = "off"
    fmap_degree: int = 1
    momentum: bool = True
    chunk: int = 0


def _shape(spec: Spec, k: Tensor, v: Tensor, d_phi: int) -> _lib.Shape:
    N, T, dk = k.shape
    return _lib.Shape(N=N, T=T, d_k=dk, d_phi=d_phi, d_v=v.shape[-1], window=spec.window,
                      fmap_mode=_lib.FMAP[spec.fmap_mode], fmap_degree=spec.fmap_degree,
                      gate_mode=spec.gate_mode, momentum=int(spec.momentum),
                      dtype_io=_lib.BF16 if k.dtype == torch.bfloat16 else _lib.F32, chunk=spec.chunk)


def _stream(dev) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


class MemoryRecurrenceFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, spec: Spec, k, q, v, lr, decay, beta, gate, S_ref, S0, Z0, buf, proj):
        ctx.set_materialize_grads(False)  # unused outputs arrive as None, not zero tensors
        dev = k.device
        N, T, _ = k.shape
        d_phi = S_ref.shape[-1]
        d_v = v.shape[-1]
        shape = _shape(spec, k, v, d_phi)
        saved_b, _, bwd_b = _lib.workspace_sizes(shape)
        saved = torch.empty(max(saved_b, 1), dtype=torch.uint8, device=dev)
        y = torch.empty(N, T, d_v, dtype=k.dtype, device=dev)
        S_end = torch.empty(N, d_v, d_phi, dtype=torch.float32, device=dev)
        Z_end = torch.empty_like(S_end) if spec.momentum else S_end.new_empty(0)
        e = spec.window
        buf_out = (torch.empty(N, e - 1, d_v, d_phi, dtype=torch.float32, device=dev) if e > 1
                   else S_end.new_empty(0))
        p = _lib.ptr
        fwd = _lib.Fwd(k=p(k), q=p(q), v=p(v), lr=p(lr), decay=p(decay), beta=p(beta), gate=p(gate),
                       S_ref=p(S_ref), S0=p(S0), Z0=p(Z0), buf_in=p(buf), proj=p(proj), y=p(y),
                       S_end=p(S_end), Z_end=p(Z_end) if spec.momentum else None,
                       buf_out=p(buf_out) if e > 1 else None, status=p(_lib.status_word(dev)))
        _lib.check(_lib.lib().atlas_mem_forward(ctypes.byref(shape), ctypes.byref(fwd), p(saved),
                                                 saved.numel(), None, 0, _stream(dev)), "forward")
        ctx.spec, ctx.shape, ctx.bwd_bytes = spec, shape, bwd_b
        ctx.saved_ws = saved
        ctx.save_for_backward(k, q, v, lr, decay, beta, gate, S_ref, S0, Z0, buf, proj)
        ctx.mark_non_differentiable(*([] if spec.momentum else [Z_end]), *([] if e > 1 else [buf_out]))
        return y, S_end, Z_end, buf_out

    @staticmethod
    def backward(ctx, dy, dS_end, dZ_end, dbuf_out):
        k, q, v, lr, decay, beta, gate, S_ref, S0, Z0, buf, proj = ctx.saved_tensors
        spec, shape = ctx.spec, ctx.shape
        dev = k.device
        need = ctx.needs_input_grad  # (spec, k, q, v, lr, decay, beta, gate, S_ref, S0, Z0, buf, proj)
        if dy is None:
            dy = torch.zeros(k.shape[0], k.shape[1], v.shape[-1], dtype=k.dtype, device=dev)
        dy = dy.to(k.dtype).contiguous()
        f32c = lambda t: None if t is None or t.numel() == 0 else t.float().contiguous()
        dS_end, dZ_end, dbuf_out = f32c(dS_end), f32c(dZ_end), f32c(dbuf_out)
        e = spec.window

        def out_like(t, flag):
            return torch.empty_like(t) if (t is not None and flag) else None

        dk, dq, dv = out_like(k, need[1]), out_like(q, need[2]), out_like(v, need[3])
        dlr, ddecay = out_like(lr, need[4]), out_like(decay, need[5])
        dbeta, dgate = out_like(beta, need[6]), out_like(gate, need[7])
        dS_ref, dS0 = out_like(S_ref, need[8]), out_like(S0, need[9])
        dZ0 = out_like(Z0, need[10])
        dbuf = None
        if e > 1 and need[11] and buf is not None:
            dbuf = torch.empty_like(buf)
        scratch = torch.empty(max(ctx.bwd_bytes, 1), dtype=torch.uint8, device=dev)
        p = _lib.ptr
        fwd = _lib.Fwd(k=p(k), q=p(q), v=p(v), lr=p(lr), decay=p(decay), beta=p(beta), gate=p(gate),
                       S_ref=p(S_ref), S0=p(S0), Z0=p(Z0), buf_in=p(buf), proj=p(proj),
                       status=p(_lib.status_word(dev)))
        bwd = _lib.Bwd(dy=p(dy), dS_end=p(dS_end), dZ_end=p(dZ_end), dbuf_out=p(dbuf_out), dk=p(dk),
                       dq=p(dq), dv=p(dv), dlr=p(dlr), ddecay=p(ddecay), dbeta=p(dbeta), dgate=p(dgate),
                       dS_ref=p(dS_ref), dS0=p(dS0), dZ0=p(dZ0), dbuf_in=p(dbuf),
                       status=p(_lib.status_word(dev)))
        saved = ctx.saved_ws
        _lib.check(_lib.lib().atlas_mem_backward(ctypes.byref(shape), ctypes.byref(fwd), ctypes.byref(bwd),
                                                  p(saved), saved.numel(), p(scratch), scratch.numel(),
                                                  _stream(dev)), "backward")
        return (None, dk, dq, dv, dlr, ddecay, dbeta, dgate, dS_ref, dS0, dZ0, dbuf, None)


def _io(t: Tensor | None, dtype) -> Tensor | None:
    return None if t is None else t.to(dtype).contiguous()


def decode_supported(spec: Spec, d_k: int, d_phi: int, d_v: int) -> bool:
    """Shapes atlas_mem_decode_step handles (T = 1, no tensor feature map, heads up to 256)."""
    return spec.fmap_mode != "tensor" and d_phi <= 256 and d_v <= 256


def decode_step(spec: Spec, k, q, v, lr, decay, beta, gate, S_ref, S0, Z0, buf, proj):
    """One token (T = 1) through atlas_mem_decode_step: inference only, no autograd
    graph, no workspaces. Operands as for MemoryRecurrenceFn (io dtype for k..gate,
    fp32 states)."""
    dev = k.device
    N, T, _ = k.shape
    d_phi, d_v = S_ref.shape[-1], v.shape[-1]
    shape = _shape(spec, k, v, d_phi)
    y = torch.empty(N, T, d_v, dtype=k.dtype, device=dev)
    S_end = torch.empty(N, d_v, d_phi, dtype=torch.float32, device=dev)
    Z_end = torch.empty_like(S_end) if spec.momentum else S_end.new_empty(0)
    e = spec.window
    buf_out = (torch.empty(N, e - 1, d_v, d_phi, dtype=torch.float32, device=dev) if e > 1
               else S_end.new_empty(0))
    p = _lib.ptr
    fwd = _lib.Fwd(k=p(k), q=p(q), v=p(v), lr=p(lr), decay=p(decay), beta=p(beta), gate=p(gate),
                   S_ref=p(S_ref), S0=p(S0), Z0=p(Z0), buf_in=p(buf), proj=p(proj), y=p(y),
                   S_end=p(S_end), Z_end=p(Z_end) if spec.momentum else None,
                   buf_out=p(buf_out) if e > 1 else None)
    _lib.check(_lib.lib().atlas_mem_decode_step(ctypes.byref(shape), ctypes.byref(fwd), _stream(dev)),
               "decode_step")
    return y, S_end, Z_end, buf_out


TC_D = 128  # state side of the tensor-core kernels


def _pad_to_tc(spec: Spec, io, d_k: int, d_phi: int, d_v: int) -> bool:
    """bf16 heads narrower than the tensor-core kernels' 128 x 128 state run those kernels
    on zero-padded heads (feature map off or elementwise, so d_phi = d_k). Exact: with
    zero-padded phi(k), phi(q), v, S_ref, S0, Z0 and buffer, the padded rows of delta are
    S_ref[pad] phi - 0 = 0 and every padded column is multiplied by phi[pad] = 0, so the
    padded part of every state stays zero and the outputs are the unpadded ones.
    ATLAS_MEM_PAD128=0 keeps such heads on the CUDA-core kernels."""
    if io != torch.bfloat16 or spec.fmap_mode == "tensor" or spec.window > 16:
        return False
    if not (d_phi == d_k and d_phi < TC_D and d_v <= TC_D):
        return False
    return os.environ.get("ATLAS_MEM_PAD128", "1") != "0" and os.environ.get("ATLAS_MEM_TC", "1") != "0"


def _padded_call(spec: Spec, d_v: int, d_phi: int, k, q, v, lr, decay, beta, gate, S_ref, S0, Z0, buf, proj,
                 vectors_padded: bool = False):
    pk, pv = TC_D - d_phi, TC_D - d_v
    vec = (lambda t, p: t) if vectors_padded else (lambda t, p: F.pad(t, (0, p)))  # [.., d] -> [.., 128]
    mat = lambda t: None if t is None else F.pad(t, (0, pk, 0, pv))  # [.., d_v, d_phi] -> [.., 128, 128]
    y, S_end, Z_end, buf_out = MemoryRecurrenceFn.apply(spec, vec(k, pk), vec(q, pk), vec(v, pv), lr, decay,
                                                        beta, gate, mat(S_ref), mat(S0), mat(Z0), mat(buf), proj)
    cut = lambda t: t[..., :d_v, :d_phi] if t is not None and t.numel() else t
    return y[..., :d_v], cut(S_end), cut(Z_end), cut(buf_out)


class FmapTensorFn(torch.autograd.Function):
    """phi = [x; vec(x x^T)] Proj (rnn_memory.py:125-130) for bf16 x [..., d_k] on the
    tensor cores (atlas_fmap_tensor_forward / _backward); phi bf16 [..., d_phi]. Proj is
    a fixed buffer (no gradient)."""

    @staticmethod
    def forward(ctx, x, proj):
        d_k, d_phi = x.shape[-1], proj.shape[-1]
        rows = x.numel() // d_k
        L = _lib.lib()
        tiles = torch.empty(L.atlas_fmap_tensor_workspace(d_k, d_phi), dtype=torch.uint8, device=x.device)
        phi = torch.empty(*x.shape[:-1], d_phi, dtype=torch.bfloat16, device=x.device)
        p = _lib.ptr
        _lib.check(L.atlas_fmap_tensor_forward(rows, d_k, d_phi, p(x), p(proj), p(tiles), p(phi),
                                               p(_lib.status_word(x.device)), _stream(x.device)), "fmap forward")
        ctx.save_for_backward(x, tiles)
        ctx.d_phi = d_phi
        return phi

    @staticmethod
    def backward(ctx, dphi):
        x, tiles = ctx.saved_tensors
        d_k = x.shape[-1]
        dphi = dphi.to(torch.bfloat16).contiguous()
        dx = torch.empty_like(x)
        p = _lib.ptr
        _lib.check(_lib.lib().atlas_fmap_tensor_backward(x.numel() // d_k, d_k, ctx.d_phi, p(x), p(tiles),
                                                         p(dphi), p(dx), p(_lib.status_word(x.device)),
                                                         _stream(x.device)), "fmap backward")
        return dx, None


def _fmap_tc_ok(d_k: int, d_phi: int) -> bool:
    return 16 <= d_k <= 64 and d_k % 16 == 0 and 16 <= d_phi <= 256 and d_phi % 16 == 0


def _split_phi_call(k, q, v, lr, decay, beta, gate, S_ref, S0, Z0, buf, proj, *, window, gate_mode, fmap_degree,
                    chunk):
    """The tensor feature map with d_phi = H * 128 (benchmark config 4: 256): phi(k), phi(q) on
    the tensor cores, then the recurrence as H units of d_phi = 128 each. The state splits by
    columns, S = [S_1 | .. | S_H], and every part evolves with the same gates and the same
    delta_t = S_ref phi_t - v_t = sum_g S_ref,g phi_g,t - v_t, so part h is the d_phi = 128
    recurrence with keys phi_h, queries psi_h, S_ref,h and values
    v_h = v - sum_{g != h} phi_g S_ref,g^T (which reproduces delta exactly); y is the sum of
    the parts' outputs (S_{t-1} psi_t = sum_h S_h,t-1 psi_h,t, the within-chunk terms too),
    and S_end, Z_end and the omega buffer are the parts side by side. The H parts run as
    H N units in one call of the tensor-core kernels; autograd carries the gradients through
    the split, the value adjustment (one batched GEMM) and the feature map."""
    N, T, _ = k.shape
    d_phi = S_ref.shape[-1]
    H = d_phi // TC_D
    phik = FmapTensorFn.apply(k.contiguous(), proj)
    phiq = FmapTensorFn.apply(q.contiguous(), proj)
    parts = lambda t: [t[..., h * TC_D:(h + 1) * TC_D] for h in range(H)]
    pk, pq, pr = parts(phik), parts(phiq), parts(S_ref)
    preds = [torch.bmm(pk[h].float(), pr[h].transpose(1, 2)) for h in range(H)]  # phi_h S_ref,h^T, fp32
    total = preds[0]
    for h in range(1, H):
        total = total + preds[h]
    vf = v.float()
    vs = [(vf - (total - preds[h])).to(v.dtype) for h in range(H)]
    cat = lambda ts: None if ts is None else torch.cat(ts, dim=0).contiguous()
    rep = lambda t: None if t is None else t.repeat(H, *([1] * (t.dim() - 1)))
    colparts = lambda t: None if t is None else cat(parts(t))
    y2, S2, Z2, b2 = memory_recurrence(cat(pk), cat(pq), cat(vs), rep(lr), rep(decay), rep(beta), rep(gate),
                                       S_ref=cat(pr), S0=colparts(S0), Z0=colparts(Z0), omega_buffer=colparts(buf),
                                       window=window, gate_mode=gate_mode, fmap_mode="off", fmap_degree=1,
                                       chunk=chunk)
    y = y2[:N]
    for h in range(1, H):
        y = y + y2[h * N:(h + 1) * N]
    join = lambda t: None if t is None else torch.cat([t[h * N:(h + 1) * N] for h in range(H)], dim=-1)
    return y, join(S2), join(Z2), join(b2)


def _chunk_ref_mode(k, q, v, lr, decay, beta, gate, *, S0, Z0, omega_buffer, window, gate_mode, fmap_mode,
                    fmap_degree, proj, chunk, ref_chunk):
    """ref_mode 'chunk' as consecutive calls whose reference state is their own start state."""
    if not ref_chunk or ref_chunk < 1:
        raise ValueError("ref_mode='chunk' needs ref_chunk >= 1 (tokens per reference state)")
    T = k.shape[1]
    S, Z, buf, ys = S0, Z0, omega_buffer, []
    cut = lambda t, lo, hi: None if t is None else t[:, lo:hi]
    for lo in range(0, T, ref_chunk):
        hi = min(T, lo + ref_chunk)
        y, S, Z, buf = memory_recurrence(cut(k, lo, hi), cut(q, lo, hi), cut(v, lo, hi), cut(lr, lo, hi),
                                         cut(decay, lo, hi), cut(beta, lo, hi), cut(gate, lo, hi), S_ref=S, S0=S,
                                         Z0=Z, omega_buffer=buf, window=window, gate_mode=gate_mode,
                                         fmap_mode=fmap_mode, fmap_degree=fmap_degree, proj=proj, chunk=chunk)
        ys.append(y)
    return torch.cat(ys, dim=1), S, Z, buf


def memory_recurrence(k: Tensor, q: Tensor, v: Tensor, lr: Tensor, decay: Tensor,
                      beta: Tensor | None = None, gate: Tensor | None = None, *, S_ref: Tensor,
                      S0: Tensor, Z0: Tensor | None = None, omega_buffer: Tensor | None = None,
                      window: int = 1, gate_mode: str | None = None, fmap_mode: str = "off",
                      fmap_degree: int = 1, proj: Tensor | None = None, chunk: int = 0,
                      ref_mode: str = "call", ref_chunk: int | None = None, heads_padded_from: tuple | None = None):
    """Memory recurrence over N = batch*heads units.

    k, q [N,T,d_k]; v [N,T,d_v]; lr (eta), decay (alpha), beta [N,T]; gate [N,T]
    (gate_mode 'token', the reference's omega gate u) or [N,T,e] (gate_mode
    'window', per-position window weights U[t, j] on the term of token t-j);
    S_ref, S0, Z0 [N,d_v,d_phi]; omega_buffer [N,e-1,d_v,d_phi].
    Returns (y [N,T,d_v], S_end (clamped to +-100), Z_end or None, new omega buffer or None).
    io tensors run in bfloat16 when k is bfloat16 or bf16 autocast is on (as autocast runs the
    reference's einsums), else float32; states in float32.
    A single token (T = 1) with no autograd graph to record runs as one decode
    kernel (atlas_mem_decode_step) unless the tensor feature map is on.
    ref_mode 'call' (default, the reference's semantics): every token's delta uses S_ref.
    ref_mode 'chunk': the chunk-start state is the reference state -- the sequence runs as
    consecutive calls of ref_chunk tokens, each with S_ref = S0 = the state (clamped to
    +-100) the call before returned, carrying Z and the omega buffer; S_ref is then unused.
    That is the reference cell called once per chunk in a loop (tests/test_rnn_all.py:804-825).
    heads_padded_from=(d_v, d_phi): k, q, v arrive zero-padded to 128 columns (``head_prep``)
    for states of d_v x d_phi; the states are padded here and the outputs cut back.
    """
    if ref_mode == "chunk":
        return _chunk_ref_mode(k, q, v, lr, decay, beta, gate, S0=S0, Z0=Z0, omega_buffer=omega_buffer,
                               window=window, gate_mode=gate_mode, fmap_mode=fmap_mode, fmap_degree=fmap_degree,
                               proj=proj, chunk=chunk, ref_chunk=ref_chunk)
    if ref_mode != "call":
        raise ValueError(f"ref_mode must be 'call' or 'chunk', not {ref_mode!r}")
    if not k.is_cuda:
        raise RuntimeError("atlas_rnn_b200.memory_recurrence: tensors must be on a CUDA device "
                           "(the library has no CPU path)")
    io = torch.bfloat16 if k.dtype == torch.bfloat16 else torch.float32
    if torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16:
        io = torch.bfloat16  # a matmul-like op under bf16 autocast: bf16 operands, fp32 state and accumulation
    d_phi = S_ref.shape[-1]
    if (fmap_mode == "tensor" and fmap_degree > 1 and io == torch.bfloat16 and heads_padded_from is None
            and d_phi > TC_D and d_phi % TC_D == 0 and v.shape[-1] <= TC_D and window <= 16
            and _fmap_tc_ok(k.shape[-1], d_phi) and os.environ.get("ATLAS_MEM_TC", "1") != "0"):
        f32 = lambda t: None if t is None else t.to(torch.float32)
        y, S_end, Z_end, buf_out = _split_phi_call(
            _io(k, io), _io(q, io), _io(v, io), _io(lr, io), _io(decay, io), _io(beta, io), _io(gate, io),
            f32(S_ref), f32(S0), f32(Z0) if beta is not None else None, f32(omega_buffer) if window > 1 else None,
            proj.to(torch.float32).contiguous(), window=window, gate_mode=gate_mode, fmap_degree=fmap_degree,
            chunk=chunk)
        S_end = S_end.to(S0.dtype)
        Z_end = Z_end.to(S0.dtype) if beta is not None else None
        return y, S_end, Z_end, buf_out
    if gate is None:
        gm = _lib.GATE_NONE
    elif gate_mode == "window" or (gate_mode is None and gate.dim() == 3):
        gm = _lib.GATE_WINDOW
    else:
        gm = _lib.GATE_TOKEN
    momentum = beta is not None
    spec = Spec(window=window, gate_mode=gm, fmap_mode=fmap_mode if fmap_degree > 1 else "off",
                fmap_degree=fmap_degree, momentum=momentum, chunk=chunk)
    state_dtype = S0.dtype
    f32 = lambda t: None if t is None else t.to(torch.float32).contiguous()
    Z0c = f32(Z0) if momentum else None
    buf = f32(omega_buffer) if window > 1 else None
    projc = f32(proj) if spec.fmap_mode == "tensor" else None
    args = (_io(k, io), _io(q, io), _io(v, io), _io(lr, io), _io(decay, io), _io(beta, io), _io(gate, io),
            f32(S_ref), f32(S0), Z0c, buf, projc)
    needs_grad = torch.is_grad_enabled() and any(
        t is not None and t.requires_grad for t in (k, q, v, lr, decay, beta, gate, S_ref, S0, Z0, omega_buffer))
    if (heads_padded_from is None and k.shape[1] == 1 and not needs_grad
            and decode_supported(spec, k.shape[-1], S_ref.shape[-1], v.shape[-1])):
        y, S_end, Z_end, buf_out = decode_step(spec, *args)
    elif heads_padded_from is not None:  # k, q, v already zero-padded to 128 columns (head_prep)
        y, S_end, Z_end, buf_out = _padded_call(spec, heads_padded_from[0], heads_padded_from[1], *args,
                                                vectors_padded=True)
    elif _pad_to_tc(spec, io, k.shape[-1], S_ref.shape[-1], v.shape[-1]):
        y, S_end, Z_end, buf_out = _padded_call(spec, v.shape[-1], S_ref.shape[-1], *args)
    else:
        y, S_end, Z_end, buf_out = MemoryRecurrenceFn.apply(spec, *args)
    S_end = S_end.to(state_dtype)
    Z_end = Z_end.to(state_dtype) if momentum else None
    buf_out = buf_out.to(state_dtype) if window > 1 else None
    return y, S_end, Z_end, buf_out
