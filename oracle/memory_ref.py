"""CPU restatement of the Atlas-RNN memory recurrence (test infrastructure only).

Boundary: the reference cell's recurrence core, taking the per-head tensors that
``_forward_impl`` builds after projections / norms (rnn_memory.py:624-653):

    k, q   [N, T, d_k]   raw (normalised) keys / queries, N = batch*heads
    v      [N, T, d_v]
    lr     [N, T]  eta      (to_lr,        rnn_memory.py:645)
    decay  [N, T]  alpha    (to_decay,     rnn_memory.py:646)
    beta   [N, T]  or None  (to_momentum,  rnn_memory.py:649; None = momentum off)
    gate   [N, T]  or None  (to_omega_gate rnn_memory.py:653; per-token u)
    U      [N, T, e] or None  window-position gates (generalisation, see below)
    S_ref  [N, d_v, d_phi]    state the deltas are taken against (rnn_memory.py:284,298)
    S0, Z0 [N, d_v, d_phi]    carried state (Z0 None = zeros, rnn_memory.py:693)
    buf    [N, e-1, d_v, d_phi] or None   carried omega_buffer (rnn_memory.py:674-678)

Every step follows the reference line it cites. The torch version is run under
autograd so the gradients are exactly the reference's own autograd gradients.

Window-gate generalisation (``U``): the reference gates each token once,
g_raw_t = u_t * delta_t phi_t^T (rnn_memory.py:666-668), then sums a window of e
(rnn_memory.py:680-681). ``U[t, j]`` instead weights the term of token t-j inside
g_t: g_t = sum_{j<e} U[t, j] * delta_{t-j} phi_{t-j}^T. With U[t, j] = u_{t-j} this
is the reference exactly. In U mode the carried buffer holds the ungated terms
(the weight depends on the consuming position, so it cannot be folded in).
"""
from __future__ import annotations

import math

import numpy as np
import torch
from torch import Tensor

from .assoc_scan_standin import scalar_assoc_scan


# ---------------------------------------------------------------------------
# feature map: PolynomialFeatureMap.forward (rnn_memory.py:113-132)
# ---------------------------------------------------------------------------
def make_tensor_proj(dim: int, generator: torch.Generator | None = None,
                     dtype=torch.float32) -> Tensor:
    """Fixed projection buffer of the 'tensor' mode (rnn_memory.py:106-111)."""
    feat = dim + dim * dim
    return torch.randn(feat, dim, generator=generator, dtype=dtype) / math.sqrt(feat)


def feature_map(x: Tensor, mode: str = "off", degree: int = 1, proj: Tensor | None = None) -> Tensor:
    if degree <= 1 or mode == "off":                       # :114-115
        return x
    if mode == "elementwise":                              # :117-123
        out = x.clone()
        power = x
        for _ in range(2, degree + 1):
            power = power * x
            out = out + power
        return out
    if mode == "tensor":                                   # :125-130
        d = x.shape[-1]
        outer = torch.einsum("...i,...j->...ij", x, x).reshape(*x.shape[:-1], d * d)
        feats = torch.cat([x, outer], dim=-1)
        return feats @ proj.to(x.device, x.dtype)
    return x


def sliding_sum_along_time(x: Tensor, window: int) -> Tensor:
    """_sliding_sum_along_time (rnn_memory.py:50-61)."""
    if window <= 1:
        return x
    T = x.shape[1]
    window = min(window, T)
    c = x.cumsum(dim=1)
    shifted = torch.cat([c.new_zeros((*c.shape[:1], window, *c.shape[2:])), c[:, :-window]], dim=1)
    return c - shifted


# ---------------------------------------------------------------------------
# recurrence core (rnn_memory.py:655-717; Titans variant :345-393 is e=1, no gate)
# ---------------------------------------------------------------------------
def memory_core(phi_k: Tensor, phi_q: Tensor, v: Tensor, lr: Tensor, decay: Tensor,
                beta: Tensor | None, gate: Tensor | None, S_ref: Tensor, S0: Tensor,
                Z0: Tensor | None, buf: Tensor | None, window: int = 1,
                U: Tensor | None = None, scan=scalar_assoc_scan):
    """Returns (y [N,T,d_v], S_end, Z_end or None, new_buf or None)."""
    N, T, _ = phi_k.shape
    e = window
    pred = torch.einsum("bde,bte->btd", S_ref, phi_k)          # :659
    delta_vec = pred - v                                        # :660
    g_raw = torch.einsum("bti,btj->btij", delta_vec, phi_k)     # :663
    if U is None and gate is not None:                          # :666-668
        g_raw = g_raw * gate[..., None, None]
    if e > 1:                                                   # :673-687
        prev_g = buf if buf is not None else g_raw.new_zeros((N, e - 1, *g_raw.shape[2:]))
        g_ext = torch.cat([prev_g, g_raw], dim=1)
        if U is None:
            g = sliding_sum_along_time(g_ext, e)[:, -T:]
        else:
            # generalised window: g_t = sum_j U[t, j] * g_ext[t + e - 1 - j]
            g = 0
            for j in range(e):
                g = g + U[:, :, j, None, None] * g_ext[:, e - 1 - j: e - 1 - j + T]
        new_buf = g_ext[:, -(e - 1):]
    else:
        g = g_raw if U is None else g_raw * U[:, :, 0, None, None]
        new_buf = None

    if Z0 is None:
        Z0 = torch.zeros_like(S0)
    lr_e = lr[..., None, None]
    if beta is not None:                                        # :697-702
        Z_all = scan(beta, g, prev=Z0)
        S_all = scan(decay, -lr_e * Z_all, prev=S0)
        Z_end = Z_all[:, -1]
    else:                                                       # :703-707
        S_all = scan(decay, -lr_e * g, prev=S0)
        Z_end = None
    S_end = S_all[:, -1].clamp(-100, 100)

    y0 = torch.einsum("bde,be->bd", S0, phi_q[:, 0])            # :712-717
    if T > 1:
        y_rest = torch.einsum("btdp,btp->btd", S_all[:, :-1], phi_q[:, 1:])
        y = torch.cat([y0.unsqueeze(1), y_rest], dim=1)
    else:
        y = y0.unsqueeze(1)
    return y, S_end, Z_end, new_buf


def memory_layer(k, q, v, lr, decay, beta, gate, S_ref, S0, Z0, buf, window=1, U=None,
                 fmap_mode="off", fmap_degree=1, proj=None, scan=scalar_assoc_scan):
    """Feature map (rnn_memory.py:637-642) followed by the recurrence core."""
    phi_k = feature_map(k, fmap_mode, fmap_degree, proj)
    phi_q = feature_map(q, fmap_mode, fmap_degree, proj)
    return memory_core(phi_k, phi_q, v, lr, decay, beta, gate, S_ref, S0, Z0, buf,
                       window=window, U=U, scan=scan)


# ---------------------------------------------------------------------------
# sequential float64 numpy restatement (independent cross-check of the above)
# ---------------------------------------------------------------------------
def memory_core_sequential_np(phi_k, phi_q, v, lr, decay, beta, gate, S_ref, S0, Z0, buf,
                              window=1, U=None):
    """Per-token loop of the same recurrence (rnn_memory.py:7-12 per-token form with
    the fixed S_ref of :284 and the window/carry of :673-687). float64 numpy."""
    phi_k, phi_q, v = (np.asarray(a, np.float64) for a in (phi_k, phi_q, v))
    N, T, dphi = phi_k.shape
    dv = v.shape[2]
    e = window
    S = np.array(S0, np.float64)
    Z = np.zeros_like(S) if Z0 is None else np.array(Z0, np.float64)
    y = np.zeros((N, T, dv))
    hist = []  # window terms, oldest first
    if e > 1:
        b = np.zeros((N, e - 1, dv, dphi)) if buf is None else np.asarray(buf, np.float64)
        hist = [b[:, i] for i in range(e - 1)]
    for t in range(T):
        y[:, t] = np.einsum("nde,ne->nd", S, phi_q[:, t])
        delta = np.einsum("nde,ne->nd", S_ref, phi_k[:, t]) - v[:, t]
        r = np.einsum("ni,nj->nij", delta, phi_k[:, t])
        if U is None and gate is not None:
            r = r * np.asarray(gate)[:, t, None, None]
        hist.append(r)
        if U is None:
            g = sum(hist[-e:])
        else:
            g = sum(np.asarray(U)[:, t, j, None, None] * hist[-1 - j] for j in range(e))
        if beta is not None:
            Z = np.asarray(beta)[:, t, None, None] * Z + g
            S = np.asarray(decay)[:, t, None, None] * S - np.asarray(lr)[:, t, None, None] * Z
        else:
            S = np.asarray(decay)[:, t, None, None] * S - np.asarray(lr)[:, t, None, None] * g
    new_buf = np.stack(hist[-(e - 1):], axis=1) if e > 1 else None
    return y, np.clip(S, -100, 100), (Z if beta is not None else None), new_buf
