"""Streaming float64 restatement of the Titans-RNN recurrence for long sequences.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): a checker, never the product.

``memory_ref.memory_layer`` materialises [N, T, d_v, d_phi] state tensors, which
does not fit at the long-context configuration (T = 131072, d = 128). This module
restates the same recurrence token by token with O(d_v d_phi) state, for the case
the long-context configuration uses: window 1, no omega gate, feature map off,
with or without momentum (rnn_memory.py:345-393, the Titans cell):

    delta_t = S_ref k_t - v_t                       rnn_memory.py:347-348
    Z_t = beta_t Z_{t-1} + delta_t k_t^T            rnn_memory.py:361-370 (momentum)
    S_t = alpha_t S_{t-1} - eta_t Z_t               rnn_memory.py:371-382
          (without momentum: S_t = alpha_t S_{t-1} - eta_t delta_t k_t^T)
    y_t = S_{t-1} q_t                               rnn_memory.py:388-393
    S_end = clamp(S_T, -100, 100), Z_end = Z_T      rnn_memory.py:372-373

``backward`` is the hand-derived reverse recurrence of the same steps (the
adjoint of each line, applied from t = T down to 1, with the states recomputed
per segment from checkpoints taken every ``seg`` tokens). It is pinned against
autograd of ``memory_ref.memory_layer`` on short sequences in tests/test_oracle.py.
"""
from __future__ import annotations

import torch


def _f64(t):
    return None if t is None else t.detach().to("cpu", torch.float64)


def forward(k, q, v, lr, decay, beta, S_ref, S0, Z0=None, checkpoint_every: int = 0):
    """Returns (y [N,T,d_v], S_end (clamped), Z_end or None, S_T unclamped, checkpoints).

    checkpoints: {t: (S_t, Z_t)} for t = 0, c, 2c, ... when checkpoint_every = c > 0.
    """
    k, q, v, lr, decay, beta, S_ref, S0, Z0 = map(_f64, (k, q, v, lr, decay, beta, S_ref, S0, Z0))
    N, T, _ = k.shape
    mom = beta is not None
    delta = torch.einsum("nde,nte->ntd", S_ref, k) - v
    S = S0.clone()
    Z = Z0.clone() if Z0 is not None else torch.zeros_like(S)
    y = torch.empty(N, T, v.shape[-1], dtype=torch.float64)
    ck = {}
    for t in range(T):
        if checkpoint_every and t % checkpoint_every == 0:
            ck[t] = (S.clone(), Z.clone())
        y[:, t] = torch.bmm(S, q[:, t, :, None])[..., 0]
        g = delta[:, t, :, None] * k[:, t, None, :]
        if mom:
            Z = beta[:, t, None, None] * Z + g
            S = decay[:, t, None, None] * S - lr[:, t, None, None] * Z
        else:
            S = decay[:, t, None, None] * S - lr[:, t, None, None] * g
    return y, S.clamp(-100, 100), (Z if mom else None), S, ck


def backward(k, q, v, lr, decay, beta, S_ref, S0, Z0, dy, dS_end=None, dZ_end=None, seg: int = 1024):
    """Gradients {k, q, v, lr, decay, beta, S_ref, S0, Z0} of
    <y, dy> + <S_end, dS_end> + <Z_end, dZ_end>, S_ref and S0 taken as separate inputs."""
    k, q, v, lr, decay, beta, S_ref, S0, Z0, dy, dS_end, dZ_end = map(
        _f64, (k, q, v, lr, decay, beta, S_ref, S0, Z0, dy, dS_end, dZ_end))
    N, T, _ = k.shape
    mom = beta is not None
    if Z0 is None:
        Z0 = torch.zeros_like(S0)
    _, _, _, S_T, ck = forward(k, q, v, lr, decay, beta, S_ref, S0, Z0, checkpoint_every=seg)
    delta = torch.einsum("nde,nte->ntd", S_ref, k) - v

    # clamp(S_T): gradient passes where -100 <= S_T <= 100 (torch.clamp's rule)
    Sh = torch.zeros_like(S0) if dS_end is None else dS_end * ((S_T >= -100) & (S_T <= 100))
    Zh = torch.zeros_like(S0) if (dZ_end is None or not mom) else dZ_end.clone()
    d_k = torch.zeros_like(k)
    d_q = torch.zeros_like(q)
    d_delta = torch.zeros_like(delta)
    d_lr = torch.zeros_like(lr)
    d_decay = torch.zeros_like(decay)
    d_beta = torch.zeros_like(beta) if mom else None

    starts = sorted(ck)
    for s0 in reversed(starts):
        s1 = min(s0 + seg, T)
        # recompute S_{t}, Z_{t} for t = s0 .. s1 (index 0 = state before token s0)
        L = s1 - s0
        Ss = torch.empty(L + 1, *S0.shape, dtype=torch.float64)
        Zs = torch.empty_like(Ss)
        S, Z = ck[s0]
        Ss[0], Zs[0] = S, Z
        for i in range(L):
            t = s0 + i
            g = delta[:, t, :, None] * k[:, t, None, :]
            if mom:
                Z = beta[:, t, None, None] * Z + g
                S = decay[:, t, None, None] * S - lr[:, t, None, None] * Z
            else:
                S = decay[:, t, None, None] * S - lr[:, t, None, None] * g
            Ss[i + 1], Zs[i + 1] = S, Z
        for i in reversed(range(L)):
            t = s0 + i
            S_prev, S_t = Ss[i], Ss[i + 1]
            # S_t = alpha_t S_{t-1} - eta_t X_t  (X = Z_t with momentum, g_t without)
            X = Zs[i + 1] if mom else delta[:, t, :, None] * k[:, t, None, :]
            d_decay[:, t] = (Sh * S_prev).sum((1, 2))
            d_lr[:, t] = -(Sh * X).sum((1, 2))
            if mom:
                Zh = Zh - lr[:, t, None, None] * Sh
                d_beta[:, t] = (Zh * Zs[i]).sum((1, 2))
                G = Zh
            else:
                G = -lr[:, t, None, None] * Sh
            # g_t = delta_t k_t^T
            d_delta[:, t] = torch.bmm(G, k[:, t, :, None])[..., 0]
            d_k[:, t] = torch.bmm(G.transpose(1, 2), delta[:, t, :, None])[..., 0]
            # y_t = S_{t-1} q_t
            d_q[:, t] = torch.bmm(S_prev.transpose(1, 2), dy[:, t, :, None])[..., 0]
            Sh = decay[:, t, None, None] * Sh + dy[:, t, :, None] * q[:, t, None, :]
            if mom:
                Zh = beta[:, t, None, None] * Zh
            del S_t
    # delta_t = S_ref k_t - v_t
    d_v = -d_delta
    d_k = d_k + torch.einsum("nde,ntd->nte", S_ref, d_delta)
    d_Sref = torch.einsum("ntd,nte->nde", d_delta, k)
    out = {"k": d_k, "q": d_q, "v": d_v, "lr": d_lr, "decay": d_decay, "S_ref": d_Sref, "S0": Sh}
    if mom:
        out["beta"] = d_beta
        out["Z0"] = Zh
    return out
