"""Stand-in for ``assoc_scan.AssocScan`` (test infrastructure only).

The reference imports ``from assoc_scan import AssocScan`` (rnn_memory.py:34) and
calls it as ``AssocScan(use_accelerated=...)(gates, inputs, prev=...)``
(rnn_memory.py:189,363,369,379,480,698,700,705). The package is third-party,
unpinned (pyproject.toml:28) and not installed here, so this module restates the
published recurrence it computes:

    h_t = a_t * h_{t-1} + x_t,   h_0 = prev (or 0),   outputs h_1..h_T

with a scalar gate ``a`` of shape [N, T] broadcast over the trailing dims of
``x`` [N, T, ...]. With ``remove_prev=False`` and ``prev`` given, ``prev`` is
prepended (T+1 outputs), the form used at omega.py:315.

Algorithm: the scalar-gate specialisation of the odd/even recursive pair
reduction in ``atlas_pytorch/affine_scan.py:102-137`` (compose adjacent pairs,
recurse on the reduced sequence, fill the even positions, interleave). The
composition of (a1, x1) followed by (a2, x2) is (a1*a2, x1*a2 + x2), the scalar
case of ``_assoc_compose_affine`` (affine_scan.py:7-33).

Pinned by the reference's scan KATs (tests/test_rnn_all.py:832-887) and the
split-scan identity (tests/test_titans.py:680-707) in tests/test_oracle.py.
"""
from __future__ import annotations

import torch
from torch import Tensor


def _bcast(a: Tensor, like: Tensor) -> Tensor:
    return a.reshape(*a.shape, *([1] * (like.ndim - a.ndim)))


def _compose(left, right):
    a1, x1 = left
    a2, x2 = right
    return a1 * a2, x1 * _bcast(a2, x1) + x2


def _interleave(even: Tensor, odd: Tensor) -> Tensor:
    n_out = even.shape[1] + odd.shape[1]
    if even.shape[1] == odd.shape[1] + 1:
        odd = torch.cat([odd, torch.zeros_like(odd[:, :1])], dim=1)
    out = torch.stack([even, odd], dim=2).flatten(1, 2)
    return out[:, :n_out]


def _scan(a: Tensor, x: Tensor):
    t = a.shape[1]
    if t < 2:
        return a, x
    a_red, x_red = _compose((a[:, :-1:2], x[:, :-1:2]), (a[:, 1::2], x[:, 1::2]))
    a_odd, x_odd = _scan(a_red, x_red)
    if t % 2 == 0:
        left = (a_odd[:, :-1], x_odd[:, :-1])
    else:
        left = (a_odd, x_odd)
    a_even, x_even = _compose(left, (a[:, 2::2], x[:, 2::2]))
    a_even = torch.cat([a[:, :1], a_even], dim=1)
    x_even = torch.cat([x[:, :1], x_even], dim=1)
    return _interleave(a_even, a_odd), _interleave(x_even, x_odd)


def scalar_assoc_scan(gates: Tensor, inputs: Tensor, prev: Tensor | None = None,
                      remove_prev: bool = True) -> Tensor:
    """Log-depth scan of h_t = gates_t * h_{t-1} + inputs_t over dim 1."""
    a_pref, x_pref = _scan(gates, inputs)
    out = x_pref
    if prev is not None:
        out = out + prev.unsqueeze(1) * _bcast(a_pref, x_pref)
        if not remove_prev:
            out = torch.cat([prev.unsqueeze(1), out], dim=1)
    return out


def sequential_assoc_scan(gates: Tensor, inputs: Tensor, prev: Tensor | None = None,
                          remove_prev: bool = True) -> Tensor:
    """Plain sequential form of the same recurrence (used to cross-check)."""
    h = prev if prev is not None else torch.zeros_like(inputs[:, 0])
    outs = [] if remove_prev or prev is None else [prev]
    for t in range(inputs.shape[1]):
        h = _bcast(gates[:, t], h) * h + inputs[:, t]
        outs.append(h)
    return torch.stack(outs, dim=1)


class AssocScan(torch.nn.Module):
    """Drop-in for ``assoc_scan.AssocScan``; ``use_accelerated`` is accepted and ignored."""

    def __init__(self, use_accelerated: bool = False, sequential: bool = False):
        super().__init__()
        self.use_accelerated = use_accelerated
        self.sequential = sequential

    def forward(self, gates: Tensor, inputs: Tensor, prev: Tensor | None = None,
                remove_prev: bool | None = None) -> Tensor:
        if remove_prev is None:
            remove_prev = True
        fn = sequential_assoc_scan if self.sequential else scalar_assoc_scan
        return fn(gates, inputs, prev=prev, remove_prev=remove_prev)
