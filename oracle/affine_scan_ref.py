"""Sequential float64 restatement of the reference's right-affine matrix scan.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): the checker of
atlas_rnn_b200.affine_associative_scan.

atlas_pytorch/affine_scan.py:36-160 computes H_t = H_{t-1} @ A_t + B_t by a
log-depth composition of the transforms (rule :7-33); this is the same
recurrence step by step, with the reference's output convention (prev first
when given and remove_prev is False; :153-158). Pinned against outputs and
autograd gradients of the reference function itself (tests/golden/affine_scan_*.npz,
made by tests/golden/make_affine_golden.py).
"""
from __future__ import annotations

import torch
from torch import Tensor


def affine_scan_sequential(A: Tensor, B: Tensor, prev: Tensor | None = None, remove_prev: bool = False) -> Tensor:
    N, T, D, _ = A.shape
    R = B.shape[2]
    H = prev if prev is not None else torch.zeros(N, R, D, dtype=A.dtype)
    outs = [prev] if (prev is not None and not remove_prev) else []
    for t in range(T):
        H = H @ A[:, t] + B[:, t]
        outs.append(H)
    return torch.stack(outs, dim=1)
