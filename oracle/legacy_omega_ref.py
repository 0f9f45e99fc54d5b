"""CPU restatement of the legacy OmegaNeuralMemory per-parameter update.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): the checker of
atlas_rnn_b200.omega_store, never the product path.

Follows atlas_pytorch/omega.py line by line for one parameter tensor (one momentum
order, no learned momentum combine, no spectral norm / Muon step):

  _sliding_sum_along_n                       omega.py:24-33
  momentum = assoc_scan(beta, surprise, prev=last_momentum)   omega.py:262-268
  next_last_momentum = momentum[:, -1]       omega.py:269
  gated = momentum * gate (broadcast)        omega.py:276-283
  ext = cat(prev_buf or zeros, gated); update = sliding_sum(ext, e)[:, -n:];
  next buffer = ext[:, -(e-1):]              omega.py:285-298
  all gates < 1e-3 -> update = zeros (not scanned), else
  update = assoc_scan(1 - decay, update, prev=last_update, remove_prev=False)   omega.py:306-315

The scans are the assoc_scan stand-in (assoc_scan_standin.py, pinned by the
reference's scan known-answer tests); the sliding sum is pinned by the
reference's own known answers (tests/test_atlas.py:147-169).
"""
from __future__ import annotations

import torch
from torch import Tensor

from .assoc_scan_standin import scalar_assoc_scan


def sliding_sum_along_n(x: Tensor, window: int) -> Tensor:
    """_sliding_sum_along_n (omega.py:24-33): sum of the last `window` entries along dim 1."""
    if window <= 1:
        return x
    n = x.shape[1]
    window = min(window, n)
    c = x.cumsum(dim=1)
    zeros = torch.zeros(*c.shape[:1], window, *c.shape[2:], dtype=c.dtype)
    shifted = torch.cat((zeros, c[:, :-window]), dim=1)
    return c - shifted


def omega_param_update(surprise: Tensor, decay_factor: Tensor, last_update: Tensor | None,
                       adaptive_momentum: Tensor | None = None, last_momentum: Tensor | None = None,
                       omega_gate: Tensor | None = None, prev_buf: Tensor | None = None, window: int = 1):
    """Returns (update, next_last_momentum or None, next buffer or None).

    surprise [(bh), n, ...]; decay_factor, adaptive_momentum, omega_gate [(bh), n]
    (any trailing singleton dims); last_update, last_momentum [(bh), ...];
    prev_buf [(bh), e-1, ...]."""
    B, n = surprise.shape[:2]
    base = surprise
    next_m = None
    if adaptive_momentum is not None:                                    # :262-268
        base = scalar_assoc_scan(adaptive_momentum.reshape(B, n), surprise, prev=last_momentum)
        next_m = base[:, -1]
    if omega_gate is not None:                                           # :276-283
        gate = omega_gate.reshape(B, n)
        while gate.ndim < base.ndim:
            gate = gate.unsqueeze(-1)
        gated = base * gate
    else:
        gated = base
    next_buf = None
    if window > 1:                                                       # :285-298
        if prev_buf is None:
            prev_buf = torch.zeros((B, window - 1, *gated.shape[2:]), dtype=gated.dtype)
        ext = torch.cat((prev_buf, gated), dim=1)
        update = sliding_sum_along_n(ext, window)[:, -n:]
        next_buf = ext[:, -(window - 1):]
    else:
        update = gated
    if omega_gate is not None and bool(torch.all(omega_gate.reshape(B, n).amax(dim=1) < 1e-3)):  # :306-309
        return torch.zeros_like(update), next_m, next_buf
    update = scalar_assoc_scan(1.0 - decay_factor.reshape(B, n), update, prev=last_update,   # :315
                               remove_prev=False)
    return update, next_m, next_buf
