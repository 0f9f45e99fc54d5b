"""Module-substitution harness around the reference's own cells (test infrastructure only).

Loads the reference ``atlas_pytorch/rnn_memory.py`` straight from its source file
(the package ``__init__`` pulls in dependencies this image lacks), with the
``assoc_scan`` stand-in registered under the missing package's name, then builds
an ``OmegaRNNMemoryCell`` / ``RNNMemoryCell`` whose projection, norm, conv and
gate sub-modules are replaced so that the cell's own ``_forward_impl``
(rnn_memory.py:300-408 / :605-730) runs at the q/k/v/gates boundary:

* ``to_q/to_k/to_v`` -> slices of x = cat[q, k, v] (rnn_memory.py:315-317,624-626)
* ``q_norm/k_norm``  -> Identity (qk_norm=False)
* ``to_lr/to_decay/to_momentum/to_omega_gate`` -> modules returning injected gates
* ``to_out``         -> Identity
* ``phi``            -> the reference's own PolynomialFeatureMap with a given proj

``load_reference_rnn_transformer`` loads the reference LM module on top of it.
Used only by ``tests/golden/make_golden.py`` where the reference sources exist;
the generated fixtures travel, the reference does not.
"""
from __future__ import annotations

import importlib.util
import sys
import types

import torch
from torch import nn

from . import assoc_scan_standin


def load_reference_rnn_memory(reference_root: str):
    """Import the reference rnn_memory.py by path with the assoc_scan stand-in."""
    if "assoc_scan" not in sys.modules:
        mod = types.ModuleType("assoc_scan")
        mod.AssocScan = assoc_scan_standin.AssocScan
        sys.modules["assoc_scan"] = mod
    path = f"{reference_root}/atlas_pytorch/rnn_memory.py"
    spec = importlib.util.spec_from_file_location("_reference_rnn_memory", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def load_reference_rnn_transformer(reference_root: str, rm):
    """Import the reference rnn_transformer.py by path on top of `rm` (the loaded
    rnn_memory module). Its attention dependencies (rotary_embedding_torch,
    x_transformers) are absent here; they are only used by the attention block types,
    so they are registered as empty placeholders for the import."""
    for name, attr in (("rotary_embedding_torch", "RotaryEmbedding"), ("x_transformers", None),
                       ("x_transformers.attend", "Attend")):
        if name not in sys.modules:
            mod = types.ModuleType(name)
            if attr:
                setattr(mod, attr, type(attr, (nn.Module,), {}))
            sys.modules[name] = mod
    if "atlas_pytorch" not in sys.modules:
        pkg = types.ModuleType("atlas_pytorch")
        pkg.__path__ = []
        sys.modules["atlas_pytorch"] = pkg
    sys.modules["atlas_pytorch.rnn_memory"] = rm
    path = f"{reference_root}/atlas_pytorch/rnn_transformer.py"
    spec = importlib.util.spec_from_file_location("_reference_rnn_transformer", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


class _Slice(nn.Module):
    def __init__(self, lo, hi):
        super().__init__()
        self.lo, self.hi = lo, hi

    def forward(self, x):
        return x[..., self.lo:self.hi]


class _Inject(nn.Module):
    """Returns a fixed [B, T, H] gate tensor whatever its input."""

    def __init__(self):
        super().__init__()
        self.value = None

    def forward(self, x):
        return self.value


def run_reference_cell(rm, *, q, k, v, lr, decay, beta, gate, S0, Z0, buf, window,
                       heads, fmap_mode="off", fmap_degree=1, proj=None, S_ref=None):
    """Run the reference cell's _forward_impl on per-head inputs.

    q, k: [B, H, T, d_k]; v: [B, H, T, d_v]; gates: [B, T, H] (reference layout before
    the '(b h) n' rearrange). Returns (y [B, H, T, d_v], next_state).
    """
    B, H, T, dk = q.shape
    dv = v.shape[-1]
    omega = window > 1 or gate is not None
    use_momentum = beta is not None
    if omega:
        cell = rm.OmegaRNNMemoryCell(dim=dk, dim_head=dk, heads=heads, omega_window=window,
                                     use_omega_gate=gate is not None, use_momentum=use_momentum,
                                     poly_degree=fmap_degree, poly_mode=fmap_mode, qk_norm=False,
                                     qkv_conv_kernel=None)
    else:
        cell = rm.RNNMemoryCell(dim=dk, dim_head=dk, heads=heads, use_momentum=use_momentum,
                                poly_degree=fmap_degree, poly_mode=fmap_mode, qk_norm=False,
                                qkv_conv_kernel=None)
    cell = cell.to(q.dtype)
    hd_k, hd_v = H * dk, H * dv
    # x = cat[q, k, v] with heads merged ('b h n d -> b n (h d)')
    merge = lambda t: t.permute(0, 2, 1, 3).reshape(B, T, -1)
    x = torch.cat([merge(q), merge(k), merge(v)], dim=-1)
    cell.to_q = _Slice(0, hd_k)
    cell.to_k = _Slice(hd_k, 2 * hd_k)
    cell.to_v = _Slice(2 * hd_k, 2 * hd_k + hd_v)
    cell.to_out = nn.Identity()
    # dim_head is used for split_heads of q/k; v is split with the same head count
    for name, val in (("to_lr", lr), ("to_decay", decay), ("to_momentum", beta),
                      ("to_omega_gate", gate)):
        if val is not None:
            inj = _Inject()
            inj.value = val
            setattr(cell, name, inj)
    if fmap_mode == "tensor" and proj is not None:
        cell.phi.proj = proj.to(q.dtype)
    state = rm.RNNMemState(seq_index=0, S=S0, Z=Z0, omega_buffer=buf)
    S_ref = S0 if S_ref is None else S_ref
    y, st = cell._forward_impl(x, x, x, x, state, S_ref=S_ref)
    y = y.reshape(B, T, H, dv).permute(0, 2, 1, 3)
    return y, st
