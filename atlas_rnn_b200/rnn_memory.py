"""Drop-in module API of atlas_pytorch/rnn_memory.py on the B200 library.

Same class names, constructor arguments, sub-module names (so a reference
``state_dict`` loads unchanged), forward signatures and ``RNNMemState``
semantics as the reference. Projections, norms, depthwise convs and gate heads
stay ordinary torch modules; the recurrence core that the reference runs as
einsum + two ``AssocScan`` calls over materialised [BH,T,d,d] tensors
(rnn_memory.py:345-393, :655-717), or as its Omega-16 CUDA kernel
(rnn_memory.py:732-814), is one call to ``memory_recurrence``.

``use_accelerated_scan`` and ``use_cuda`` are accepted and ignored: there is a
single backend and no CPU path.
"""
from __future__ import annotations

import math
import os
from functools import partial
from typing import NamedTuple

import torch
import torch.nn.functional as F
from torch import Tensor, nn
from torch.nn import Conv1d, Linear, Module, Parameter

from .conv import qkv_depthwise_conv
from .headprep import HEAD_DIMS, head_prep
from .ops import TC_D, memory_recurrence


def exists(v):
    return v is not None


def default(v, d):
    return v if exists(v) else d


LinearNoBias = partial(Linear, bias=False)


class RNNMemState(NamedTuple):
    """Carried state (rnn_memory.py:68-73)."""
    seq_index: int
    S: Tensor
    Z: Tensor | None
    omega_buffer: Tensor | None


def state_detach(state: RNNMemState) -> RNNMemState:
    """Detach the carried tensors (rnn_memory.py:76-83)."""
    det = lambda t: t.detach() if exists(t) else None
    return RNNMemState(state.seq_index, det(state.S), det(state.Z), det(state.omega_buffer))


class PolynomialFeatureMap(Module):
    """Feature map modes off / elementwise / tensor (rnn_memory.py:90-132).

    Inside the cells the map is evaluated by the CUDA kernels; ``forward`` here
    is the plain torch form, kept for callers that use the module directly.
    """

    def __init__(self, dim: int, degree: int = 1, mode: str = "off"):
        super().__init__()
        self.dim, self.degree, self.mode = dim, degree, mode
        if mode == "tensor":
            feat = dim + dim * dim
            self.register_buffer("proj", torch.randn(feat, dim) / math.sqrt(feat))

    def forward(self, x: Tensor) -> Tensor:
        if self.degree <= 1 or self.mode == "off":
            return x
        if self.mode == "elementwise":
            acc, pw = x, x
            for _ in range(2, self.degree + 1):
                pw = pw * x
                acc = acc + pw
            return acc
        if self.mode == "tensor":
            outer = (x.unsqueeze(-1) * x.unsqueeze(-2)).flatten(-2)
            return torch.cat([x, outer], dim=-1) @ self.proj.to(x.device, x.dtype)
        return x


class MultiheadRMSNorm(Module):
    """Per-head RMS norm with a learned gain (rnn_memory.py:139-147)."""

    def __init__(self, dim: int, heads: int):
        super().__init__()
        self.scale = dim ** -0.5
        self.gamma = Parameter(torch.ones(heads, 1, dim))

    def forward(self, x: Tensor) -> Tensor:
        rms = x.norm(dim=-1, keepdim=True) * self.scale
        return (x / rms.clamp(min=1e-8)) * self.gamma


def _gate_head(dim: int, heads: int, bias: float) -> nn.Sequential:
    head = nn.Sequential(Linear(dim, heads), nn.Sigmoid())
    nn.init.zeros_(head[0].weight)
    nn.init.constant_(head[0].bias, bias)
    return head


class _MemoryCellBase(Module):
    """Shared body of RNNMemoryCell and OmegaRNNMemoryCell."""

    omega_window = 1
    use_omega_gate = False

    def _build(self, dim, dim_head, heads, use_momentum, poly_degree, poly_mode, qk_norm,
               qkv_conv_kernel, scan_chunk_len):
        self.dim, self.dim_head, self.heads = dim, dim_head, heads
        self.use_momentum = use_momentum
        self.qkv_conv_kernel = qkv_conv_kernel
        self.scan_chunk_len = scan_chunk_len
        inner = dim_head * heads
        self.activation = nn.Identity()
        self.to_q = LinearNoBias(dim, inner)
        self.to_k = LinearNoBias(dim, inner)
        self.to_v = LinearNoBias(dim, inner)
        self.to_out = LinearNoBias(inner, dim)
        if exists(qkv_conv_kernel) and qkv_conv_kernel > 1:
            conv = lambda: Conv1d(dim, dim, qkv_conv_kernel, padding=qkv_conv_kernel // 2, groups=dim, bias=False)
            self.q_conv, self.k_conv, self.v_conv = conv(), conv(), conv()
        else:
            self.q_conv = self.k_conv = self.v_conv = None
        # gate heads and their initial biases (rnn_memory.py:212-223, 503-520)
        self.to_lr = _gate_head(dim, heads, -4.0)
        self.to_decay = _gate_head(dim, heads, 4.0)
        self.to_momentum = _gate_head(dim, heads, 2.0) if use_momentum else None
        self.pre_norm = nn.RMSNorm(dim)
        self.q_norm = MultiheadRMSNorm(dim_head, heads) if qk_norm else nn.Identity()
        self.k_norm = MultiheadRMSNorm(dim_head, heads) if qk_norm else nn.Identity()
        self.phi = PolynomialFeatureMap(dim_head, poly_degree, poly_mode)
        self.register_buffer("_dummy", torch.zeros(1))

    def _head_prep_ok(self, proj_q: Tensor, seq_len: int) -> bool:
        """bf16 operands (bf16 inputs or bf16 autocast) on the tensor-core kernels: q, k, v go
        through head_prep (ATLAS_MEM_HEADPREP=0 turns it off)."""
        if not proj_q.is_cuda or seq_len < 2 or os.environ.get("ATLAS_MEM_HEADPREP", "1") == "0":
            return False
        bf16 = proj_q.dtype == torch.bfloat16 or (torch.is_autocast_enabled("cuda")
                                                   and torch.get_autocast_dtype("cuda") == torch.bfloat16)
        mode = self.phi.mode if self.phi.degree > 1 else "off"
        if not bf16 or mode == "tensor" or self.omega_window > 16 or self.dim_head not in HEAD_DIMS:
            return False
        if os.environ.get("ATLAS_MEM_TC", "1") == "0":
            return False
        return self.dim_head == TC_D or os.environ.get("ATLAS_MEM_PAD128", "1") != "0"

    # [b, n, (h d)] -> [b, h, n, d]
    def split_heads(self, t: Tensor) -> Tensor:
        b, n, hd = t.shape
        return t.view(b, n, self.heads, hd // self.heads).transpose(1, 2)

    def merge_heads(self, t: Tensor) -> Tensor:
        b, h, n, d = t.shape
        return t.transpose(1, 2).reshape(b, n, h * d)

    def init_state(self, batch: int, device=None, dtype=None) -> RNNMemState:
        device = default(device, self._dummy.device)
        dtype = default(dtype, self._dummy.dtype)
        S = torch.zeros(batch * self.heads, self.dim_head, self.dim_head, device=device, dtype=dtype)
        Z = torch.zeros_like(S) if self.use_momentum else None
        buf = None
        if self.omega_window > 1:
            buf = torch.zeros(batch * self.heads, self.omega_window - 1, self.dim_head, self.dim_head,
                              device=device, dtype=dtype)
        return RNNMemState(seq_index=0, S=S, Z=Z, omega_buffer=buf)

    def forward(self, x: Tensor, state: RNNMemState | None = None):
        batch, seq_len, _ = x.shape
        fresh = not exists(state)  # init_state's omega buffer is all zero: the kernels skip it
        if fresh:
            state = self.init_state(batch, x.device, x.dtype)
        x_act = self.activation(self.pre_norm(x))
        q_in = k_in = v_in = x_act
        if exists(self.q_conv) and self.qkv_conv_kernel <= 8:
            # the three depthwise convs in one GPU pass (first T outputs, as the reference keeps)
            q_in, k_in, v_in = qkv_depthwise_conv(x_act, self.q_conv.weight, self.k_conv.weight,
                                                  self.v_conv.weight)
        elif exists(self.q_conv):  # kernel sizes above 8: torch's Conv1d on the same device
            q_in = self.q_conv(q_in.transpose(1, 2)).transpose(1, 2)
            k_in = self.k_conv(k_in.transpose(1, 2)).transpose(1, 2)
            v_in = self.v_conv(v_in.transpose(1, 2)).transpose(1, 2)
        tile = self.scan_chunk_len
        if exists(tile) and seq_len > tile:
            # tiles share the call-start reference state (rnn_memory.py:279-296)
            S_ref, cur, outs = state.S, state, []
            for lo in range(0, seq_len, tile):
                hi = min(seq_len, lo + tile)
                out, cur = self._forward_impl(x_act[:, lo:hi], q_in[:, lo:hi], k_in[:, lo:hi],
                                              v_in[:, lo:hi], cur, S_ref=S_ref, zero_buffer=fresh and lo == 0)
                outs.append(out)
            return torch.cat(outs, dim=1), cur
        return self._forward_impl(x_act, q_in, k_in, v_in, state, S_ref=state.S, zero_buffer=fresh)

    def _forward_impl(self, x_act, q_in, k_in, v_in, state: RNNMemState, *, S_ref: Tensor,
                      zero_buffer: bool = False):
        batch, seq_len, _ = x_act.shape
        pq, pk, pv = self.to_q(q_in), self.to_k(k_in), self.to_v(v_in)
        bh = batch * self.heads
        flat = lambda t: t.reshape(bh, seq_len, t.shape[-1])
        padded_from = None
        if self._head_prep_ok(pq, seq_len):
            # split, per-head norm, cast and zero-pad to 128 columns in one pass per tensor
            cut = lambda t: t if t.shape[1] == seq_len else t[:, :seq_len].contiguous()
            gain = lambda norm: norm.gamma if isinstance(norm, MultiheadRMSNorm) else None
            d = self.dim_head
            k = head_prep(cut(pk), gain(self.k_norm), self.heads, TC_D, torch.bfloat16)
            q = head_prep(cut(pq), gain(self.q_norm), self.heads, TC_D, torch.bfloat16)
            v = head_prep(cut(pv), None, self.heads, TC_D, torch.bfloat16)
            padded_from, flat = (d, d), (lambda t: t)
        else:
            q = self.split_heads(pq)[:, :, :seq_len]
            k = self.split_heads(pk)[:, :, :seq_len]
            v = self.split_heads(pv)[:, :, :seq_len]
            q, k = self.q_norm(q), self.k_norm(k)
        heads_first = lambda g: g.transpose(1, 2).reshape(bh, seq_len)   # 'b n h -> (b h) n'
        # the gate heads (Linear(dim, heads) + sigmoid each) as one projection: x_act is read,
        # cast and back-propagated once instead of once per head
        heads = [self.to_lr, self.to_decay] + ([self.to_momentum] if self.use_momentum else []) + \
            ([self.to_omega_gate] if self.use_omega_gate else [])
        w = torch.cat([h[0].weight for h in heads])
        b = torch.cat([h[0].bias for h in heads])
        gates = F.linear(x_act, w, b).sigmoid().split(self.heads, dim=-1)
        lr, decay = heads_first(gates[0]), heads_first(gates[1])
        beta = heads_first(gates[2]) if self.use_momentum else None
        gate = heads_first(gates[-1]) if self.use_omega_gate else None
        e = self.omega_window
        # no buffer = zero history (the same result; the buffer kernels do not run)
        buf = state.omega_buffer if e > 1 and not zero_buffer else None
        y, S_end, Z_end, new_buf = memory_recurrence(
            flat(k), flat(q), flat(v), lr, decay, beta, gate, S_ref=S_ref, S0=state.S,
            Z0=state.Z if self.use_momentum else None, omega_buffer=buf, window=e,
            gate_mode="token", fmap_mode=self.phi.mode, fmap_degree=self.phi.degree,
            proj=getattr(self.phi, "proj", None), heads_padded_from=padded_from)
        if not (y.dtype == torch.bfloat16 and torch.is_autocast_enabled("cuda")
                and torch.get_autocast_dtype("cuda") == torch.bfloat16):
            y = y.to(x_act.dtype)  # (under bf16 autocast to_out takes bf16: the round trip is skipped)
        y = y.view(batch, self.heads, seq_len, -1)
        out = self.to_out(self.merge_heads(y))
        nxt = RNNMemState(seq_index=state.seq_index + seq_len, S=S_end, Z=Z_end,
                          omega_buffer=new_buf if e > 1 else None)
        return out, nxt


class RNNMemoryCell(_MemoryCellBase):
    """Titans-RNN cell (rnn_memory.py:154-408)."""

    def __init__(self, dim: int, dim_head: int = 64, heads: int = 1, use_momentum: bool = True,
                 poly_degree: int = 1, poly_mode: str = "off", qk_norm: bool = True,
                 qkv_conv_kernel: int | None = 4, use_accelerated_scan: bool = False,
                 scan_chunk_len: int | None = None):
        super().__init__()
        self._build(dim, dim_head, heads, use_momentum, poly_degree, poly_mode, qk_norm,
                    qkv_conv_kernel, scan_chunk_len)

    def init_state(self, batch: int, device=None, dtype=None) -> RNNMemState:
        st = super().init_state(batch, device, dtype)
        return st._replace(omega_buffer=None)


class OmegaRNNMemoryCell(_MemoryCellBase):
    """OmegaNet-RNN cell with the sliding window and omega gate (rnn_memory.py:415-814)."""

    def __init__(self, dim: int, dim_head: int = 64, heads: int = 1, omega_window: int = 1,
                 use_omega_gate: bool = True, use_momentum: bool = True, poly_degree: int = 1,
                 poly_mode: str = "off", qk_norm: bool = True, qkv_conv_kernel: int | None = 4,
                 use_accelerated_scan: bool = False, scan_chunk_len: int | None = None,
                 use_cuda: bool = False):
        super().__init__()
        self.omega_window = omega_window
        self.use_omega_gate = use_omega_gate
        self.use_cuda = use_cuda
        self._build(dim, dim_head, heads, use_momentum, poly_degree, poly_mode, qk_norm,
                    qkv_conv_kernel, scan_chunk_len)
        self.to_omega_gate = _gate_head(dim, heads, 0.0) if use_omega_gate else None


class RNNMemory(Module):
    """Wrapper choosing the cell (rnn_memory.py:821-881)."""

    def __init__(self, dim: int, dim_head: int | None = None, heads: int = 1, use_momentum: bool = True,
                 poly_degree: int = 1, poly_mode: str = "off", omega_window: int = 1,
                 use_omega_gate: bool = False, chunk_size: int = 1, use_accelerated_scan: bool = False,
                 scan_chunk_len: int | None = None, use_cuda: bool = False, **kwargs):
        super().__init__()
        dim_head = default(dim_head, dim)
        if omega_window > 1 or use_omega_gate:
            self.cell = OmegaRNNMemoryCell(dim=dim, dim_head=dim_head, heads=heads, omega_window=omega_window,
                                           use_omega_gate=use_omega_gate, use_momentum=use_momentum,
                                           poly_degree=poly_degree, poly_mode=poly_mode,
                                           use_accelerated_scan=use_accelerated_scan,
                                           scan_chunk_len=scan_chunk_len, use_cuda=use_cuda, **kwargs)
        else:
            self.cell = RNNMemoryCell(dim=dim, dim_head=dim_head, heads=heads, use_momentum=use_momentum,
                                      poly_degree=poly_degree, poly_mode=poly_mode,
                                      use_accelerated_scan=use_accelerated_scan, scan_chunk_len=scan_chunk_len,
                                      **kwargs)

    def forward(self, seq: Tensor, state: RNNMemState | None = None, **kwargs):
        return self.cell(seq, state)


OmegaRNNMemory = partial(RNNMemory, omega_window=4, use_omega_gate=True)
