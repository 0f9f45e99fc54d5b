"""Long-term memory language model (the reference's LMM path) over the GPU memory cells.

Mirrors ``atlas_pytorch/rnn_transformer.py`` for ``block_type='lmm'``:

* ``GEGLU`` / ``FeedForward``  -- rnn_transformer.py:65-76 (RMSNorm, Linear to 2x inner,
  silu-gated half, Linear back; inner = int(dim * mult * 2 / 3))
* ``LMMBlock``                 -- :665-716 (memory cell residual, then feed-forward residual)
* ``RNNMemoryTransformer``     -- :720-862 (embedding + LayerNorm, blocks, LayerNorm, logits,
  next-token cross-entropy with ``return_loss``), ``generate`` :864-904 with
  ``min_p_filter`` / ``gumbel_sample`` :42-58
* ``LongTermMemoryModel``      -- :912

Parameter names and module nesting are the reference's, so a reference state_dict loads
unchanged. The memory cells are this package's ``RNNMemoryCell`` / ``OmegaRNNMemoryCell``,
whose recurrence runs in the CUDA kernels (one decode-kernel launch per cell for the
one-token steps of ``generate``). The attention block types of the reference ('mag', 'mal',
'mac': sliding-window attention around the memory) are not part of this package.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor, cat, nn
from torch.nn import Module, ModuleList

from .rnn_memory import OmegaRNNMemoryCell, RNNMemoryCell, RNNMemState, exists


def log(t: Tensor, eps: float = 1e-20) -> Tensor:
    return torch.log(t.clamp(min=eps))


def gumbel_noise(t: Tensor) -> Tensor:
    noise = torch.rand_like(t)
    return -log(-log(noise))


def gumbel_sample(t: Tensor, temperature: float = 1.0) -> Tensor:
    """rnn_transformer.py:50-53: argmax of logits / temperature plus Gumbel noise."""
    if temperature > 0.0:
        t = t / temperature + gumbel_noise(t)
    return t.argmax(dim=-1, keepdim=True)


def min_p_filter(logits: Tensor, min_p: float = 0.1) -> Tensor:
    """rnn_transformer.py:55-59: drop tokens below min_p times the top probability."""
    probs = logits.softmax(dim=-1)
    limit = min_p * probs.amax(dim=-1, keepdim=True)
    return torch.where(probs < limit, float("-inf"), logits)


class GEGLU(Module):
    """Second half of the projection, through silu, gates the first half."""

    def forward(self, x: Tensor) -> Tensor:
        x, gate = x.chunk(2, dim=-1)
        return F.silu(gate) * x


def FeedForward(dim: int, mult: float = 4) -> nn.Sequential:
    inner = int(dim * mult * 2 / 3)
    return nn.Sequential(nn.RMSNorm(dim), nn.Linear(dim, inner * 2), GEGLU(), nn.Linear(inner, dim))


class LMMBlock(Module):
    """Pure memory block: x + memory(x), then x + ff(x)."""

    def __init__(self, dim: int, dim_head: int = 64, heads: int = 8, ff_mult: float = 4, omega_window: int = 1,
                 use_omega_gate: bool = False, use_momentum: bool = True, poly_degree: int = 1,
                 poly_mode: str = "off", qkv_conv_kernel: int | None = None):
        super().__init__()
        if omega_window > 1 or use_omega_gate:
            self.memory = OmegaRNNMemoryCell(dim=dim, dim_head=dim_head, heads=heads, omega_window=omega_window,
                                             use_omega_gate=use_omega_gate, use_momentum=use_momentum,
                                             poly_degree=poly_degree, poly_mode=poly_mode,
                                             qkv_conv_kernel=qkv_conv_kernel)
        else:
            self.memory = RNNMemoryCell(dim=dim, dim_head=dim_head, heads=heads, use_momentum=use_momentum,
                                        poly_degree=poly_degree, poly_mode=poly_mode,
                                        qkv_conv_kernel=qkv_conv_kernel)
        self.ff = FeedForward(dim, mult=ff_mult)

    def forward(self, x: Tensor, mem_state: RNNMemState | None = None):
        mem_out, new_state = self.memory(x, state=mem_state)
        x = x + mem_out
        x = x + self.ff(x)
        return x, new_state


class RNNMemoryTransformer(Module):
    """Token embedding, a stack of memory blocks, final norm and logits (rnn_transformer.py:720-862).

    Only ``block_type='lmm'`` is provided; the attention block types raise ``ValueError``.
    ``window_size``, ``num_persist_mem_tokens`` and the legacy arguments are accepted for
    signature compatibility and have no effect on the LMM blocks, as in the reference."""

    def __init__(self, num_tokens: int, dim: int, depth: int, block_type: str = "lmm", window_size: int = 64,
                 dim_head: int = 64, heads: int = 8, ff_mult: float = 4, num_persist_mem_tokens: int = 0,
                 omega_window: int = 1, use_omega_gate: bool = False, use_momentum: bool = True,
                 poly_degree: int = 1, poly_mode: str = "off", qkv_conv_kernel: int | None = 4,
                 mem_chunk_size: int = 1, use_accelerated_scan: bool = False):
        super().__init__()
        if block_type != "lmm":
            raise ValueError(f"block_type {block_type!r}: only the memory-only 'lmm' blocks are provided "
                             "(the attention blocks 'mag', 'mal', 'mac' are not part of this package)")
        self.num_tokens, self.dim, self.depth, self.block_type = num_tokens, dim, depth, block_type
        self.embed = nn.Embedding(num_tokens, dim)
        self.embed_norm = nn.LayerNorm(dim)
        kw = dict(dim=dim, dim_head=dim_head, heads=heads, ff_mult=ff_mult, omega_window=omega_window,
                  use_omega_gate=use_omega_gate, use_momentum=use_momentum, poly_degree=poly_degree,
                  poly_mode=poly_mode, qkv_conv_kernel=qkv_conv_kernel)
        self.layers = ModuleList([LMMBlock(**kw) for _ in range(depth)])
        self.norm = nn.LayerNorm(dim)
        self.to_logits = nn.Linear(dim, num_tokens, bias=False)
        nn.init.normal_(self.embed.weight, std=0.02)
        nn.init.normal_(self.to_logits.weight, std=0.02)

    def forward(self, x: Tensor, return_loss: bool = False, mem_states=None, attn_caches=None,
                return_cache: bool = False):
        if return_loss:
            x, labels = x[:, :-1], x[:, 1:]
        h = self.embed_norm(self.embed(x))
        mem_states = mem_states if exists(mem_states) else [None] * self.depth
        new_states = []
        for layer, st in zip(self.layers, mem_states):
            h, nst = layer(h, mem_state=st)
            new_states.append(nst)
        logits = self.to_logits(self.norm(h))
        caches = [None] * self.depth
        if return_loss:
            loss = F.cross_entropy(logits.view(-1, self.num_tokens), labels.reshape(-1))
            return (loss, logits, new_states, caches) if return_cache else loss
        return (logits, new_states, caches) if return_cache else logits

    @torch.no_grad()
    def generate(self, prompt: Tensor, max_length: int = 100, temperature: float = 1.0, min_p: float = 0.1,
                 use_cache: bool = True) -> Tensor:
        """Autoregressive sampling (rnn_transformer.py:864-904). With the cache each new
        token is one T = 1 call per layer, which runs the single-token decode kernel."""
        self.eval()
        full = prompt.clone()
        x, states = prompt, None
        for _ in range(max_length - prompt.shape[1]):
            if use_cache:
                logits, states, _ = self(x, mem_states=states, return_cache=True)
            else:
                logits = self(full)
            logits = min_p_filter(logits[:, -1:], min_p=min_p)
            nxt = gumbel_sample(logits, temperature=temperature).squeeze(-1)
            full = cat([full, nxt], dim=-1)
            x = nxt if use_cache else full
        return full


def MemoryAsGateTransformer(**kwargs):
    return RNNMemoryTransformer(block_type="mag", **kwargs)


def MemoryAsLayerTransformer(**kwargs):
    return RNNMemoryTransformer(block_type="mal", **kwargs)


def LongTermMemoryModel(**kwargs):
    return RNNMemoryTransformer(block_type="lmm", **kwargs)
