"""Seeded synthetic workloads of the benchmark configurations.

Config k follows the input recipe stated for it: q, k, v ~ N(0,1) per element,
L2-normalised over the head dim (cast to bf16 for the bf16 configs); gates per
token and unit alpha = sigmoid(N(3, .5)), eta = 0.1 sigmoid(N(0,1)),
beta = sigmoid(N(1, .5)), per-token omega gate u = sigmoid(N(0,1)) or window
gates U = softmax over the window of N(0,1) logits; S0 = Z0 = 0, empty omega
buffer; upstream gradient dy ~ N(0,1). The tensor-map projection is
N(0, 1/sqrt(d + d^2)) of shape [d + d^2, d_phi].
"""
from __future__ import annotations

import math
from dataclasses import dataclass, replace

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    B: int
    H: int
    T: int
    d_k: int
    d_phi: int
    d_v: int
    window: int
    gate: str          # 'none' | 'token' | 'window'
    fmap_mode: str
    fmap_degree: int
    momentum: bool
    dtype: torch.dtype
    chunk: int         # the reference config's chunk (a tiling; results do not depend on it)

    @property
    def N(self):
        return self.B * self.H


CONFIGS = {
    0: Workload("titans_rnn_c0", 2, 4, 256, 64, 64, 64, 1, "none", "off", 1, True, torch.float32, 64),
    1: Workload("omega_rnn_c1", 8, 16, 4096, 128, 128, 128, 4, "window", "elementwise", 2, True,
                torch.bfloat16, 64),
    2: Workload("titans_rnn_longctx_c2", 1, 32, 131072, 128, 128, 128, 1, "none", "off", 1, True,
                torch.bfloat16, 128),
    4: Workload("omega_rnn_tensor_c4", 4, 8, 16384, 64, 256, 128, 16, "token", "tensor", 2, True,
                torch.bfloat16, 64),
    # not a benchmark config: the one shape the reference's own CUDA kernels run (window 16, head 64,
    # bf16, per-token omega gate), for timing those kernels beside ours (bench.py --impl reference-cuda)
    5: Workload("omega16_d64_refkernel", 8, 16, 4096, 64, 64, 64, 16, "token", "off", 1, True,
                torch.bfloat16, 0),
}


def shrink(w: Workload, B: int | None = None, H: int | None = None, T: int | None = None) -> Workload:
    return replace(w, B=w.B if B is None else B, H=w.H if H is None else H, T=w.T if T is None else T)


def make_inputs(w: Workload, seed: int = 0, device="cpu", state_scale: float = 0.0):
    """Returns a dict of tensors for ``memory_recurrence`` (plus dy)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    N, T = w.N, w.T
    rn = lambda *s: torch.randn(*s, generator=g)
    sig = lambda mu, s: torch.sigmoid(mu + s * rn(N, T))
    unit = lambda t: t / t.norm(dim=-1, keepdim=True)
    out = {
        "k": unit(rn(N, T, w.d_k)),
        "q": unit(rn(N, T, w.d_k)),
        "v": unit(rn(N, T, w.d_v)),
        "decay": sig(3.0, 0.5),
        "lr": 0.1 * sig(0.0, 1.0),
    }
    out["beta"] = sig(1.0, 0.5) if w.momentum else None
    if w.gate == "token":
        out["gate"] = sig(0.0, 1.0)
    elif w.gate == "window":
        out["gate"] = torch.softmax(rn(N, T, w.window), dim=-1)
    else:
        out["gate"] = None
    D = (N, w.d_v, w.d_phi)
    out["S0"] = state_scale * rn(*D)
    out["Z0"] = state_scale * rn(*D) if w.momentum else None
    out["omega_buffer"] = state_scale * rn(N, w.window - 1, w.d_v, w.d_phi) if w.window > 1 else None
    if w.fmap_mode == "tensor":
        feat = w.d_k + w.d_k * w.d_k
        out["proj"] = rn(feat, w.d_phi) / math.sqrt(feat)
    else:
        out["proj"] = None
    out["dy"] = rn(N, T, w.d_v)
    io = ("k", "q", "v", "decay", "lr", "beta", "gate", "dy")
    for key, t in out.items():
        if t is None:
            continue
        t = t.to(w.dtype) if key in io else t.float()
        out[key] = t.to(device)
    return out
