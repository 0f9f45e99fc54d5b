"""Algorithmic work of the memory layer and of its kernels.

Step level, per token-head (one token of one batch*head unit), following the
counting used for the benchmark configs:
  forward flops  F  = 2 d_v d_phi (1 + 2 ns) + 2 C (d_phi + d_v)   (ns = 2 with momentum, else 1)
                      + 4 (d_k + d_k^2) d_phi with the tensor feature map
  backward flops Fb = 2 F
  forward bytes  Bf = s_in (2 d_k + d_v) + s_in n_g + s_out d_v     (n_g = 3 gates + u (1) or U (e))
  backward bytes Bb = Bf + s_out d_v (dy) + s_in (2 d_k + d_v + n_g) (input gradients)
C is the reference config's chunk length.

Kernel level: the GEMM work each chunk kernel has to do in the chunked
decomposition, per chunk of L tokens with K = L + e - 1 keys (multiply-adds x 2).
"""
from __future__ import annotations

from .workloads import Workload


def step_flops_per_token(w: Workload) -> tuple[float, float]:
    ns = 2 if w.momentum else 1
    F = 2 * w.d_v * w.d_phi * (1 + 2 * ns) + 2 * w.chunk * (w.d_phi + w.d_v)
    if w.fmap_mode == "tensor":
        F += 4 * (w.d_k + w.d_k * w.d_k) * w.d_phi
    return float(F), float(2 * F)


def step_bytes_per_token(w: Workload) -> tuple[float, float]:
    s = 2 if w.dtype.itemsize == 2 else 4
    ng = 3 + (1 if w.gate == "token" else (w.window if w.gate == "window" else 0))
    Bf = s * (2 * w.d_k + w.d_v) + s * ng + s * w.d_v
    Bb = Bf + s * w.d_v + s * (2 * w.d_k + w.d_v + ng)
    return float(Bf), float(Bb)


def tc_chunk(w: Workload) -> int:
    """Tokens per chunk of the tensor-core path (keys = chunk + e - 1 fill 128 rows)."""
    return 128 - w.window


def kernel_flops(name: str, w: Workload, C: int) -> float:
    """Algorithmic flops of one launch of a chunk kernel over the whole workload:
    the contractions the chunked decomposition has to do (multiply-adds x 2),
    without the padding of the 128-row tensor-core tiles."""
    e, dv, dp = w.window, w.d_v, w.d_phi
    total = 0.0
    for t0 in range(0, w.T, C):
        L = min(C, w.T - t0)
        K = L + e - 1
        if name == "k_fwd_chunk":
            fma = K * dp * dv + 2 * dv * K * dp
        elif name == "k_fwd_out":
            fma = L * K * dp + L * dv * (K + 2 * dp)
        elif name == "k_bwd_chunk":
            fma = 2 * dv * L * dp
        elif name == "k_fwd_chunk_tc":
            fma = K * dp * dv + 2 * dv * K * dp
        elif name == "k_fwd_out_tc":
            fma = L * K * dp + 2 * L * dp * dv + L * K * dv
        elif name == "k_bwd_chunk_tc":
            fma = 2 * dv * L * dp
        elif name == "k_bwd_state_tc":
            fma = 2 * L * dp * dv + 2 * L * dv * dp
        elif name == "k_bwd_keys_tc":
            fma = (2 * K * dp * dv + 2 * K * dv * dp + 4 * dv * dp
                   + L * K * dv + L * K * dp + K * L * dv + K * L * dp + L * K * dp)
        elif name == "k_bwd_gates_tc":
            fma = 4 * L * K * L
        elif name == "k_bwd_grads":
            fma = (L * K * dv + L * K * dp + L * 2 * dv * dp + 2 * K * dp * dv + 3 * (L + 2) * (K + 2) * L
                   + L * K * (L + 2) + K * L * dv + K * dp * (2 * dv + L) + L * dp * (2 * dv + K) + 4 * dv * dp)
        else:
            raise KeyError(name)
        total += 2.0 * fma
    return total * w.N
