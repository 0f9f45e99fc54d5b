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
    if name in ("k_fmap_fwd_tc", "k_fmap_bwd_tc"):
        # one launch maps one of k / q (the stand-alone feature map the d_phi > 128 path calls):
        # [x; vec(x x^T)] Proj, or its transpose product in the backward, per token
        return 2.0 * (w.d_k + w.d_k * w.d_k) * dp * w.T * w.N
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
        elif name == "k_bwd_state_gates_tc":
            fma = 2 * L * dp * dv + 2 * L * dv * dp + 4 * L * K * L
        elif name == "k_bwd_keys_tc":
            fma = (2 * K * dp * dv + 2 * K * dv * dp + 4 * dv * dp
                   + L * K * dv + L * K * dp + K * L * dv + K * L * dp + L * K * dp)
        elif name == "k_bwd_grads":
            fma = (L * K * dv + L * K * dp + L * 2 * dv * dp + 2 * K * dp * dv + 3 * (L + 2) * (K + 2) * L
                   + L * K * (L + 2) + K * L * dv + K * dp * (2 * dv + L) + L * dp * (2 * dv + K) + 4 * dv * dp)
        else:
            raise KeyError(name)
        total += 2.0 * fma
    return total * w.N


def kernel_bytes(name: str, w: Workload, C: int) -> float:
    """Compulsory HBM bytes of one launch of a tensor-core kernel (bf16 io,
    d_phi = d_v = 128): every operand it must read once and every result it must
    write, per chunk of L tokens with K = L + e - 1 keys, without re-reads and
    without padding rows. A row of a [*, 128] bf16 matrix is 256 B, a 128 x 128
    bf16 tile 32 KB; per-token gates are (3 + n_u) bf16 values (n_u = 1 or e)."""
    e = w.window
    row, tile = 2.0 * w.d_v, 2.0 * w.d_v * w.d_phi
    ng = 3 + (1 if w.gate == "token" else (e if w.gate == "window" else 0))
    total = 0.0
    if name == "k_bwd_finalize_tc":  # per 128-token tile
        for t0 in range(0, w.T, 128):
            TT = min(128, w.T - t0)
            # reads d delta, d phi (bf16 hand-off), d psi, q, k; writes dv, dq, dk
            total += 8 * TT * row + 2 * (e - 1) * 2 * row
        return total * w.N
    for t0 in range(0, w.T, C):
        L = min(C, w.T - t0)
        K = L + e - 1
        gates = 2.0 * ng * L
        if name == "k_fwd_chunk_tc":    # k, v rows in; delta rows, two increment tiles out
            b = 2 * K * row + L * row + 2 * tile
        elif name == "k_fwd_out_tc":    # q, k, delta rows and the two state tiles in; y out
            b = L * row + 2 * K * row + 2 * tile + L * row
        elif name == "k_bwd_chunk_tc":  # q, dy rows in; two adjoint increment tiles out
            b = 2 * L * row + 2 * tile
        elif name == "k_bwd_state_gates_tc":  # q, dy rows, state / adjoint tiles, d psi, G in; d psi, gate grads out
            b = 2 * L * row + 4 * tile + 2 * L * row + tile + 2 * 1024 + gates
        elif name == "k_bwd_keys_tc":   # k, delta, q, dy rows and adjoint tiles in; G, d delta, d phi, d psi out
            b = 2 * K * row + 2 * L * row + 2 * tile + tile + 2 * L * row + 4 * (e - 1) * row + L * row
        else:
            raise KeyError(name)
        total += b + gates
    return total * w.N
