"""CPU: host side of the multi-GPU paths -- carry composition of sequence
parallelism (against the CPU oracle), the same over world_size-2 gloo ranks, and
failure detection of a rank that never joins (host-side, no GPU involved)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from atlas_rnn_b200.parallel import compose_backward_carries, compose_forward_carries, shard_units
from oracle import memory_ref

D = torch.float64


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _problem(seed=0, N=3, T=40, d=6):
    g = torch.Generator().manual_seed(seed)
    rn = lambda *s: torch.randn(*s, generator=g, dtype=D)
    sig = lambda mu, s: torch.sigmoid(mu + s * rn(N, T))
    return dict(k=rn(N, T, d), q=rn(N, T, d), v=rn(N, T, d), lr=0.1 * sig(0, 1), decay=sig(3, .5), beta=sig(1, .5),
                S_ref=0.3 * rn(N, d, d), S0=0.3 * rn(N, d, d), Z0=0.3 * rn(N, d, d))


def _segment_transform(p, lo, hi):
    """Forward transform of tokens [lo, hi) from a zero carry (CPU oracle)."""
    sl = lambda t: t[:, lo:hi]
    zero = torch.zeros_like(p["S0"])
    _, S_T, Z_T, _ = memory_ref.memory_core(sl(p["k"]), sl(p["q"]), sl(p["v"]), sl(p["lr"]), sl(p["decay"]),
                                            sl(p["beta"]), None, p["S_ref"], zero, zero, None)
    a, b, c = (torch.ones(p["S0"].shape[0], dtype=D), torch.zeros(p["S0"].shape[0], dtype=D),
               torch.ones(p["S0"].shape[0], dtype=D))
    for t in range(lo, hi):   # S -> alpha S - eta Z', Z' = beta Z  (rnn_memory.py:697-700)
        al, et, be = p["decay"][:, t], p["lr"][:, t], p["beta"][:, t]
        c = be * c
        b = al * b - et * c
        a = al * a
    # the oracle clamps S_T; keep values inside the clamp range
    return torch.stack([a, b, c], 1), S_T, Z_T


def test_shard_units_cover():
    for N, W in ((128, 8), (10, 3), (5, 8)):
        seen = []
        for r in range(W):
            s = shard_units(N, r, W)
            seen += list(range(N))[s]
        assert seen == list(range(N))


def test_forward_carries_match_full_run():
    p = _problem()
    T, P = 40, 4
    bounds = [(r * T // P, (r + 1) * T // P) for r in range(P)]
    segs = [_segment_transform(p, lo, hi) for lo, hi in bounds]
    carries, (S_T, Z_T) = compose_forward_carries([s[0] for s in segs], [s[1] for s in segs],
                                                  [s[2] for s in segs], p["S0"], p["Z0"])
    _, S_full, Z_full, _ = memory_ref.memory_core(p["k"], p["q"], p["v"], p["lr"], p["decay"], p["beta"], None,
                                                  p["S_ref"], p["S0"], p["Z0"], None)
    assert torch.allclose(S_T.clamp(-100, 100), S_full, atol=1e-10)
    assert torch.allclose(Z_T, Z_full, atol=1e-10)
    for r, (lo, _) in enumerate(bounds):
        if lo == 0:
            continue
        _, S_mid, Z_mid, _ = memory_ref.memory_core(*(p[n][:, :lo] for n in ("k", "q", "v", "lr", "decay", "beta")),
                                                    None, p["S_ref"], p["S0"], p["Z0"], None)
        assert torch.allclose(carries[r][0], S_mid, atol=1e-10)
        assert torch.allclose(carries[r][1], Z_mid, atol=1e-10)


def test_backward_carries_are_the_adjoint_of_forward_carries():
    """<adjoint, forward perturbation> identity: the composed backward transforms are
    the transposes of the composed forward ones."""
    g = torch.Generator().manual_seed(3)
    N, d, P = 2, 4, 3
    coefs = [torch.rand(N, 3, generator=g, dtype=D) for _ in range(P)]
    zeros = [torch.zeros(N, d, d, dtype=D) for _ in range(P)]
    S0, Z0 = torch.randn(N, d, d, generator=g, dtype=D), torch.randn(N, d, d, generator=g, dtype=D)
    FS, FZ = torch.randn(N, d, d, generator=g, dtype=D), torch.randn(N, d, d, generator=g, dtype=D)
    _, (ST, ZT) = compose_forward_carries(coefs, zeros, zeros, S0, Z0)
    _, (dS0, dZ0) = compose_backward_carries(coefs, zeros, zeros, FS, FZ)
    lhs = (FS * ST + FZ * ZT).sum()
    rhs = (dS0 * S0 + dZ0 * Z0).sum()
    assert torch.allclose(lhs, rhs, atol=1e-10)


def _gloo_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    p = _problem(seed=5)
    T = 40
    lo, hi = rank * T // world, (rank + 1) * T // world
    coef, dS, dZ = _segment_transform(p, lo, hi)
    gat = lambda t: (lambda out: (dist.all_gather(out, t), out)[1])([torch.empty_like(t) for _ in range(world)])
    carries, _ = compose_forward_carries(gat(coef), gat(dS), gat(dZ), p["S0"], p["Z0"])
    S_in, Z_in = carries[rank]
    if lo == 0:
        ok = torch.allclose(S_in, p["S0"]) and torch.allclose(Z_in, p["Z0"])
    else:
        _, S_mid, Z_mid, _ = memory_ref.memory_core(*(p[n][:, :lo] for n in ("k", "q", "v", "lr", "decay", "beta")),
                                                    None, p["S_ref"], p["S0"], p["Z0"], None)
        ok = torch.allclose(S_in, S_mid, atol=1e-10) and torch.allclose(Z_in, Z_mid, atol=1e-10)
    q.put((rank, bool(ok)))
    dist.destroy_process_group()


def test_gloo_two_ranks_carry_exchange():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_gloo_worker, args=(r, 2, port, q)) for r in range(2)]
    for pr in ps:
        pr.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for pr in ps:
        pr.join(timeout=60)
    assert res == {0: True, 1: True}


def _dead_peer_worker(rank, world, port, q):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)   # leaves between steps, before the exchange
    try:
        out = [torch.empty(4) for _ in range(world)]
        dist.all_gather(out, torch.ones(4))
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error: " + type(e).__name__))


def test_dead_rank_is_detected_by_collective_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_dead_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for pr in ps:
        pr.start()
    res = dict([q.get(timeout=120)])
    for pr in ps:
        pr.join(timeout=60)
        if pr.is_alive():
            pr.kill()
    assert ps[1].exitcode == 3
    assert res[0].startswith("error"), res[0]
