"""CPU: the oracle against the reference's golden vectors and known-answer tests."""
import numpy as np
import pytest
import torch

from oracle import memory_ref
from oracle.assoc_scan_standin import AssocScan, scalar_assoc_scan, sequential_assoc_scan
from tests.helpers import golden_files, load, oracle_run, rel_l2


# ---- scan KATs (tests/test_rnn_all.py:832-887 of the reference) ------------------
def test_scan_identity():
    x0 = torch.randn(2, 4, 4)
    out = AssocScan()(torch.ones(2, 5), torch.zeros(2, 5, 4, 4), prev=x0)
    for t in range(5):
        assert torch.allclose(out[:, t], x0, atol=1e-5)


def test_scan_additive():
    out = AssocScan()(torch.ones(1, 4), torch.ones(1, 4, 2, 2), prev=torch.zeros(1, 2, 2))
    for t in range(4):
        assert torch.allclose(out[:, t], torch.full((1, 2, 2), float(t + 1)))


def test_scan_decay():
    out = AssocScan()(torch.full((1, 4), 0.5), torch.zeros(1, 4, 2, 2), prev=torch.ones(1, 2, 2))
    for t in range(4):
        assert torch.allclose(out[:, t], torch.full((1, 2, 2), 0.5 ** (t + 1)), atol=1e-5)


def test_scan_mixed():
    out = AssocScan()(torch.full((1, 3), 0.5), torch.ones(1, 3, 2, 2), prev=torch.zeros(1, 2, 2))
    exp = torch.tensor([1.0, 1.5, 1.75]).view(1, 3, 1, 1).expand(1, 3, 2, 2)
    assert torch.allclose(out, exp, atol=1e-4)


def test_split_scan_identity():
    """scan(all)[-1] == scan(2nd half, prev=scan(1st half)[-1])  (tests/test_titans.py:680-707)."""
    g = torch.randn(2, 128, 16).sigmoid()
    x = torch.randn(2, 128, 16)
    full = scalar_assoc_scan(g, x)
    first = scalar_assoc_scan(g[:, :64], x[:, :64])
    second = scalar_assoc_scan(g[:, 64:], x[:, 64:], prev=first[:, -1])
    assert torch.allclose(full[:, -1], second[:, -1], atol=1e-5)


@pytest.mark.parametrize("T", [1, 2, 3, 7, 16, 33])
def test_logdepth_matches_sequential(T):
    g = torch.rand(3, T, dtype=torch.float64)
    x = torch.randn(3, T, 4, 5, dtype=torch.float64)
    p = torch.randn(3, 4, 5, dtype=torch.float64)
    for rp in (True, False):
        a = scalar_assoc_scan(g, x, prev=p, remove_prev=rp)
        b = sequential_assoc_scan(g, x, prev=p, remove_prev=rp)
        assert torch.allclose(a, b, atol=1e-12)


def test_window_kat():
    """Sliding sum [1..6], window 3 (tests/test_rnn_all.py:890-896)."""
    x = torch.arange(1, 7).float().view(1, 6, 1)
    exp = torch.tensor([1, 3, 6, 9, 12, 15], dtype=torch.float32).view(1, 6, 1)
    assert torch.allclose(memory_ref.sliding_sum_along_time(x, 3), exp)


# ---- oracle vs goldens produced by the reference module ----------------------------
@pytest.mark.parametrize("path", golden_files("core_"), ids=lambda p: p.split("/")[-1])
def test_oracle_matches_reference_golden(path):
    z = load(path)
    B, H, T, d, e, gate_on, mom, deg = (int(x) for x in z["meta"])
    mode = str(z["fmap_mode"])
    t = lambda n: torch.from_numpy(z[n]) if n in z else None
    inp = {"k": t("k"), "q": t("q"), "v": t("v"), "lr": t("lr"), "decay": t("decay"), "beta": t("beta"),
           "gate": t("gate"), "S0": t("S0"), "Z0": t("Z0"), "omega_buffer": t("buf"), "proj": t("proj")}
    up = {n: t("up_" + n) for n in ("y", "S_end", "Z_end", "buf_out")}
    out, gr = oracle_run(inp, e, "token" if gate_on else None, mode, deg, up=up)
    for n in ("y", "S_end", "Z_end", "buf_out"):
        if n in z:
            assert rel_l2(out[n], z[n]) < 1e-12, n
    # S_ref is S0 in the reference cell: its gradient is the sum of both paths
    names = {"k": "k", "q": "q", "v": "v", "lr": "lr", "decay": "decay", "beta": "beta", "gate": "gate",
             "Z0": "Z0", "omega_buffer": "buf"}
    for mine, theirs in names.items():
        if "d_" + theirs in z:
            assert rel_l2(gr[mine], z["d_" + theirs]) < 1e-10, mine
    assert rel_l2(gr["S0"], z["d_S0"]) < 1e-10


def test_window_gate_generalisation_reduces_to_token_gate():
    """U[t, j] = u_{t-j} reproduces the reference's per-token gate exactly."""
    torch.manual_seed(0)
    N, T, d, e = 2, 19, 6, 4
    D = torch.float64
    k, q, v = (torch.randn(N, T, d, dtype=D) for _ in range(3))
    lr, decay, beta, u = (torch.rand(N, T, dtype=D) for _ in range(4))
    S0, Z0 = torch.randn(N, d, d, dtype=D), torch.randn(N, d, d, dtype=D)
    # zero buffer: in token mode the buffer is stored gated, in window mode ungated
    U = torch.zeros(N, T, e, dtype=D)
    for j in range(e):
        U[:, j:, j] = u[:, : T - j]
    a = memory_ref.memory_layer(k, q, v, lr, decay, beta, u, S0, S0, Z0, None, window=e)
    b = memory_ref.memory_layer(k, q, v, lr, decay, beta, None, S0, S0, Z0, None, window=e, U=U)
    for x, y in zip(a[:3], b[:3]):
        assert torch.allclose(x, y, atol=1e-12)


@pytest.mark.parametrize("e,mom,gate", [(1, True, False), (3, True, True), (4, False, True)])
def test_sequential_numpy_restatement_agrees(e, mom, gate):
    torch.manual_seed(1)
    N, T, d = 2, 11, 5
    D = torch.float64
    k, q, v = (torch.randn(N, T, d, dtype=D) for _ in range(3))
    lr, decay = torch.rand(N, T, dtype=D), torch.rand(N, T, dtype=D)
    beta = torch.rand(N, T, dtype=D) if mom else None
    u = torch.rand(N, T, dtype=D) if gate else None
    S0 = torch.randn(N, d, d, dtype=D)
    Z0 = torch.randn(N, d, d, dtype=D) if mom else None
    buf = torch.randn(N, e - 1, d, d, dtype=D) if e > 1 else None
    a = memory_ref.memory_core(k, q, v, lr, decay, beta, u, S0, S0, Z0, buf, window=e)
    npf = lambda t: None if t is None else t.numpy()
    b = memory_ref.memory_core_sequential_np(*(npf(x) for x in (k, q, v, lr, decay, beta, u, S0, S0, Z0, buf)),
                                             window=e)
    for x, y in zip(a, b):
        if x is not None:
            assert np.allclose(x.numpy(), y, atol=1e-10)


# ---- streaming restatement for long sequences, pinned against the autograd oracle ---------
@pytest.mark.parametrize("mom", [True, False])
@pytest.mark.parametrize("saturate", [False, True])
def test_streaming_oracle_matches_autograd(mom, saturate):
    """oracle/streaming_ref.py (token-by-token forward, hand-derived reverse recurrence with
    checkpointed segments) equals autograd of memory_ref.memory_layer, including the
    clamp of S_end when |S_T| passes 100."""
    from oracle import streaming_ref
    g = torch.Generator().manual_seed(5)
    N, T, d = 2, 150, 16
    rn = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)
    unit = lambda t: t / t.norm(dim=-1, keepdim=True)
    k, q, v = unit(rn(N, T, d)), unit(rn(N, T, d)), unit(rn(N, T, d))
    decay = torch.sigmoid(3 + 0.5 * rn(N, T))
    if saturate:
        decay = 0.999 + 0.001 * torch.rand(N, T, generator=g, dtype=torch.float64)
    lr = 0.1 * torch.sigmoid(rn(N, T))
    beta = torch.sigmoid(1 + 0.5 * rn(N, T)) if mom else None
    scale = 150.0 if saturate else 0.1
    S_ref, S0 = 0.1 * rn(N, d, d), scale * rn(N, d, d)
    Z0 = 0.1 * rn(N, d, d) if mom else None
    dy, dS, dZ = rn(N, T, d), rn(N, d, d), rn(N, d, d)
    leaves = [t.clone().requires_grad_(True) if t is not None else None
              for t in (k, q, v, lr, decay, beta, S_ref, S0, Z0)]
    y, S_end, Z_end, _ = memory_ref.memory_layer(leaves[0], leaves[1], leaves[2], leaves[3], leaves[4],
                                                 leaves[5], None, leaves[6], leaves[7], leaves[8], None)
    outs, ups = [y, S_end], [dy, dS]
    if mom:
        outs.append(Z_end)
        ups.append(dZ)
    torch.autograd.backward(outs, ups)
    ys, Ss, Zs, S_T, _ = streaming_ref.forward(k, q, v, lr, decay, beta, S_ref, S0, Z0)
    if saturate:
        assert (S_T.abs() > 100).float().mean() > 0.2
    assert rel_l2(ys, y.detach()) < 1e-12 and rel_l2(Ss, S_end.detach()) < 1e-12
    gr = streaming_ref.backward(k, q, v, lr, decay, beta, S_ref, S0, Z0, dy, dS, dZ if mom else None, seg=32)
    names = ["k", "q", "v", "lr", "decay", "beta", "S_ref", "S0", "Z0"]
    for name, leaf in zip(names, leaves):
        if leaf is None:
            continue
        assert rel_l2(gr[name], leaf.grad) < 1e-10, name


# ---- legacy OmegaNeuralMemory window: the reference's known answers (tests/test_atlas.py:147-169) ----
def test_legacy_sliding_sum_known_answers():
    from oracle.legacy_omega_ref import sliding_sum_along_n
    x = torch.tensor([[[1., 2.], [3., 4.], [5., 6.], [7., 8.]],
                      [[2., 1.], [4., 3.], [6., 5.], [8., 7.]]])
    assert torch.equal(sliding_sum_along_n(x, 1), x)
    assert torch.equal(sliding_sum_along_n(x, 2), torch.tensor([[[1., 2.], [4., 6.], [8., 10.], [12., 14.]],
                                                                [[2., 1.], [6., 4.], [10., 8.], [14., 12.]]]))
    assert torch.equal(sliding_sum_along_n(x, 3), torch.tensor([[[1., 2.], [4., 6.], [9., 12.], [15., 18.]],
                                                                [[2., 1.], [6., 4.], [12., 9.], [18., 15.]]]))


def test_legacy_omega_update_matches_sequential():
    """The restated omega.py:262-315 chain against a token-by-token loop of the same recurrences."""
    from oracle.legacy_omega_ref import omega_param_update
    g = torch.Generator().manual_seed(3)
    B, n, e = 3, 9, 4
    s = torch.randn(B, n, 2, 3, generator=g, dtype=torch.float64)
    beta, gate, decay = (torch.rand(B, n, generator=g, dtype=torch.float64) for _ in range(3))
    m0, h0 = torch.randn(B, 2, 3, generator=g, dtype=torch.float64), torch.randn(B, 2, 3, generator=g,
                                                                                  dtype=torch.float64)
    buf = torch.randn(B, e - 1, 2, 3, generator=g, dtype=torch.float64)
    upd, m_last, nb = omega_param_update(s, decay, h0, beta, m0, gate, buf, window=e)
    m, h, hist, outs = m0.clone(), h0.clone(), [buf[:, i] for i in range(e - 1)], [h0]
    for t in range(n):
        m = beta[:, t, None, None] * m + s[:, t]
        hist.append(gate[:, t, None, None] * m)
        h = (1 - decay[:, t, None, None]) * h + sum(hist[-e:])
        outs.append(h)
    assert torch.allclose(upd, torch.stack(outs, 1)) and torch.allclose(m_last, m)
    assert torch.allclose(nb, torch.stack(hist[-(e - 1):], 1))


# ---- right-affine matrix scan: the sequential restatement against the reference function's goldens ----
@pytest.mark.parametrize("path", golden_files("affine_scan_"), ids=lambda p: p.split("/")[-1])
def test_affine_scan_oracle_matches_reference(path):
    from oracle.affine_scan_ref import affine_scan_sequential
    z = load(path)
    A = torch.tensor(z["A"]).requires_grad_(True)
    B = torch.tensor(z["B"]).requires_grad_(True)
    prev = torch.tensor(z["prev"]).requires_grad_(True) if "prev" in z else None
    out = affine_scan_sequential(A, B, prev, bool(z["remove_prev"]))
    assert rel_l2(out, z["out"]) < 1e-12
    (out * torch.tensor(z["W"])).sum().backward()
    assert rel_l2(A.grad, z["dA"]) < 1e-12 and rel_l2(B.grad, z["dB"]) < 1e-12
    if prev is not None:
        assert rel_l2(prev.grad, z["dprev"]) < 1e-12
