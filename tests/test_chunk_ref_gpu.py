"""GPU: ref_mode='chunk' (the chunk-start state as the reference state) against the CPU
oracle called the same way -- once per ref_chunk tokens with S_ref = S0 = the clamped
state of the call before, Z and the omega buffer carried (the reference cell called per
chunk, tests/test_rnn_all.py:804-825) -- outputs and every input gradient.
fp32 at rel-L2 <= 1e-5, bf16 at <= 2e-2."""
import pytest
import torch

from atlas_rnn_b200 import memory_recurrence
from atlas_rnn_b200.workloads import Workload, make_inputs
from tests.helpers import TOL_BF16, TOL_F32, rel_l2

pytestmark = pytest.mark.gpu

NAMES = ("k", "q", "v", "lr", "decay", "beta", "gate", "S0", "Z0", "omega_buffer")


def W(name, T, d=32, e=1, gate="none", fm="off", deg=1, mom=True, dtype=torch.float32, N=(1, 3)):
    return Workload(name, N[0], N[1], T, d, d, d, e, gate, fm, deg, mom, dtype, 0)


CASES = [
    (W("titans_f32", 150), 40),
    (W("omega_e4_token_f32", 131, e=4, gate="token", fm="elementwise", deg=2), 33),
    (W("omega_e3_window_f32", 97, e=3, gate="window"), 50),
    (W("tc_bf16_e4_window", 300, d=128, e=4, gate="window", fm="elementwise", deg=2, dtype=torch.bfloat16), 64),
]


def oracle_chunked(inp, w, L, up):
    from oracle import memory_ref
    c = lambda t: None if t is None else t.detach().to("cpu", torch.float64).clone().requires_grad_(True)
    leaf = {n: c(inp.get(n)) for n in NAMES}
    gm = w.gate
    S, Z, buf, ys = leaf["S0"], leaf["Z0"], leaf["omega_buffer"], []
    cut = lambda t, lo, hi: None if t is None else t[:, lo:hi]
    for lo in range(0, w.T, L):
        hi = min(w.T, lo + L)
        g = cut(leaf["gate"], lo, hi)
        y, S, Z, buf = memory_ref.memory_layer(
            cut(leaf["k"], lo, hi), cut(leaf["q"], lo, hi), cut(leaf["v"], lo, hi), cut(leaf["lr"], lo, hi),
            cut(leaf["decay"], lo, hi), cut(leaf["beta"], lo, hi), g if gm == "token" else None, S, S, Z, buf,
            window=w.window, U=g if gm == "window" else None, fmap_mode=w.fmap_mode, fmap_degree=w.fmap_degree,
            proj=None)
        ys.append(y)
    out = {"y": torch.cat(ys, 1), "S_end": S, "Z_end": Z, "buf_out": buf}
    pairs = [(out[n], up[n].double()) for n in up if out.get(n) is not None and up[n] is not None]
    torch.autograd.backward([p[0] for p in pairs], [p[1] for p in pairs])
    return out, {n: t.grad for n, t in leaf.items() if t is not None}


@pytest.mark.parametrize("w,L", CASES, ids=lambda c: c.name if hasattr(c, "name") else str(c))
def test_chunk_ref_mode_matches_oracle(native_lib, w, L):
    tol = TOL_F32 if w.dtype == torch.float32 else TOL_BF16
    inp = make_inputs(w, seed=4, device="cuda", state_scale=0.1)
    leaves = {n: (inp[n].clone().requires_grad_(True) if inp.get(n) is not None else None) for n in NAMES}
    gm = "window" if w.gate == "window" else "token"
    y, S_end, Z_end, nb = memory_recurrence(
        *(leaves[n] for n in ("k", "q", "v", "lr", "decay", "beta", "gate")), S_ref=leaves["S0"], S0=leaves["S0"],
        Z0=leaves["Z0"], omega_buffer=leaves["omega_buffer"], window=w.window, gate_mode=gm,
        fmap_mode=w.fmap_mode, fmap_degree=w.fmap_degree, ref_mode="chunk", ref_chunk=L)
    gen = torch.Generator().manual_seed(8)
    up = {"y": inp["dy"].float().cpu(), "S_end": torch.randn(S_end.shape, generator=gen),
          "Z_end": torch.randn(S_end.shape, generator=gen) if Z_end is not None else None,
          "buf_out": torch.randn(nb.shape, generator=gen) if nb is not None else None}
    ref, gref = oracle_chunked(inp, w, L, up)
    mine = {"y": y, "S_end": S_end, "Z_end": Z_end, "buf_out": nb}
    errs = {n: rel_l2(o.float(), ref[n]) for n, o in mine.items() if o is not None}
    pairs = [(mine[n], up[n].to(mine[n].dtype).cuda()) for n in mine if mine[n] is not None]
    torch.autograd.backward([p[0] for p in pairs], [p[1] for p in pairs])
    for n, t in leaves.items():
        if t is not None and n in gref:
            errs["d_" + n] = rel_l2(t.grad.float(), gref[n])
    bad = {k: v for k, v in errs.items() if not v < tol}
    assert not bad, (bad, errs)


def test_chunk_ref_mode_one_chunk_equals_call_mode(native_lib):
    """ref_chunk >= T is a single call: identical to the default mode."""
    w = W("one", 90, e=3, gate="token")
    inp = make_inputs(w, seed=2, device="cuda", state_scale=0.1)
    args = [inp[n] for n in ("k", "q", "v", "lr", "decay", "beta", "gate")]
    kw = dict(S_ref=inp["S0"], S0=inp["S0"], Z0=inp["Z0"], omega_buffer=inp["omega_buffer"], window=3,
              gate_mode="token")
    a = memory_recurrence(*args, **kw)
    b = memory_recurrence(*args, **kw, ref_mode="chunk", ref_chunk=90)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
