"""GPU: the one-token decode step (atlas_mem_decode_step, used by memory_recurrence
for T = 1 without autograd) against the CPU oracle and against the general chunk
kernels, in every gate / feature-map mode it handles, and over a chain of steps
that carries S, Z and the omega buffer from call to call with S_ref = the
incoming state (how the reference cell is driven token by token in generate).

Tolerances: fp32 rel-L2 <= 1e-5, bf16 inputs (fp32 state) <= 2e-2."""
import pytest
import torch

from atlas_rnn_b200 import memory_recurrence
from atlas_rnn_b200.workloads import Workload, make_inputs
from tests.helpers import TOL_BF16, TOL_F32, oracle_run, rel_l2

pytestmark = pytest.mark.gpu


def W(name, d=32, dv=None, e=1, gate="none", fm="off", deg=1, mom=True, dtype=torch.float32, N=(2, 3), dphi=None):
    return Workload(name, N[0], N[1], 1, d, dphi or d, dv or d, e, gate, fm, deg, mom, dtype, 0)


CASES = [
    W("titans"),
    W("titans_nomom", mom=False),
    W("omega_e4_window", e=4, gate="window"),
    W("omega_e3_token_nomom", e=3, gate="token", mom=False),
    W("omega_e16_token", e=16, gate="token", d=64),
    W("elementwise_deg3", e=2, gate="token", fm="elementwise", deg=3),
    W("rect_dv48_dphi32", d=32, dv=48, e=3, gate="window"),
    W("head256", d=256, e=2, gate="token", N=(1, 2)),
    W("bf16_c1_like", d=128, e=4, gate="window", fm="elementwise", deg=2, dtype=torch.bfloat16, N=(2, 4)),
    W("bf16_titans", d=128, dtype=torch.bfloat16, N=(2, 4)),
]


def call(inp, w, S_ref=None, S0=None, Z0=None, buf=None):
    gm = "window" if w.gate == "window" else "token"
    return memory_recurrence(
        inp["k"], inp["q"], inp["v"], inp["lr"], inp["decay"], inp["beta"], inp["gate"],
        S_ref=S_ref if S_ref is not None else inp["S0"], S0=S0 if S0 is not None else inp["S0"],
        Z0=Z0 if Z0 is not None else inp["Z0"], omega_buffer=buf if buf is not None else inp["omega_buffer"],
        window=w.window, gate_mode=gm, fmap_mode=w.fmap_mode, fmap_degree=w.fmap_degree)


@pytest.mark.parametrize("w", CASES, ids=lambda w: w.name)
def test_decode_step_matches_oracle_and_general_path(native_lib, w):
    tol = TOL_F32 if w.dtype == torch.float32 else TOL_BF16
    inp = make_inputs(w, seed=3, device="cuda", state_scale=0.1)
    with torch.no_grad():
        out = call(inp, w)                       # decode kernel
    lead = inp["k"].clone().requires_grad_(True)  # a graph to record -> the general chunk kernels
    gen = call(dict(inp, k=lead), w)
    gm = "window" if w.gate == "window" else ("token" if w.gate == "token" else None)
    ref, _ = oracle_run(inp, w.window, gm, w.fmap_mode, w.fmap_degree, grads=False)
    for name, a, g in zip(("y", "S_end", "Z_end", "buf_out"), out, gen):
        if a is None:
            assert g is None and ref[name] is None, name
            continue
        assert rel_l2(a.float(), ref[name]) <= tol, (name, rel_l2(a.float(), ref[name]))
        assert rel_l2(a.float(), g.detach().float()) <= tol, (name, rel_l2(a.float(), g.detach().float()))


@pytest.mark.parametrize("w", [CASES[2], CASES[3], CASES[8]], ids=lambda w: w.name)
def test_decode_chain_carries_state(native_lib, w):
    """Five calls of one token each, state and buffer carried, S_ref = incoming state."""
    tol = TOL_F32 if w.dtype == torch.float32 else TOL_BF16
    steps = 5
    inps = [make_inputs(w, seed=10 + t, device="cuda", state_scale=0.1) for t in range(steps)]
    S, Z, buf = inps[0]["S0"], inps[0]["Z0"], inps[0]["omega_buffer"]
    Sr, Zr, bufr = S.cpu().double(), (Z.cpu().double() if Z is not None else None), \
        (buf.cpu().double() if buf is not None else None)
    gm = "window" if w.gate == "window" else ("token" if w.gate == "token" else None)
    for t in range(steps):
        with torch.no_grad():
            y, S, Z, buf = call(inps[t], w, S_ref=S, S0=S, Z0=Z, buf=buf)
        ref_in = dict(inps[t], S0=Sr, Z0=Zr, omega_buffer=bufr)
        ref, _ = oracle_run(ref_in, w.window, gm, w.fmap_mode, w.fmap_degree, grads=False, S_ref=Sr)
        assert rel_l2(y.float(), ref["y"]) <= tol, (t, "y", rel_l2(y.float(), ref["y"]))
        assert rel_l2(S, ref["S_end"]) <= tol, (t, "S", rel_l2(S, ref["S_end"]))
        Sr, Zr, bufr = ref["S_end"], ref["Z_end"], ref["buf_out"]


@pytest.mark.parametrize("w", [CASES[2], CASES[8]], ids=lambda w: w.name)
def test_decode_step_clamp_saturated(native_lib, w):
    """The clamp of S_end (rnn_memory.py:701) in the one-token kernel: |S0| of order 150 and alpha
    close to 1, so most of S_T lies beyond +-100; against the oracle and the general kernels."""
    tol = TOL_F32 if w.dtype == torch.float32 else TOL_BF16
    inp = make_inputs(w, seed=5, device="cuda", state_scale=0.1)
    inp["S0"] = (1500.0 * inp["S0"]).contiguous()
    inp["decay"] = torch.full_like(inp["decay"], 0.9995)
    g = torch.Generator().manual_seed(6)
    S_ref = (0.1 * torch.randn(inp["S0"].shape, generator=g)).cuda()
    with torch.no_grad():
        out = call(inp, w, S_ref=S_ref)
    gen = call(dict(inp, k=inp["k"].clone().requires_grad_(True)), w, S_ref=S_ref)
    gm = "window" if w.gate == "window" else ("token" if w.gate == "token" else None)
    ref, _ = oracle_run(inp, w.window, gm, w.fmap_mode, w.fmap_degree, grads=False, S_ref=S_ref)
    assert (out[1].abs() >= 100).float().mean() > 0.3
    for name, a, gg in zip(("y", "S_end", "Z_end", "buf_out"), out, gen):
        if a is None:
            continue
        assert rel_l2(a.float(), ref[name]) <= tol, name
        assert rel_l2(a.float(), gg.detach().float()) <= tol, name
