"""GPU: the long-context configuration (Titans, d = 128, bf16 q/k/v, fp32 state,
momentum, window 1) against the streaming float64 oracle at its full length.

The tensor-core path keeps chunk increments and chunk-start states as bf16
tiles; these tests show that the error does not grow with the sequence:
the forward over all 131072 tokens of one unit (rel-L2 of y per 16384-token
block, and of S_end / Z_end), and every input gradient over a 16384-token
prefix, all within the bf16 tolerance (rel-L2 2e-2). The oracle
(oracle/streaming_ref.py) runs token by token in float64 on the host.
"""
import pytest
import torch

from atlas_rnn_b200 import memory_recurrence
from atlas_rnn_b200.workloads import CONFIGS, make_inputs, shrink
from tests.helpers import TOL_BF16, rel_l2

pytestmark = pytest.mark.gpu

BLOCK = 16384


def _inputs(T, seed):
    w = shrink(CONFIGS[2], B=1, H=1, T=T)
    return w, make_inputs(w, seed=seed, device="cuda", state_scale=0.1)


def test_config2_forward_full_length(native_lib):
    from oracle import streaming_ref
    w, x = _inputs(CONFIGS[2].T, seed=21)
    with torch.no_grad():
        y, S_end, Z_end, _ = memory_recurrence(x["k"], x["q"], x["v"], x["lr"], x["decay"], x["beta"], None,
                                               S_ref=x["S0"], S0=x["S0"], Z0=x["Z0"])
    torch.cuda.synchronize()
    c = lambda t: t.cpu()
    yr, Sr, Zr, _, _ = streaming_ref.forward(c(x["k"]), c(x["q"]), c(x["v"]), c(x["lr"]), c(x["decay"]),
                                             c(x["beta"]), c(x["S0"]), c(x["S0"]), c(x["Z0"]))
    per_block = [rel_l2(y[:, i:i + BLOCK].float(), yr[:, i:i + BLOCK]) for i in range(0, w.T, BLOCK)]
    print("config-2 forward rel-L2 of y per 16k block:", ["%.2e" % e for e in per_block])
    assert max(per_block) < TOL_BF16, per_block
    # no drift: the last block is no worse than a small multiple of the first
    assert per_block[-1] < 4 * per_block[0] + 1e-3, per_block
    assert rel_l2(S_end, Sr) < TOL_BF16
    assert rel_l2(Z_end, Zr) < TOL_BF16


def test_config2_backward_prefix(native_lib):
    from oracle import streaming_ref
    T = 16384
    w, x = _inputs(T, seed=22)
    names = ("k", "q", "v", "lr", "decay", "beta", "S0", "Z0")
    leaves = {n: x[n].clone().requires_grad_(True) for n in names}
    y, S_end, Z_end, _ = memory_recurrence(leaves["k"], leaves["q"], leaves["v"], leaves["lr"], leaves["decay"],
                                           leaves["beta"], None, S_ref=leaves["S0"], S0=leaves["S0"],
                                           Z0=leaves["Z0"])
    g = torch.Generator().manual_seed(23)
    dS = torch.randn(S_end.shape, generator=g)
    dZ = torch.randn(S_end.shape, generator=g)
    torch.autograd.backward([y, S_end, Z_end], [x["dy"], dS.cuda(), dZ.cuda()])
    torch.cuda.synchronize()
    c = lambda t: t.detach().cpu()
    gr = streaming_ref.backward(c(x["k"]), c(x["q"]), c(x["v"]), c(x["lr"]), c(x["decay"]), c(x["beta"]),
                                c(x["S0"]), c(x["S0"]), c(x["Z0"]), c(x["dy"]), dS, dZ, seg=1024)
    gr["S0"] = gr["S0"] + gr["S_ref"]  # S_ref is the same tensor as S0 (rnn_memory.py:284)
    errs = {n: rel_l2(leaves[n].grad.float(), gr[n]) for n in names}
    print("config-2 backward (16k prefix) rel-L2:", {n: "%.2e" % e for n, e in errs.items()})
    bad = {n: e for n, e in errs.items() if not e < TOL_BF16}
    assert not bad, errs
