"""GPU: the resident-wave chunk scans of the tensor-core path (tc_scan.cuh)
against the generic per-unit scans (ATLAS_MEM_SCAN_GENERIC=1) at a unit count
that needs 4 float4 slots per thread and two rounds, and at a small one (1 slot).
Both apply the same recurrence in fp32; the compiler may contract the
multiply-adds differently, so states agree to a few fp32 ulps and the bf16
outputs downstream to an occasional flipped rounding: rel-L2 <= 1e-4."""
import os

import pytest
import torch

from atlas_rnn_b200 import memory_recurrence
from atlas_rnn_b200.workloads import Workload, make_inputs

pytestmark = pytest.mark.gpu


def run(w, generic):
    if generic:
        os.environ["ATLAS_MEM_SCAN_GENERIC"] = "1"
    else:
        os.environ.pop("ATLAS_MEM_SCAN_GENERIC", None)
    try:
        inp = make_inputs(w, seed=5, device="cuda", state_scale=0.5)
        leaves = {n: (t.clone().requires_grad_(True) if t is not None else None) for n, t in inp.items()
                  if n not in ("dy", "proj")}
        y, S_end, Z_end, nb = memory_recurrence(
            leaves["k"], leaves["q"], leaves["v"], leaves["lr"], leaves["decay"], leaves["beta"], leaves["gate"],
            S_ref=leaves["S0"], S0=leaves["S0"], Z0=leaves["Z0"], omega_buffer=leaves["omega_buffer"],
            window=w.window, gate_mode="window", fmap_mode=w.fmap_mode, fmap_degree=w.fmap_degree)
        g = torch.Generator(device="cpu").manual_seed(9)
        torch.autograd.backward([y, S_end, Z_end], [inp["dy"], torch.randn(S_end.shape, generator=g).cuda(),
                                                    torch.randn(Z_end.shape, generator=g).cuda()])
        torch.cuda.synchronize()
        out = {"y": y, "S_end": S_end, "Z_end": Z_end}
        out.update({"d_" + n: t.grad for n, t in leaves.items() if t is not None and t.grad is not None})
        return {k: v.detach().float().cpu() for k, v in out.items()}
    finally:
        os.environ.pop("ATLAS_MEM_SCAN_GENERIC", None)


@pytest.mark.parametrize("B,H,T", [(10, 16, 300), (1, 2, 500)])
def test_resident_scan_matches_generic(B, H, T):
    w = Workload("scan", B, H, T, 128, 128, 128, 4, "window", "elementwise", 2, True, torch.bfloat16, 0)
    a, b = run(w, False), run(w, True)
    assert a.keys() == b.keys()
    for k in a:
        err = ((a[k] - b[k]).double().norm() / b[k].double().norm().clamp_min(1e-30)).item()
        assert err <= 1e-4, (k, err)
