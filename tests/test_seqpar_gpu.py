"""GPU: sequence-parallel pieces (segment transform, carry composition, finish)
emulated as P consecutive segments in one process, against the full-sequence call."""
import pytest
import torch

from atlas_rnn_b200 import memory_recurrence
from atlas_rnn_b200.ops import Spec
from atlas_rnn_b200.parallel import (Segment, compose_backward_carries, compose_carries_device,
                                    compose_forward_carries)
from atlas_rnn_b200.workloads import CONFIGS, make_inputs, shrink
from tests.helpers import TOL_BF16, TOL_F32, rel_l2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,T,P,d,saturate", [(torch.float32, 200, 4, 32, False), (torch.float32, 97, 3, 16, False),
                                                  (torch.bfloat16, 8192, 4, 128, False),
                                                  (torch.float32, 200, 4, 32, True)])
def test_segments_match_full_call(native_lib, dtype, T, P, d, saturate):
    w = shrink(CONFIGS[2], B=1, H=2, T=T)
    from dataclasses import replace
    w = replace(w, d_k=d, d_phi=d, d_v=d, dtype=dtype)
    inp = make_inputs(w, seed=3, device="cuda", state_scale=0.1)
    if saturate:  # the clamp of S_end active: alpha close to 1, |S0| of order 150 (S_ref = S0)
        inp["S0"] = (1500.0 * inp["S0"]).contiguous()
        inp["decay"] = torch.full_like(inp["decay"], 0.9995)
    tol = TOL_F32 if dtype == torch.float32 else TOL_BF16
    names = ("k", "q", "v", "lr", "decay", "beta")
    # full call with autograd
    leaves = {n: inp[n].clone().requires_grad_(True) for n in names}
    Sr = inp["S0"].clone().requires_grad_(True)
    S0 = inp["S0"].clone().requires_grad_(True)
    Z0 = inp["Z0"].clone().requires_grad_(True)
    y, S_end, Z_end, _ = memory_recurrence(*(leaves[n] for n in names), S_ref=Sr, S0=S0, Z0=Z0)
    g = torch.Generator().manual_seed(9)
    dS_end = torch.randn(S_end.shape, generator=g).cuda()
    dZ_end = torch.randn(S_end.shape, generator=g).cuda()
    torch.autograd.backward([y, S_end, Z_end], [inp["dy"], dS_end, dZ_end])
    # segments
    spec = Spec(window=1, momentum=True)
    bounds = [(r * T // P, (r + 1) * T // P) for r in range(P)]
    segs = [Segment(spec, *(inp[n][:, lo:hi].contiguous() for n in names), inp["S0"]) for lo, hi in bounds]
    tr = [s.forward_local() for s in segs]
    carries, (S_T, Z_T) = compose_forward_carries([t[0] for t in tr], [t[1] for t in tr], [t[2] for t in tr],
                                                  inp["S0"], inp["Z0"])
    # the device composition over the packed records agrees with the torch one
    recs = torch.stack([s.record for s in segs])
    for r in range(P):
        iS, iZ, oS, oSc, oZ = compose_carries_device(segs[r], recs, r, False, inp["S0"], inp["Z0"], clamped=True)
        assert rel_l2(iS, carries[r][0]) < 1e-6 and rel_l2(iZ, carries[r][1]) < 1e-6, r
        assert rel_l2(oS, S_T) < 1e-6 and rel_l2(oZ, Z_T) < 1e-6 and torch.equal(oSc, oS.clamp(-100, 100))
    ys = [s.forward_finish(*c)[0] for s, c in zip(segs, carries)]
    assert rel_l2(torch.cat(ys, 1).float(), y.float()) < tol
    assert rel_l2(S_T.clamp(-100, 100), S_end) < tol
    if saturate:
        assert (S_T.abs() > 100).float().mean() > 0.1  # 17% of S_T beyond the clamp here
    assert rel_l2(Z_T, Z_end) < tol
    btr = [s.backward_local(inp["dy"][:, lo:hi].contiguous()) for s, (lo, hi) in zip(segs, bounds)]
    FS_end = dS_end * ((S_T >= -100) & (S_T <= 100))
    inc, (dS0, dZ0) = compose_backward_carries([t[0] for t in btr], [t[1] for t in btr], [t[2] for t in btr],
                                               FS_end, dZ_end)
    brecs = torch.stack([s.record for s in segs])
    for r in range(P):
        iS, iZ, oS, _, oZ = compose_carries_device(segs[r], brecs, r, True, dS_end, dZ_end, S_T=S_T)
        assert rel_l2(iS, inc[r][0]) < 1e-6 and rel_l2(iZ, inc[r][1]) < 1e-6, r
        assert rel_l2(oS, dS0) < 1e-6 and rel_l2(oZ, dZ0) < 1e-6
    grads = [s.backward_finish(inp["dy"][:, lo:hi].contiguous(), *c, apply_mask=False)
             for s, c, (lo, hi) in zip(segs, inc, bounds)]
    for n in names:
        got = torch.cat([gr[n] for gr in grads], 1)
        assert rel_l2(got.float(), leaves[n].grad.float()) < tol, n
    assert rel_l2(sum(gr["S_ref"] for gr in grads), Sr.grad) < tol
    assert rel_l2(dS0, S0.grad) < tol
    assert rel_l2(dZ0, Z0.grad) < tol
    # the first segment's own dS0 equals the composed one
    assert rel_l2(grads[0]["S0"], S0.grad) < tol


@pytest.mark.parametrize("H", [2, 40, 160])
def test_resident_segment_scans_match_generic(native_lib, monkeypatch, H):
    """The zero-carry segment transforms of the resident tensor-core scans (1, 2 and
    4 state groups per thread by the unit count) against the generic scans."""
    from dataclasses import replace
    w = replace(shrink(CONFIGS[2], B=1, H=H, T=1000), d_k=128, d_phi=128, d_v=128, dtype=torch.bfloat16)
    inp = make_inputs(w, seed=5, device="cuda", state_scale=0.1)
    names = ("k", "q", "v", "lr", "decay", "beta")
    out = {}
    for mode in ("resident", "generic"):
        if mode == "generic":
            monkeypatch.setenv("ATLAS_MEM_SCAN_GENERIC", "1")
        seg = Segment(Spec(window=1, momentum=True), *(inp[n] for n in names), inp["S0"])
        fwd = [t.clone() for t in seg.forward_local()]
        seg.forward_finish(inp["S0"], inp["Z0"])
        bwd = [t.clone() for t in seg.backward_local(inp["dy"])]
        out[mode] = fwd + bwd
    for a, b in zip(out["resident"], out["generic"]):
        assert rel_l2(a, b) < 1e-5, rel_l2(a, b)
