"""GPU: the right-affine matrix scan (atlas_rnn_b200.affine_associative_scan, the drop-in of the
reference's affine_scan.affine_associative_scan) against the reference function's own golden
outputs and gradients and against the float64 sequential restatement, fp32 at rel-L2 1e-5."""
import numpy as np
import pytest
import torch

from tests.helpers import TOL_F32, golden_files, load, rel_l2

pytestmark = pytest.mark.gpu


def _run(A, B, prev, remove_prev, W):
    from atlas_rnn_b200 import affine_associative_scan
    leaves = [t.float().cuda().requires_grad_(True) if t is not None else None for t in (A, B, prev)]
    out = affine_associative_scan(leaves[0], leaves[1], prev=leaves[2], remove_prev=remove_prev)
    (out * W.float().cuda()).sum().backward()
    return out, [t.grad if t is not None else None for t in leaves]


@pytest.mark.parametrize("path", golden_files("affine_scan_"), ids=lambda p: p.split("/")[-1])
def test_affine_scan_vs_reference_goldens(native_lib, path):
    z = load(path)
    prev = torch.tensor(z["prev"]) if "prev" in z else None
    out, (dA, dB, dp) = _run(torch.tensor(z["A"]), torch.tensor(z["B"]), prev, bool(z["remove_prev"]),
                             torch.tensor(z["W"]))
    assert rel_l2(out, z["out"]) < TOL_F32
    assert rel_l2(dA, z["dA"]) < TOL_F32 and rel_l2(dB, z["dB"]) < TOL_F32
    if prev is not None:
        assert rel_l2(dp, z["dprev"]) < TOL_F32


@pytest.mark.parametrize("prev_mode", ["kept", "removed", "none"])
def test_affine_scan_full_width(native_lib, prev_mode):
    """R = D = 128 (a 128 x 128 state), 24 steps, against the float64 sequential oracle."""
    from oracle.affine_scan_ref import affine_scan_sequential
    g = torch.Generator().manual_seed(7)
    N, T, R, D = 3, 24, 128, 128
    A = 0.95 * torch.eye(D, dtype=torch.float64) + 0.2 * torch.randn(N, T, D, D, generator=g, dtype=torch.float64) / D ** 0.5
    B = torch.randn(N, T, R, D, generator=g, dtype=torch.float64)
    prev = None if prev_mode == "none" else torch.randn(N, R, D, generator=g, dtype=torch.float64)
    rm = prev_mode == "removed"
    A, B = A.float().double(), B.float().double()
    prev = prev.float().double() if prev is not None else None
    leaves = [t.clone().requires_grad_(True) if t is not None else None for t in (A, B, prev)]
    ref = affine_scan_sequential(leaves[0], leaves[1], leaves[2], rm)
    W = torch.randn(ref.shape, generator=g, dtype=torch.float64)
    (ref * W).sum().backward()
    out, grads = _run(A, B, prev, rm, W)
    assert out.shape == ref.shape
    assert rel_l2(out, ref.detach()) < TOL_F32
    for mine, leaf in zip(grads, leaves):
        if leaf is not None:
            assert rel_l2(mine, leaf.grad) < TOL_F32
