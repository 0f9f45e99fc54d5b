"""GPU: the scalar-gated scan drop-in (atlas_rnn_b200.AssocScan, kernels
atlas_scan_forward / atlas_scan_backward) against the CPU restatement of
assoc_scan.AssocScan (oracle/assoc_scan_standin.py, float64 autograd), with and
without prev, with remove_prev false (omega.py:315), over odd trailing sizes.
fp32 rel-L2 <= 1e-5, bf16 inputs <= 2e-2."""
import pytest
import torch

from atlas_rnn_b200 import AssocScan
from oracle.assoc_scan_standin import scalar_assoc_scan
from tests.helpers import TOL_BF16, TOL_F32, rel_l2

pytestmark = pytest.mark.gpu

CASES = [
    # (B, T, trailing, with prev, remove_prev, dtype)
    (2, 37, (4, 5), False, True, torch.float32),
    (3, 64, (33,), True, True, torch.float32),
    (2, 29, (16, 16), True, False, torch.float32),
    (1, 1, (7,), True, False, torch.float32),
    (4, 130, (300,), False, True, torch.float32),
    (2, 45, (8, 32), True, True, torch.bfloat16),
    (2, 64, (128,), True, False, torch.bfloat16),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"B{c[0]}_T{c[1]}_D{'x'.join(map(str, c[2]))}_"
                         f"{'prev' if c[3] else 'noprev'}_{'rm' if c[4] else 'keep'}_{str(c[5])[6:]}")
def test_scan_matches_standin(native_lib, case):
    B, T, trail, with_prev, remove_prev, dtype = case
    tol = TOL_F32 if dtype == torch.float32 else TOL_BF16
    g = torch.Generator().manual_seed(B * 1000 + T)
    gates = torch.sigmoid(torch.randn(B, T, generator=g) + 2.0)
    x = torch.randn(B, T, *trail, generator=g)
    prev = torch.randn(B, *trail, generator=g) if with_prev else None
    gd, xd = gates.cuda().requires_grad_(True), x.to(dtype).cuda().requires_grad_(True)
    pd = prev.cuda().requires_grad_(True) if with_prev else None
    out = AssocScan()(gd, xd, prev=pd, remove_prev=remove_prev)
    gr, xr = gates.double().requires_grad_(True), x.to(dtype).double().requires_grad_(True)
    pr = prev.double().requires_grad_(True) if with_prev else None
    ref = scalar_assoc_scan(gr, xr, prev=pr, remove_prev=remove_prev)
    assert out.shape == ref.shape, (out.shape, ref.shape)
    assert rel_l2(out.float(), ref) <= tol
    up = torch.randn(ref.shape, generator=g)
    out.backward(up.to(out.dtype).cuda())
    ref.backward(up.to(dtype).double())
    assert rel_l2(gd.grad, gr.grad) <= tol, rel_l2(gd.grad, gr.grad)
    assert rel_l2(xd.grad.float(), xr.grad) <= tol, rel_l2(xd.grad.float(), xr.grad)
    if with_prev:
        assert rel_l2(pd.grad, pr.grad) <= tol, rel_l2(pd.grad, pr.grad)
