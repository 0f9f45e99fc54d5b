"""GPU: head preparation (atlas_head_prep_forward / _backward) against the torch chain it
replaces -- split_heads, MultiheadRMSNorm (rnn_memory.py:139-147), '(b h) n d' reshape,
cast, zero-pad -- forward, input gradient and gain gradient; and the cells under bf16
autocast with it on and off (ATLAS_MEM_HEADPREP). fp32 rel-L2 <= 1e-5, bf16 <= 2e-2."""
import pytest
import torch
import torch.nn.functional as F

import atlas_rnn_b200 as A
from atlas_rnn_b200.headprep import head_prep
from tests.helpers import TOL_BF16, TOL_F32, rel_l2

pytestmark = pytest.mark.gpu


def torch_prep(t, gamma, H, d_out, out_dtype):
    B, T, HD = t.shape
    d = HD // H
    x = t.view(B, T, H, d).transpose(1, 2)
    if gamma is not None:
        rms = x.norm(dim=-1, keepdim=True) * d ** -0.5
        x = x / rms.clamp(min=1e-8) * gamma
    return F.pad(x.reshape(B * H, T, d), (0, d_out - d)).to(out_dtype)


@pytest.mark.parametrize("d,norm,dtype", [(64, True, torch.float32), (32, True, torch.float32),
                                          (128, True, torch.float32), (96, False, torch.float32),
                                          (64, True, torch.bfloat16)])
def test_head_prep_matches_torch(native_lib, d, norm, dtype):
    g = torch.Generator(device="cuda").manual_seed(d)
    B, T, H = 2, 37, 3
    t = torch.randn(B, T, H * d, device="cuda", generator=g).to(dtype)
    t[0, 5] = 0.0  # rows whose norm clamps
    t = t.requires_grad_(True)
    gamma = (1 + 0.1 * torch.randn(H, 1, d, device="cuda", generator=g)).requires_grad_(True) if norm else None
    out = head_prep(t, gamma, H, 128, dtype)
    t2 = t.detach().clone().requires_grad_(True)
    g2 = gamma.detach().clone().requires_grad_(True) if norm else None
    ref = torch_prep(t2, g2, H, 128, dtype)
    tol = TOL_F32 if dtype == torch.float32 else TOL_BF16
    assert out.shape == ref.shape and rel_l2(out.float(), ref.float()) < tol
    assert torch.all(out[..., d:] == 0)
    up = torch.randn(out.shape, device="cuda", generator=g).to(dtype)
    out.backward(up)
    ref.backward(up)
    assert rel_l2(t.grad.float(), t2.grad.float()) < tol
    if norm:
        assert rel_l2(gamma.grad, g2.grad) < tol


@pytest.mark.parametrize("cls,kw", [
    ("OmegaRNNMemoryCell", dict(dim=128, dim_head=64, heads=2, omega_window=8, use_omega_gate=True,
                                poly_mode="elementwise", poly_degree=2)),
    ("RNNMemoryCell", dict(dim=256, dim_head=128, heads=2)),
    ("OmegaRNNMemoryCell", dict(dim=96, dim_head=32, heads=3, omega_window=4, use_omega_gate=False,
                                qkv_conv_kernel=None)),
])
def test_cell_with_head_prep_under_autocast(native_lib, monkeypatch, cls, kw):
    torch.manual_seed(0)
    cell = getattr(A, cls)(**kw).cuda()
    with torch.no_grad():
        for n, p in cell.named_parameters():
            if "gamma" in n:
                p.add_(0.1 * torch.randn_like(p))
    x = torch.randn(2, 300, kw["dim"], device="cuda")
    outs = {}
    for mode in ("1", "0"):
        monkeypatch.setenv("ATLAS_MEM_HEADPREP", mode)
        cell.zero_grad(set_to_none=True)
        xx = x.clone().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y, st = cell(xx)
        y.float().square().mean().backward()
        outs[mode] = (y.float(), st.S, xx.grad, {n: p.grad.float().clone() for n, p in cell.named_parameters()
                                                 if p.grad is not None})
    a, b = outs["1"], outs["0"]
    assert rel_l2(a[0], b[0]) < TOL_BF16 and rel_l2(a[1], b[1]) < TOL_BF16 and rel_l2(a[2], b[2]) < TOL_BF16
    assert a[3].keys() == b[3].keys()
    for n in a[3]:
        assert rel_l2(a[3][n], b[3][n]) < TOL_BF16, n
