"""GPU: the fused q/k/v depthwise convolutions (atlas_dwconv3_forward / _backward)
against torch's Conv1d(C, C, K, padding=K // 2, groups=C, bias=False) on x^T with the
first T outputs kept (the reference cells' convs, rnn_memory.py:196-202,334-340):
outputs, dx and the three weight gradients. fp32 at rel-L2 <= 1e-5; bf16 outputs
(bf16 autocast) at <= 2e-2."""
import pytest
import torch
import torch.nn.functional as F

from atlas_rnn_b200.conv import qkv_depthwise_conv
from tests.helpers import TOL_BF16, TOL_F32, rel_l2

pytestmark = pytest.mark.gpu


def torch_ref(x, ws):
    T = x.shape[1]
    return [F.conv1d(x.transpose(1, 2), w, padding=w.shape[-1] // 2, groups=x.shape[-1])[..., :T].transpose(1, 2)
            for w in ws]


@pytest.mark.parametrize("B,T,C,K", [(2, 300, 96, 4), (3, 17, 40, 3), (1, 2, 8, 4), (2, 513, 768, 4),
                                     (1, 70, 33, 2), (2, 129, 64, 5), (1, 90, 16, 8)])
def test_qkv_conv_fp32(native_lib, B, T, C, K):
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + T + K)
    x = torch.randn(B, T, C, device="cuda", generator=g).requires_grad_(True)
    ws = [(0.3 * torch.randn(C, 1, K, device="cuda", generator=g)).requires_grad_(True) for _ in range(3)]
    ys = qkv_depthwise_conv(x, *ws)
    x2 = x.detach().clone().requires_grad_(True)
    ws2 = [w.detach().clone().requires_grad_(True) for w in ws]
    refs = torch_ref(x2, ws2)
    for a, b in zip(ys, refs):
        assert a.dtype == torch.float32 and rel_l2(a, b) < TOL_F32
    ups = [torch.randn(B, T, C, device="cuda", generator=g) for _ in range(3)]
    torch.autograd.backward(list(ys), ups)
    torch.autograd.backward(refs, ups)
    assert rel_l2(x.grad, x2.grad) < TOL_F32
    for w, w2 in zip(ws, ws2):
        assert rel_l2(w.grad, w2.grad) < TOL_F32


def test_qkv_conv_under_bf16_autocast(native_lib):
    g = torch.Generator(device="cuda").manual_seed(3)
    B, T, C, K = 2, 1000, 256, 4
    x = torch.randn(B, T, C, device="cuda", generator=g).requires_grad_(True)
    ws = [(0.3 * torch.randn(C, 1, K, device="cuda", generator=g)).requires_grad_(True) for _ in range(3)]
    with torch.autocast("cuda", dtype=torch.bfloat16):
        ys = qkv_depthwise_conv(x, *ws)
        refs = torch_ref(x, ws)
    for a, b in zip(ys, refs):
        assert a.dtype == torch.bfloat16 and rel_l2(a.float(), b.float()) < TOL_BF16
    ups = [torch.randn(B, T, C, device="cuda", generator=g, dtype=torch.bfloat16) for _ in range(3)]
    gx = torch.autograd.grad(list(ys), [x] + ws, ups)
    gr = torch.autograd.grad(refs, [x] + ws, ups)
    for a, b in zip(gx, gr):
        assert a.dtype == b.dtype and rel_l2(a.float(), b.float()) < TOL_BF16
