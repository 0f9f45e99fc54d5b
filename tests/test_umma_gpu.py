"""GPU: the tcgen05 GEMM building block (smem descriptors, instruction
descriptor, TMEM load path) against torch, for both operand major-nesses."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("a_mn", [0, 1])
@pytest.mark.parametrize("b_mn", [0, 1])
@pytest.mark.parametrize("N,K", [(128, 128), (64, 32), (256, 64), (80, 16)])
def test_umma_gemm(native_lib, a_mn, b_mn, N, K):
    from atlas_rnn_b200 import _lib
    g = torch.Generator(device="cpu").manual_seed(N * 7 + K)
    A = torch.randn(128, K, generator=g).bfloat16()
    B = torch.randn(N, K, generator=g).bfloat16()
    ref = A.float() @ B.float().T
    Ad = (A.T.contiguous() if a_mn else A).cuda()
    Bd = (B.T.contiguous() if b_mn else B).cuda()
    D = torch.full((128, N), float("nan"), device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = native_lib.atlas_mem_selftest_umma(_lib.ptr(Ad), _lib.ptr(Bd), _lib.ptr(D), N, K, a_mn, b_mn, _lib.ptr(st),
                                            None)
    torch.cuda.synchronize()
    assert rc == 0
    assert st.item() == 0
    err = ((D.cpu() - ref).norm() / ref.norm()).item()
    assert err < 1e-5, err
