"""GPU: the legacy OmegaNeuralMemory per-parameter update (omega.py:262-315) as one
fused kernel (atlas_rnn_b200.omega_store_update) against the CPU restatement
(oracle/legacy_omega_ref.py, float64 autograd): updates, next momentum, next
buffer and the gradients of every input, fp32 at rel-L2 1e-5, bf16 at 2e-2."""
import pytest
import torch

from tests.helpers import TOL_BF16, TOL_F32, rel_l2

pytestmark = pytest.mark.gpu


def _case(B, n, shape, e, mom, gate, buf, prev, dtype=torch.float32, seed=0, tiny_gate=False):
    from atlas_rnn_b200 import omega_store_update
    from oracle.legacy_omega_ref import omega_param_update
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g)
    x = {"s": r(B, n, *shape), "decay": torch.rand(B, n, 1, generator=g) * 0.5}
    if mom:
        x["beta"], x["m0"] = torch.rand(B, n, generator=g), r(B, *shape)
    if gate:
        x["gate"] = torch.rand(B, n, 1, generator=g) * (1e-4 if tiny_gate else 1.0)
    if buf and e > 1:
        x["buf"] = r(B, e - 1, *shape)
    if prev:
        x["h0"] = r(B, *shape)
    dev = {k: (v.to(dtype) if k == "s" else v).cuda().requires_grad_(True) for k, v in x.items()}
    cpu = {k: (v.to(dtype) if k == "s" else v).double().requires_grad_(True) for k, v in x.items()}

    def run(t, fn, **kw):
        return fn(t["s"], t["decay"], t.get("h0"), adaptive_momentum=t.get("beta"), last_momentum=t.get("m0"),
                  omega_gate=t.get("gate"), prev_buf=t.get("buf"), window=e, **kw)

    mine = run(dev, omega_store_update)
    ref = omega_param_update(cpu["s"], cpu["decay"], cpu.get("h0"), cpu.get("beta"), cpu.get("m0"),
                             cpu.get("gate"), cpu.get("buf"), window=e)
    tol = TOL_F32 if dtype == torch.float32 else TOL_BF16
    ups = [torch.randn(o.shape, generator=g, dtype=torch.float64) if o is not None else None for o in ref]
    for a, b in zip(mine, ref):
        assert (a is None) == (b is None)
        if a is not None:
            assert a.shape == b.shape
            assert rel_l2(a.float(), b) < tol
    torch.autograd.backward([o for o in mine if o is not None and o.requires_grad],
                            [u.to(o.dtype).cuda() for o, u in zip(mine, ups) if o is not None and o.requires_grad])
    torch.autograd.backward([o for o in ref if o is not None and o.requires_grad],
                            [u for o, u in zip(ref, ups) if o is not None and o.requires_grad])
    for k in x:
        if cpu[k].grad is None:
            assert dev[k].grad is None or dev[k].grad.abs().max() == 0, k
            continue
        assert rel_l2(dev[k].grad.float(), cpu[k].grad) < tol, k


@pytest.mark.parametrize("e", [1, 2, 4, 16])
@pytest.mark.parametrize("mom", [True, False])
@pytest.mark.parametrize("gate", [True, False])
def test_omega_store_modes(native_lib, e, mom, gate):
    _case(3, 12, (8, 5), e, mom, gate, buf=True, prev=True)


def test_omega_store_no_prev_no_buffer(native_lib):
    _case(2, 7, (33,), 4, True, True, buf=False, prev=False)


def test_omega_store_shorter_than_window(native_lib):
    _case(2, 2, (16, 3), 6, True, True, buf=True, prev=True)  # n < e - 1: old buffer entries carry on


def test_omega_store_large_params_bf16(native_lib):
    _case(4, 16, (64, 64), 3, True, True, buf=True, prev=True, dtype=torch.bfloat16)


def test_omega_store_all_gates_small(native_lib):
    """omega.py:306-309: every gate below 1e-3 -> zero update (momentum and buffer still carried)."""
    _case(2, 5, (4, 4), 3, True, True, buf=True, prev=True, tiny_gate=True)
