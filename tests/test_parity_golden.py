"""GPU: the CUDA path against the reference's golden vectors (fp32, rel-L2 <= 1e-5)."""
import numpy as np
import pytest
import torch

from tests.helpers import TOL_F32, golden_files, load, rel_l2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("path", golden_files("core_"), ids=lambda p: p.split("/")[-1])
def test_core_golden(native_lib, path):
    from atlas_rnn_b200 import memory_recurrence
    z = load(path)
    B, H, T, d, e, gate_on, mom, deg = (int(x) for x in z["meta"])
    mode = str(z["fmap_mode"])
    dev = "cuda"
    t = lambda n: (torch.from_numpy(z[n]).float().to(dev).requires_grad_(True) if n in z else None)
    k, q, v, lr, decay = t("k"), t("q"), t("v"), t("lr"), t("decay")
    beta, gate, S0, Z0, buf = t("beta"), t("gate"), t("S0"), t("Z0"), t("buf")
    proj = torch.from_numpy(z["proj"]).float().to(dev) if "proj" in z else None
    y, S_end, Z_end, nb = memory_recurrence(k, q, v, lr, decay, beta, gate, S_ref=S0, S0=S0, Z0=Z0,
                                            omega_buffer=buf, window=e, gate_mode="token", fmap_mode=mode,
                                            fmap_degree=deg, proj=proj)
    outs = {"y": y, "S_end": S_end, "Z_end": Z_end, "buf_out": nb}
    for n, o in outs.items():
        if n in z:
            assert rel_l2(o, z[n]) < TOL_F32, (n, rel_l2(o, z[n]))
    pairs = [(outs[n], torch.from_numpy(z["up_" + n]).float().to(dev)) for n in outs if "up_" + n in z]
    torch.autograd.backward([p[0] for p in pairs], [p[1] for p in pairs])
    for n, leaf in (("k", k), ("q", q), ("v", v), ("lr", lr), ("decay", decay), ("beta", beta), ("gate", gate),
                    ("S0", S0), ("Z0", Z0), ("buf", buf)):
        if "d_" + n in z:
            err = rel_l2(leaf.grad, z["d_" + n])
            assert err < TOL_F32, (n, err)


@pytest.mark.parametrize("path", golden_files("module_"), ids=lambda p: p.split("/")[-1])
def test_module_golden(native_lib, path):
    """A whole reference cell (projections, conv, norms, gates) as a drop-in: same
    constructor, its state_dict loaded unchanged, same outputs, state and x.grad."""
    import atlas_rnn_b200 as A
    from tests.golden.make_golden import MODULE_CASES
    name = path.split("/")[-1][:-4]
    cls, kw, B, T, sk = MODULE_CASES[name]
    z = load(path)
    cell = getattr(A, cls)(**kw)
    sd = {k[3:]: torch.from_numpy(v).float() for k, v in z.items() if k.startswith("sd.")}
    cell.load_state_dict(sd)
    cell = cell.cuda()
    x = torch.from_numpy(z["x"]).float().cuda().requires_grad_(True)
    state = None
    if "S0" in z:
        g = lambda n: torch.from_numpy(z[n]).float().cuda() if n in z else None
        state = A.RNNMemState(seq_index=3, S=g("S0"), Z=g("Z0"), omega_buffer=g("buf"))
    y, st = cell(x, state)
    assert rel_l2(y, z["y"]) < TOL_F32
    assert rel_l2(st.S, z["S_end"]) < TOL_F32
    if "Z_end" in z:
        assert rel_l2(st.Z, z["Z_end"]) < TOL_F32
    else:
        assert st.Z is None
    if "buf_out" in z:
        assert rel_l2(st.omega_buffer, z["buf_out"]) < TOL_F32
    assert st.seq_index == int(z["seq_index"])
    y.backward(torch.from_numpy(z["up_y"]).float().cuda())
    assert rel_l2(x.grad, z["d_x"]) < TOL_F32
