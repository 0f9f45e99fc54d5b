"""Shared test utilities: golden loading, rel-L2, oracle invocation."""
import glob
import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# tolerances (rel-L2) stated for this path: fp32 1e-5, bf16 inputs with fp32 accumulate 2e-2
TOL_F32 = 1e-5
TOL_BF16 = 2e-2


def rel_l2(a, b):
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    den = b.norm()
    if den == 0:
        return (a - b).norm().item()
    return ((a - b).norm() / den).item()


def golden_files(prefix):
    return sorted(glob.glob(os.path.join(GOLDEN, prefix + "*.npz")))


def load(path):
    z = np.load(path, allow_pickle=False)
    return {k: z[k] for k in z.files}


def oracle_run(inp, window, gate_mode, fmap_mode, fmap_degree, dtype=torch.float64, grads=True, up=None,
               S_ref=None):
    """Run the CPU oracle with autograd. inp: dict of tensors in memory_recurrence layout."""
    from oracle import memory_ref
    c = lambda t: None if t is None else t.detach().to("cpu", dtype).clone().requires_grad_(grads)
    k, q, v, lr, decay = (c(inp[n]) for n in ("k", "q", "v", "lr", "decay"))
    beta, gate = c(inp.get("beta")), c(inp.get("gate"))
    S0, Z0, buf = c(inp["S0"]), c(inp.get("Z0")), c(inp.get("omega_buffer"))
    Sr = c(S_ref) if S_ref is not None else None
    proj = inp.get("proj")
    proj = None if proj is None else proj.detach().to("cpu", dtype)
    U = gate if gate_mode == "window" else None
    u = gate if gate_mode == "token" else None
    y, S_end, Z_end, nb = memory_ref.memory_layer(k, q, v, lr, decay, beta, u, Sr if Sr is not None else S0,
                                                  S0, Z0, buf, window=window, U=U, fmap_mode=fmap_mode,
                                                  fmap_degree=fmap_degree, proj=proj)
    out = {"y": y, "S_end": S_end, "Z_end": Z_end, "buf_out": nb}
    grads_out = {}
    if grads:
        ups = up if up is not None else {}
        pairs = [(out[n], ups[n]) for n in ups if out.get(n) is not None and ups[n] is not None]
        torch.autograd.backward([p[0] for p in pairs], [p[1].to(dtype) for p in pairs])
        for name, t in (("k", k), ("q", q), ("v", v), ("lr", lr), ("decay", decay), ("beta", beta),
                        ("gate", gate), ("S0", S0), ("Z0", Z0), ("omega_buffer", buf), ("S_ref", Sr)):
            if t is not None:
                grads_out[name] = t.grad
    return {n: (t.detach() if t is not None else None) for n, t in out.items()}, grads_out
