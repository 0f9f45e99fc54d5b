"""Generate the golden fixtures in this folder from the reference implementation.

Runs the reference's own ``RNNMemoryCell`` / ``OmegaRNNMemoryCell`` (loaded from
the reference sources with the assoc_scan stand-in, see oracle/harness.py) in
float64 on seeded inputs, and stores inputs, outputs, upstream gradients and
every input gradient (the reference's own autograd) as .npz files.

    python tests/golden/make_golden.py --reference <path to atlas-rnn checkout>

Two kinds of fixture:
* ``core_*.npz``   -- the recurrence at the q/k/v/gates boundary (harness), N = B*H
* ``module_*.npz`` -- a whole reference cell (projections, convs, norms, gates) with
                      its state_dict, input x and outputs / x.grad.
* ``lm_*.npz``     -- the reference LMM language model (RNNMemoryTransformer,
                      block_type 'lmm'): state_dict, tokens, loss, logits, every
                      parameter gradient, and the logits of one-token cached steps.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import harness, memory_ref  # noqa: E402

DT = torch.float64

CORE_CASES = {
    # name: (B, H, T, d, e, gate, momentum, fmap_mode, degree, nonzero_state)
    "core_titans_t37": (2, 2, 37, 16, 1, False, True, "off", 1, True),
    "core_titans_nomom": (1, 2, 29, 8, 1, False, False, "off", 1, True),
    "core_omega_e4_elem": (2, 2, 41, 16, 4, True, True, "elementwise", 2, True),
    "core_omega_e3_tensor_nomom": (1, 2, 23, 8, 3, False, False, "tensor", 2, True),
    "core_omega_e16": (1, 2, 45, 16, 16, True, True, "off", 1, True),
    "core_omega_short_t2_e5": (1, 2, 2, 8, 5, True, True, "elementwise", 3, True),
    "core_titans_t1": (1, 2, 1, 8, 1, False, True, "off", 1, True),
    "core_omega_zero_state": (1, 2, 33, 16, 2, True, True, "off", 1, False),
}


def sg(mu, s, *shape, g):
    return torch.sigmoid(mu + s * torch.randn(*shape, generator=g, dtype=DT))


def make_core(rm, name, B, H, T, d, e, gate_on, mom, mode, deg, nonzero, seed):
    g = torch.Generator().manual_seed(seed)
    N = B * H
    q = torch.randn(B, H, T, d, generator=g, dtype=DT)
    k = torch.randn(B, H, T, d, generator=g, dtype=DT)
    v = torch.randn(B, H, T, d, generator=g, dtype=DT)
    q = q / q.norm(dim=-1, keepdim=True)
    k = k / k.norm(dim=-1, keepdim=True)
    v = v / v.norm(dim=-1, keepdim=True)
    # gate distributions of the benchmark configs (alpha, eta, beta, u), reference layout [B, T, H]
    lr = 0.1 * sg(0, 1, B, T, H, g=g)
    decay = sg(3, 0.5, B, T, H, g=g)
    beta = sg(1, 0.5, B, T, H, g=g) if mom else None
    gate = sg(0, 1, B, T, H, g=g) if gate_on else None
    scale = 0.1 if nonzero else 0.0
    S0 = (scale * torch.randn(N, d, d, generator=g, dtype=DT)).clamp(-10, 10)
    Z0 = scale * torch.randn(N, d, d, generator=g, dtype=DT) if mom else None
    buf = scale * torch.randn(N, e - 1, d, d, generator=g, dtype=DT) if e > 1 else None
    proj = memory_ref.make_tensor_proj(d, generator=g, dtype=DT) if mode == "tensor" else None
    leaves = {"q": q, "k": k, "v": v, "lr": lr, "decay": decay, "beta": beta, "gate": gate, "S0": S0,
              "Z0": Z0, "buf": buf}
    for t in leaves.values():
        if t is not None:
            t.requires_grad_(True)
    y, st = harness.run_reference_cell(rm, q=q, k=k, v=v, lr=lr, decay=decay, beta=beta, gate=gate, S0=S0,
                                       Z0=Z0, buf=buf, window=e, heads=H, fmap_mode=mode, fmap_degree=deg,
                                       proj=proj)
    outs = {"y": y, "S_end": st.S, "Z_end": st.Z, "buf_out": st.omega_buffer}
    ups = {k2: torch.randn(o.shape, generator=g, dtype=DT) for k2, o in outs.items() if o is not None}
    torch.autograd.backward([outs[k2] for k2 in ups], [ups[k2] for k2 in ups])
    to_nt = lambda t: t.permute(0, 2, 1).reshape(N, T)            # [B,T,H] -> [(b h), T]
    flat = lambda t: t.reshape(N, T, -1)
    rec = {"meta": np.array([B, H, T, d, e, int(gate_on), int(mom), deg]), "fmap_mode": np.array(mode)}
    for key, t in leaves.items():
        if t is None:
            continue
        val, grad = t.detach(), t.grad
        if key in ("q", "k", "v"):
            val, grad = flat(val), flat(grad)
        elif key in ("lr", "decay", "beta", "gate"):
            val, grad = to_nt(val), to_nt(grad)
        rec[key] = val.numpy()
        rec["d_" + key] = grad.numpy()
    if proj is not None:
        rec["proj"] = proj.numpy()
    for key, o in outs.items():
        if o is None:
            continue
        rec[key] = (flat(o) if key == "y" else o).detach().numpy()
        rec["up_" + key] = (flat(ups[key]) if key == "y" else ups[key]).numpy()
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **rec)


MODULE_CASES = {
    # name: (cell, kwargs, B, T, state_kind)
    "module_omega_e3_elem_conv": ("OmegaRNNMemoryCell",
                                  dict(dim=32, dim_head=16, heads=2, omega_window=3, use_omega_gate=True,
                                       poly_mode="elementwise", poly_degree=2, qkv_conv_kernel=4), 2, 19, "random"),
    "module_titans_chunked": ("RNNMemoryCell",
                              dict(dim=32, dim_head=16, heads=2, use_momentum=True, qkv_conv_kernel=4,
                                   scan_chunk_len=5), 2, 17, "random"),
    "module_omega_init_state": ("OmegaRNNMemoryCell",
                                dict(dim=24, dim_head=8, heads=3, omega_window=4, use_omega_gate=True,
                                     use_momentum=False, qkv_conv_kernel=None), 1, 21, "init"),
}


def make_module(rm, name, cls, kw, B, T, state_kind, seed):
    torch.manual_seed(seed)
    cell = getattr(rm, cls)(**kw).to(DT)
    # non-default gate heads so every gate varies per token
    with torch.no_grad():
        for head in ("to_lr", "to_decay", "to_momentum", "to_omega_gate"):
            mod = getattr(cell, head, None)
            if mod is not None:
                mod[0].weight.normal_(0, 0.2)
    x = torch.randn(B, T, kw["dim"], dtype=DT, requires_grad=True)
    H, d = kw["heads"], kw["dim_head"]
    e = kw.get("omega_window", 1)
    mom = kw.get("use_momentum", True)
    if state_kind == "random":
        S = (0.1 * torch.randn(B * H, d, d, dtype=DT)).clamp(-10, 10)
        Z = 0.1 * torch.randn(B * H, d, d, dtype=DT) if mom else None
        buf = 0.1 * torch.randn(B * H, e - 1, d, d, dtype=DT) if e > 1 else None
        state = rm.RNNMemState(seq_index=3, S=S, Z=Z, omega_buffer=buf)
    else:
        state = None
    y, st = cell(x, state)
    up = torch.randn(y.shape, dtype=DT)
    y.backward(up)
    rec = {"x": x.detach().numpy(), "y": y.detach().numpy(), "up_y": up.numpy(), "d_x": x.grad.numpy(),
           "S_end": st.S.detach().numpy(), "seq_index": np.array(st.seq_index)}
    if st.Z is not None:
        rec["Z_end"] = st.Z.detach().numpy()
    if st.omega_buffer is not None:
        rec["buf_out"] = st.omega_buffer.detach().numpy()
    if state is not None:
        rec["S0"] = state.S.numpy()
        if state.Z is not None:
            rec["Z0"] = state.Z.numpy()
        if state.omega_buffer is not None:
            rec["buf"] = state.omega_buffer.numpy()
    for key, t in cell.state_dict().items():
        rec["sd." + key] = t.numpy()
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **rec)


LM_CASES = {
    # name: (RNNMemoryTransformer kwargs, B, T, decode steps)
    "lm_lmm_omega_e3_elem": (dict(num_tokens=256, dim=32, depth=2, block_type="lmm", heads=2, dim_head=16,
                                  omega_window=3, use_omega_gate=True, poly_mode="elementwise", poly_degree=2,
                                  qkv_conv_kernel=4), 2, 23, 5),
    "lm_lmm_titans": (dict(num_tokens=256, dim=24, depth=2, block_type="lmm", heads=3, dim_head=8,
                           use_momentum=True, qkv_conv_kernel=None), 1, 17, 4),
}


def make_lm(rt, name, kw, B, T, steps, seed):
    """The reference LM (rnn_transformer.py:720-862): next-token loss, logits and every
    parameter gradient; then `steps` one-token calls carrying the memory states (the
    cached path of generate, :880-886) on fixed tokens, with their logits."""
    torch.manual_seed(seed)
    m = rt.RNNMemoryTransformer(**kw).to(DT)
    with torch.no_grad():  # non-default gate heads so every gate varies per token
        for blk in m.layers:
            for head in ("to_lr", "to_decay", "to_momentum", "to_omega_gate"):
                mod = getattr(blk.memory, head, None)
                if mod is not None:
                    mod[0].weight.normal_(0, 0.2)
    tokens = torch.randint(0, kw["num_tokens"], (B, T))
    loss, logits, states, _ = m(tokens, return_loss=True, return_cache=True)
    loss.backward()
    rec = {"tokens": tokens.numpy(), "loss": np.array(loss.item()), "logits": logits.detach().numpy()}
    for key, p in m.named_parameters():
        rec["grad." + key] = p.grad.numpy()
    for key, t in m.state_dict().items():
        rec["sd." + key] = t.numpy()
    step_tokens = torch.randint(0, kw["num_tokens"], (steps, B, 1))
    with torch.no_grad():
        st, outs = None, []
        for s in range(steps):
            lg, st, _ = m(step_tokens[s], mem_states=st, return_cache=True)
            outs.append(lg.numpy())
    rec["step_tokens"] = step_tokens.numpy()
    rec["step_logits"] = np.stack(outs)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **rec)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ATLAS_RNN_REFERENCE"), required=False)
    args = ap.parse_args()
    if not args.reference:
        sys.exit("pass --reference <atlas-rnn checkout> or set ATLAS_RNN_REFERENCE")
    rm = harness.load_reference_rnn_memory(args.reference)
    for i, (name, case) in enumerate(CORE_CASES.items()):
        make_core(rm, name, *case, seed=100 + i)
        print("wrote", name)
    for i, (name, (cls, kw, B, T, sk)) in enumerate(MODULE_CASES.items()):
        make_module(rm, name, cls, kw, B, T, sk, seed=200 + i)
        print("wrote", name)
    rt = harness.load_reference_rnn_transformer(args.reference, rm)
    for i, (name, (kw, B, T, steps)) in enumerate(LM_CASES.items()):
        make_lm(rt, name, kw, B, T, steps, seed=300 + i)
        print("wrote", name)


if __name__ == "__main__":
    main()
