"""Golden fixtures of the reference's affine_associative_scan (atlas_pytorch/affine_scan.py).

Imports the reference's affine_scan.py by path (it needs only torch), runs it in float64 on
seeded inputs with and without prev, and stores inputs, outputs and the autograd gradients
of <out, W> for a seeded W:

    python tests/golden/make_affine_golden.py --reference <path to atlas-rnn checkout>
"""
import argparse
import importlib.util
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    spec = importlib.util.spec_from_file_location("_ref_affine_scan",
                                                  os.path.join(args.reference, "atlas_pytorch", "affine_scan.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    for name, (N, T, R, D, with_prev, remove_prev) in {
        "affine_scan_prev_kept": (2, 7, 16, 24, True, False),
        "affine_scan_no_prev": (3, 5, 8, 32, False, False),
        "affine_scan_prev_removed": (1, 6, 32, 16, True, True),
    }.items():
        g = torch.Generator().manual_seed(len(name))
        eye = torch.eye(D, dtype=torch.float64)
        A = (0.9 * eye + 0.3 * torch.randn(N, T, D, D, generator=g, dtype=torch.float64) / D ** 0.5).float().double()
        B = torch.randn(N, T, R, D, generator=g, dtype=torch.float64).float().double()
        prev = torch.randn(N, R, D, generator=g, dtype=torch.float64).float().double() if with_prev else None
        leaves = [t.clone().requires_grad_(True) if t is not None else None for t in (A, B, prev)]
        out = mod.affine_associative_scan(leaves[0], leaves[1], prev=leaves[2], remove_prev=remove_prev)
        W = torch.randn(out.shape, generator=g, dtype=torch.float64)
        (out * W).sum().backward()
        arrs = {"A": A.numpy(), "B": B.numpy(), "out": out.detach().numpy(), "W": W.numpy(),
                "dA": leaves[0].grad.numpy(), "dB": leaves[1].grad.numpy(),
                "remove_prev": np.array(int(remove_prev))}
        if prev is not None:
            arrs["prev"], arrs["dprev"] = prev.numpy(), leaves[2].grad.numpy()
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrs)
        print(name, out.shape)


if __name__ == "__main__":
    main()
