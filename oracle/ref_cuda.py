"""Build and load the reference's own Omega-16 CUDA kernels (test and reference-arm infrastructure).

The reference ships a PyTorch C++/CUDA extension, ``atlas_pytorch/cuda/atlas_omega.cpp`` +
``atlas_omega.cu`` (exact window 16, head 64, bf16 I/O; compile recipe
``atlas_pytorch/cuda/compile.py:24-46``). ``build()`` compiles those two source files where
they lie in the reference checkout, with the reference's own flags plus sm_100a code
generation, into ``oracle/_ref/omega16/``; nothing of the reference is copied into this
repository. ``load()`` imports the built module on a machine without the checkout.

``forward_backward`` restates the reference's autograd wrapper
(``atlas_pytorch/cuda/atlas_omega_autograd.py:98-204``): delta = S_ref phi_k - v in torch,
the forward kernel with bf16 checkpoints every 16 steps, the backward kernel, and the
torch terms of delta's gradient. Used only by ``bench.py --impl reference-cuda`` to time
the reference's GPU path.
"""
from __future__ import annotations

import glob
import importlib.util
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref", "omega16")
NAME = "atlas_omega_ref"


def reference_root() -> str | None:
    """The reference checkout: $ATLAS_RNN_REFERENCE, else a 'reference' folder beside this repository."""
    cand = os.environ.get("ATLAS_RNN_REFERENCE") or os.path.join(os.path.dirname(os.path.dirname(HERE)),
                                                                 "reference")
    src = os.path.join(cand, "atlas_pytorch", "cuda", "atlas_omega.cu")
    return cand if os.path.exists(src) else None


def built_path() -> str | None:
    hits = glob.glob(os.path.join(OUT, NAME + "*.so"))
    return hits[0] if hits else None


def build(verbose: bool = False) -> str | None:
    """Compile the reference extension into oracle/_ref/omega16 (skipped when it is up to date
    or the reference checkout is absent). Returns the .so path or None."""
    root = reference_root()
    have = built_path()
    if root is None:
        return have
    srcs = [os.path.join(root, "atlas_pytorch", "cuda", f) for f in ("atlas_omega.cpp", "atlas_omega.cu")]
    if have and os.path.getmtime(have) >= max(os.path.getmtime(s) for s in srcs):
        return have
    from torch.utils.cpp_extension import load
    os.makedirs(OUT, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    # the reference's flags (compile.py:36-45), code for sm_100a
    flags = ["-O3", "-lineinfo", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_BFLOAT16_OPERATORS__",
             "-U__CUDA_NO_BFLOAT162_CONVERSIONS__", "-D_C_=64", "-D_E_=16", "--use_fast_math",
             "-gencode", "arch=compute_100a,code=sm_100a"]
    load(name=NAME, sources=srcs, extra_cuda_cflags=flags, build_directory=OUT, verbose=verbose,
         is_python_module=True)
    return built_path()


def load():
    """Import the built extension (raises if it was not built)."""
    path = built_path()
    if path is None:
        raise RuntimeError("the reference Omega-16 extension is not built (oracle/ref_cuda.py build())")
    if NAME in sys.modules:
        return sys.modules[NAME]
    spec = importlib.util.spec_from_file_location(NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sys.modules[NAME] = mod
    return mod


def forward_backward(ext, phi_k, phi_q, v, S_ref, lr, decay, beta, gate, S0, Z0, dy):
    """One forward + backward of the reference's Omega-16 path (all bf16, [BH, T, 64] / [BH, T] /
    [BH, 64, 64]); returns (y, S_T, Z_T) and the input gradients."""
    BH, T, d = phi_k.shape
    delta = (torch.einsum("bde,bte->btd", S_ref, phi_k) - v).contiguous()
    bf = dict(device=phi_k.device, dtype=torch.bfloat16)
    y = torch.empty(BH, T, d, **bf)
    S_T = torch.empty(BH, d, d, **bf)
    Z_T = torch.empty(BH, d, d, **bf)
    n_ckpt = (T + 15) // 16
    S_ck = torch.empty(BH, n_ckpt, d, d, **bf)
    Z_ck = torch.empty(BH, n_ckpt, d, d, **bf)
    ext.forward_exact(phi_k, phi_q, delta, lr, decay, beta, gate, S0, Z0, y, S_T, Z_T, S_ck, Z_ck)
    dS_T, dZ_T = torch.zeros_like(S_T), torch.zeros_like(Z_T)
    g = {n: torch.empty_like(phi_k) for n in ("phi_k", "phi_q", "delta")}
    s = {n: torch.empty(BH, T, **bf) for n in ("lr", "decay", "beta", "gate")}
    dS0, dZ0 = torch.empty(BH, d, d, **bf), torch.empty(BH, d, d, **bf)
    ext.backward_exact(phi_k, phi_q, delta, lr, decay, beta, gate, S_T, Z_T, S_ck, Z_ck, dy, dS_T, dZ_T,
                       g["phi_k"], g["phi_q"], g["delta"], s["lr"], s["decay"], s["beta"], s["gate"], dS0, dZ0)
    dv = -g["delta"]
    dphi_k = g["phi_k"] + torch.einsum("bde,btd->bte", S_ref.transpose(1, 2), g["delta"])
    dS_ref = torch.einsum("btd,bte->bde", g["delta"], phi_k)
    return (y, S_T, Z_T), dict(phi_k=dphi_k, phi_q=g["phi_q"], v=dv, S_ref=dS_ref, S0=dS0, Z0=dZ0, **s)
