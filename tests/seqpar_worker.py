"""Worker for tests/test_seqpar_multigpu.py (one rank per GPU, torchrun).

Rank r runs its token slice through ``seq_parallel_memory`` over NCCL; rank 0
compares the gathered outputs and gradients with a single-GPU full-sequence call.
Prints one line 'SEQPAR_OK <max_err>' on rank 0 when every check passes.
"""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from atlas_rnn_b200 import memory_recurrence  # noqa: E402
from atlas_rnn_b200.parallel import seq_parallel_memory  # noqa: E402
from atlas_rnn_b200.workloads import CONFIGS, make_inputs, shrink  # noqa: E402


def rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def main():
    T = int(os.environ.get("SEQPAR_T", "4096"))
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    r, P = dist.get_rank(), dist.get_world_size()
    w = shrink(CONFIGS[2], B=1, H=4, T=T)
    inp = make_inputs(w, seed=11, device=dev, state_scale=0.1)
    names = ("k", "q", "v", "lr", "decay", "beta")
    lo, hi = r * T // P, (r + 1) * T // P
    loc = {n: inp[n][:, lo:hi].clone().requires_grad_(True) for n in names}
    Sr, S0, Z0 = (inp[n].clone().requires_grad_(True) for n in ("S0", "S0", "Z0"))
    y, S_end, Z_end = seq_parallel_memory(*(loc[n] for n in names), S_ref=Sr, S0=S0, Z0=Z0)
    gen = torch.Generator().manual_seed(5)
    dS = torch.randn(S_end.shape, generator=gen).to(dev) / P
    dZ = torch.randn(S_end.shape, generator=gen).to(dev) / P
    torch.autograd.backward([y, S_end, Z_end], [inp["dy"][:, lo:hi], dS, dZ])
    # full-sequence reference on every rank (same inputs)
    full = {n: inp[n].clone().requires_grad_(True) for n in names}
    Sr2, S02, Z02 = (inp[n].clone().requires_grad_(True) for n in ("S0", "S0", "Z0"))
    y2, S2, Z2, _ = memory_recurrence(*(full[n] for n in names), S_ref=Sr2, S0=S02, Z0=Z02)
    torch.autograd.backward([y2, S2, Z2], [inp["dy"], dS * P, dZ * P])  # sum of the ranks' dS / P
    errs = [rel(y, y2[:, lo:hi]), rel(S_end, S2), rel(Z_end, Z2), rel(Sr.grad, Sr2.grad), rel(S0.grad, S02.grad),
            rel(Z0.grad, Z02.grad)]
    errs += [rel(loc[n].grad, full[n].grad[:, lo:hi]) for n in names]
    worst = torch.tensor([max(errs)], device=dev)
    dist.all_reduce(worst, op=dist.ReduceOp.MAX)
    if r == 0:
        print("errs", [f"{e:.2e}" for e in errs], flush=True)
        print(("SEQPAR_OK" if worst.item() < 2e-2 else "SEQPAR_FAIL"), worst.item(), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
