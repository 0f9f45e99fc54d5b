"""GPU: the forward entry point that allocates nothing.

Some callers of this library own only their input and output buffers and
cannot call cudaMalloc: a plugin slot in a host framework that passes tensors
but no workspace, or a serving loop whose device memory is all reserved by its
own pool. ``atlas_mem_forward_noalloc`` serves them with scratch kept in a
fixed array inside the library. This test calls it through the C ABI twice in
a row, on two different inputs, and checks each result against the regular
``atlas_mem_forward`` (caller-provided workspace) on the same inputs, within
the fp32 tolerance used by the other parity tests (rel-L2 1e-5). It lives in
its own file so that pytest collects it last.
"""
import ctypes

import pytest
import torch

from tests.helpers import TOL_F32, rel_l2

pytestmark = pytest.mark.gpu


def _inputs(seed, N=4, T=200, d=32, e=4):
    g = torch.Generator().manual_seed(seed)
    rn = lambda *s: torch.randn(*s, generator=g)
    sig = lambda mu, s: torch.sigmoid(mu + s * rn(N, T))
    unit = lambda t: t / t.norm(dim=-1, keepdim=True)
    x = {"k": unit(rn(N, T, d)), "q": unit(rn(N, T, d)), "v": unit(rn(N, T, d)), "lr": 0.1 * sig(0, 1),
         "decay": sig(3, 0.5), "beta": sig(1, 0.5), "gate": sig(0, 1), "S0": 0.1 * rn(N, d, d),
         "Z0": 0.1 * rn(N, d, d), "buf": 0.1 * rn(N, e - 1, d, d)}
    return {k: v.cuda().contiguous() for k, v in x.items()}


def _shape(x, e=4):
    from atlas_rnn_b200 import _lib
    N, T, d = x["k"].shape
    return _lib.Shape(N=N, T=T, d_k=d, d_phi=d, d_v=d, window=e, fmap_mode=1, fmap_degree=2,
                      gate_mode=_lib.GATE_TOKEN, momentum=1, dtype_io=_lib.F32, chunk=0)


def _outputs(x, e=4):
    N, T, d = x["k"].shape
    return {"y": torch.empty(N, T, d, device="cuda"), "S_end": torch.empty(N, d, d, device="cuda"),
            "Z_end": torch.empty(N, d, d, device="cuda"), "buf_out": torch.empty(N, e - 1, d, d, device="cuda")}


def _fwd_struct(x, o):
    from atlas_rnn_b200 import _lib
    p = _lib.ptr
    return _lib.Fwd(k=p(x["k"]), q=p(x["q"]), v=p(x["v"]), lr=p(x["lr"]), decay=p(x["decay"]), beta=p(x["beta"]),
                    gate=p(x["gate"]), S_ref=p(x["S0"]), S0=p(x["S0"]), Z0=p(x["Z0"]), buf_in=p(x["buf"]),
                    proj=None, y=p(o["y"]), S_end=p(o["S_end"]), Z_end=p(o["Z_end"]), buf_out=p(o["buf_out"]))


def _regular_forward(lib, x):
    from atlas_rnn_b200 import _lib
    shape = _shape(x)
    saved_b, _, _ = _lib.workspace_sizes(shape)
    saved = torch.empty(saved_b, dtype=torch.uint8, device="cuda")
    o = _outputs(x)
    f = _fwd_struct(x, o)
    rc = lib.atlas_mem_forward(ctypes.byref(shape), ctypes.byref(f), _lib.ptr(saved), saved.numel(), None, 0, None)
    assert rc == 0
    return o


def test_forward_noalloc_matches_forward_twice(native_lib):
    from atlas_rnn_b200 import _lib
    lib = native_lib
    assert lib.atlas_mem_noalloc_scratch_bytes() == 32 << 20
    for seed in (1, 2):  # two calls in a row through the shared scratch array
        x = _inputs(seed)
        shape = _shape(x)
        o = _outputs(x)
        f = _fwd_struct(x, o)
        rc = lib.atlas_mem_forward_noalloc(ctypes.byref(shape), ctypes.byref(f), None)
        assert rc == 0, _lib.lib().atlas_mem_error_string(rc)
        torch.cuda.synchronize()
        ref = _regular_forward(lib, x)
        torch.cuda.synchronize()
        for name in ("y", "S_end", "Z_end", "buf_out"):
            assert rel_l2(o[name], ref[name]) < TOL_F32, (seed, name)


def test_forward_noalloc_rejects_oversized_shape(native_lib):
    from atlas_rnn_b200 import _lib
    x = _inputs(3, N=1, T=8)
    shape = _shape(x)
    shape.N = 4096
    shape.T = 65536  # forward workspace far above the fixed array
    o = _outputs(x)
    f = _fwd_struct(x, o)
    rc = native_lib.atlas_mem_forward_noalloc(ctypes.byref(shape), ctypes.byref(f), None)
    assert rc == 6
    assert b"no-alloc" in native_lib.atlas_mem_error_string(rc)


def _tc_case(seed, N, T, e=4):
    """bf16 io, d = 128, window gates, elementwise map: the shape the tensor-core kernels run."""
    from atlas_rnn_b200 import _lib
    from atlas_rnn_b200.workloads import Workload, make_inputs
    w = Workload("noalloc_tc", 1, N, T, 128, 128, 128, e, "window", "elementwise", 2, True, torch.bfloat16, 0)
    inp = make_inputs(w, seed=seed, device="cuda", state_scale=0.1)
    x = {"k": inp["k"], "q": inp["q"], "v": inp["v"], "lr": inp["lr"], "decay": inp["decay"],
         "beta": inp["beta"], "gate": inp["gate"], "S0": inp["S0"], "Z0": inp["Z0"], "buf": inp["omega_buffer"]}
    shape = _lib.Shape(N=N, T=T, d_k=128, d_phi=128, d_v=128, window=e, fmap_mode=1, fmap_degree=2,
                       gate_mode=_lib.GATE_WINDOW, momentum=1, dtype_io=_lib.BF16, chunk=0)
    o = {"y": torch.empty(N, T, 128, device="cuda", dtype=torch.bfloat16),
         "S_end": torch.empty(N, 128, 128, device="cuda"), "Z_end": torch.empty(N, 128, 128, device="cuda"),
         "buf_out": torch.empty(N, e - 1, 128, 128, device="cuda")}
    return inp, x, shape, o


def test_forward_noalloc_tensor_core_path(native_lib):
    """The tensor-core layout of the scratch (bf16 delta rows, state tiles, S_ref tile) run
    through the fixed array: T is not a multiple of the chunk, the array holds another,
    larger call's data before each checked call, and the results are compared with
    atlas_mem_forward (caller workspace) and with the CPU oracle at the bf16 tolerance."""
    from atlas_rnn_b200 import _lib
    from tests.helpers import TOL_BF16, oracle_run
    lib = native_lib
    for seed in (1, 2):
        # a larger call first, so the array is full of unrelated data
        _, xb, sb, ob = _tc_case(seed + 10, N=6, T=900)
        assert lib.atlas_mem_forward_noalloc(ctypes.byref(sb), ctypes.byref(_fwd_struct(xb, ob)), None) == 0
        inp, x, shape, o = _tc_case(seed, N=2, T=300)
        saved_b, _, _ = _lib.workspace_sizes(shape)
        assert saved_b <= lib.atlas_mem_noalloc_scratch_bytes()
        rc = lib.atlas_mem_forward_noalloc(ctypes.byref(shape), ctypes.byref(_fwd_struct(x, o)), None)
        assert rc == 0, lib.atlas_mem_error_string(rc)
        torch.cuda.synchronize()
        ref = {n: torch.empty_like(t) for n, t in o.items()}
        saved = torch.empty(saved_b, dtype=torch.uint8, device="cuda")
        rc = lib.atlas_mem_forward(ctypes.byref(shape), ctypes.byref(_fwd_struct(x, ref)), _lib.ptr(saved),
                                   saved.numel(), None, 0, None)
        assert rc == 0
        torch.cuda.synchronize()
        out_ref, _ = oracle_run(inp, 4, "window", "elementwise", 2, grads=False)
        for name in ("y", "S_end", "Z_end", "buf_out"):
            assert rel_l2(o[name].float(), ref[name].float()) < TOL_F32, (seed, name)
            assert rel_l2(o[name].float(), out_ref[name]) < TOL_BF16, (seed, name)
