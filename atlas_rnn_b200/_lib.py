"""ctypes binding of the C ABI in include/atlas_mem.h (libatlas_mem.so).

The shared library is built in-tree (``atlas_rnn_b200/build.py``) and loaded
from this package directory. There is no fallback: if the library is missing
or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("ATLAS_MEM_LIB") or os.path.join(_HERE, "libatlas_mem.so")

FMAP = {"off": 0, "elementwise": 1, "tensor": 2}
GATE_NONE, GATE_TOKEN, GATE_WINDOW = 0, 1, 2
F32, BF16 = 0, 1


class Shape(ctypes.Structure):
    _fields_ = [("N", ctypes.c_int64), ("T", ctypes.c_int64), ("d_k", ctypes.c_int32),
                ("d_phi", ctypes.c_int32), ("d_v", ctypes.c_int32), ("window", ctypes.c_int32),
                ("fmap_mode", ctypes.c_int32), ("fmap_degree", ctypes.c_int32),
                ("gate_mode", ctypes.c_int32), ("momentum", ctypes.c_int32),
                ("dtype_io", ctypes.c_int32), ("chunk", ctypes.c_int32)]


_vp = ctypes.c_void_p


class Fwd(ctypes.Structure):
    _fields_ = [(n, _vp) for n in ("k", "q", "v", "lr", "decay", "beta", "gate", "S_ref", "S0", "Z0",
                                   "buf_in", "proj", "y", "S_end", "Z_end", "buf_out", "status")]


class Bwd(ctypes.Structure):
    _fields_ = [(n, _vp) for n in ("dy", "dS_end", "dZ_end", "dbuf_out", "dk", "dq", "dv", "dlr",
                                   "ddecay", "dbeta", "dgate", "dS_ref", "dS0", "dZ0", "dbuf_in",
                                   "status")]


_lib = None


def lib():
    """Load the library once; raise with the path if it is absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"atlas_rnn_b200: native library not built ({LIB_PATH}); run "
                "`python -m atlas_rnn_b200.build` (there is no non-CUDA fallback)")
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.POINTER
        sz = P(ctypes.c_size_t)
        L.atlas_mem_abi_version.restype = ctypes.c_int
        L.atlas_mem_error_string.restype = ctypes.c_char_p
        L.atlas_mem_error_string.argtypes = [ctypes.c_int]
        L.atlas_mem_workspace_size.argtypes = [P(Shape), sz, sz, sz]
        L.atlas_mem_forward.argtypes = [P(Shape), P(Fwd), _vp, ctypes.c_size_t, _vp, ctypes.c_size_t, _vp]
        L.atlas_mem_backward.argtypes = [P(Shape), P(Fwd), P(Bwd), _vp, ctypes.c_size_t, _vp,
                                         ctypes.c_size_t, _vp]
        L.atlas_mem_forward_local.argtypes = [P(Shape), P(Fwd), _vp, ctypes.c_size_t, _vp, ctypes.c_size_t,
                                              _vp, _vp, _vp, _vp]
        L.atlas_mem_forward_finish.argtypes = [P(Shape), P(Fwd), _vp, ctypes.c_size_t, _vp, ctypes.c_size_t,
                                               _vp]
        L.atlas_mem_backward_local.argtypes = [P(Shape), P(Fwd), P(Bwd), _vp, ctypes.c_size_t, _vp,
                                               ctypes.c_size_t, _vp, _vp, _vp, _vp]
        L.atlas_mem_backward_finish.argtypes = [P(Shape), P(Fwd), P(Bwd), _vp, ctypes.c_size_t, _vp,
                                                ctypes.c_size_t, ctypes.c_int, _vp]
        L.atlas_mem_final_state_raw.argtypes = [P(Shape), _vp, ctypes.c_size_t, _vp, _vp]
        L.atlas_mem_final_state_raw.restype = ctypes.c_int
        L.atlas_mem_forward_noalloc.argtypes = [P(Shape), P(Fwd), _vp]
        L.atlas_mem_forward_noalloc.restype = ctypes.c_int
        L.atlas_mem_noalloc_scratch_bytes.restype = ctypes.c_size_t
        L.atlas_mem_decode_step.argtypes = [P(Shape), P(Fwd), _vp]
        L.atlas_mem_decode_step.restype = ctypes.c_int
        L.atlas_scan_forward.argtypes = [_vp, _vp, _vp, _vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int, _vp]
        L.atlas_scan_forward.restype = ctypes.c_int
        L.atlas_scan_backward.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int, _vp]
        L.atlas_scan_backward.restype = ctypes.c_int
        L.atlas_mem_compose_carries.argtypes = [_vp, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int64,
                                                ctypes.c_int64, ctypes.c_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                                _vp, _vp]
        L.atlas_mem_compose_carries.restype = ctypes.c_int
        L.atlas_dwconv3_forward.argtypes = [_vp, ctypes.c_int, _vp, _vp, _vp, ctypes.c_int, _vp, _vp, _vp,
                                            ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _vp]
        L.atlas_dwconv3_forward.restype = ctypes.c_int
        L.atlas_dwconv3_backward.argtypes = [_vp, ctypes.c_int, _vp, _vp, _vp, ctypes.c_int, _vp, _vp, _vp,
                                             ctypes.c_int, _vp, _vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                             _vp]
        L.atlas_dwconv3_backward.restype = ctypes.c_int
        L.atlas_head_prep_forward.argtypes = [_vp, ctypes.c_int, _vp, _vp, ctypes.c_int, ctypes.c_int64,
                                              ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp]
        L.atlas_head_prep_forward.restype = ctypes.c_int
        L.atlas_head_prep_backward.argtypes = [_vp, ctypes.c_int, _vp, _vp, ctypes.c_int, _vp, _vp, ctypes.c_int64,
                                               ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp]
        L.atlas_head_prep_backward.restype = ctypes.c_int
        L.atlas_mem_selftest_umma.argtypes = [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_int, _vp, _vp]
        L.atlas_mem_selftest_umma.restype = ctypes.c_int
        L.atlas_fmap_tensor_workspace.argtypes = [ctypes.c_int, ctypes.c_int]
        L.atlas_fmap_tensor_workspace.restype = ctypes.c_size_t
        L.atlas_fmap_tensor_forward.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp, _vp, _vp, _vp]
        L.atlas_fmap_tensor_forward.restype = ctypes.c_int
        L.atlas_fmap_tensor_backward.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp, _vp, _vp,
                                                 _vp]
        L.atlas_fmap_tensor_backward.restype = ctypes.c_int
        i64, ci = ctypes.c_int64, ctypes.c_int
        L.atlas_omega_store_forward.argtypes = [_vp] * 11 + [i64, i64, i64, ci, ci, _vp]
        L.atlas_omega_store_forward.restype = ctypes.c_int
        L.atlas_omega_store_backward.argtypes = [_vp] * 18 + [i64, i64, i64, ci, ci, _vp]
        L.atlas_omega_store_backward.restype = ctypes.c_int
        L.atlas_affine_scan_forward.argtypes = [_vp] * 4 + [i64, i64, ci, ci, ci, _vp]
        L.atlas_affine_scan_forward.restype = ctypes.c_int
        L.atlas_affine_scan_backward.argtypes = [_vp] * 7 + [i64, i64, ci, ci, ci, _vp]
        L.atlas_affine_scan_backward.restype = ctypes.c_int
        L.atlas_mem_read_status.argtypes = [_vp, _vp]
        L.atlas_mem_read_status.restype = ctypes.c_int
        L.atlas_mem_selftest_wait_timeout.argtypes = [_vp, ctypes.c_int, _vp]
        L.atlas_mem_selftest_wait_timeout.restype = ctypes.c_int
        L.atlas_mem_profile_enable.argtypes = [ctypes.c_int]
        L.atlas_mem_profile_read.argtypes = [ctypes.c_int, P(ctypes.c_double), P(ctypes.c_longlong)]
        L.atlas_mem_launch_count.restype = ctypes.c_longlong
        L.atlas_mem_kernel_count.restype = ctypes.c_int
        L.atlas_mem_kernel_name.restype = ctypes.c_char_p
        L.atlas_mem_kernel_name.argtypes = [ctypes.c_int]
        for name in ("atlas_mem_profile_enable", "atlas_mem_profile_read", "atlas_mem_workspace_size", "atlas_mem_forward", "atlas_mem_backward",
                     "atlas_mem_forward_local", "atlas_mem_forward_finish", "atlas_mem_backward_local",
                     "atlas_mem_backward_finish"):
            getattr(L, name).restype = ctypes.c_int
        _lib = L
    return _lib


def check(code: int, what: str):
    if code != 0:
        msg = lib().atlas_mem_error_string(code).decode()
        raise RuntimeError(f"atlas_rnn_b200: {what} failed: {msg} (code {code})")


def ptr(t):
    """Device pointer of a tensor (or None)."""
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def workspace_sizes(shape: Shape):
    s, f, b = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
    check(lib().atlas_mem_workspace_size(ctypes.byref(shape), ctypes.byref(s), ctypes.byref(f),
                                         ctypes.byref(b)), "workspace_size")
    return s.value, f.value, b.value


_status_words = {}


def status_word(device):
    """The per-device int32 status word this package hands to every call
    (``status`` in the Fwd / Bwd structs). Kernels set it when a bounded wait
    for tensor-core work runs out; ``check_device_status`` reads it."""
    import torch
    idx = torch.device(device).index
    idx = torch.cuda.current_device() if idx is None else idx
    w = _status_words.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=f"cuda:{idx}")
        _status_words[idx] = w
    return w


def check_device_status(device=None, reset: bool = True):
    """Synchronise the current stream of ``device``, read its status word and
    raise RuntimeError (ATLAS_ERR_DEVICE) if a kernel reported a timed-out
    wait since the last check. The word is cleared afterwards unless
    ``reset`` is False."""
    import torch
    w = status_word(device if device is not None else torch.device("cuda"))
    stream = ctypes.c_void_p(torch.cuda.current_stream(w.device).cuda_stream)
    code = lib().atlas_mem_read_status(ptr(w), stream)
    if code != 0 and reset:
        w.zero_()
    check(code, "device status")


def profile_enable(on: bool):
    check(lib().atlas_mem_profile_enable(int(on)), "profile_enable")


def profile_read() -> dict:
    """{kernel name: (total event-timed ms, timed launches)} since the last reset."""
    L = lib()
    out = {}
    for i in range(L.atlas_mem_kernel_count()):
        ms, n = ctypes.c_double(), ctypes.c_longlong()
        check(L.atlas_mem_profile_read(i, ctypes.byref(ms), ctypes.byref(n)), "profile_read")
        out[L.atlas_mem_kernel_name(i).decode()] = (ms.value, n.value)
    return out


def launch_count() -> int:
    return int(lib().atlas_mem_launch_count())
