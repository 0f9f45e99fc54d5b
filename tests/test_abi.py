"""CPU: the C-ABI library loads, exports every declared entry point, and its
struct layouts match the header; the product path has no CPU fallback."""
import ctypes
import os
import re
import subprocess
import tempfile

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "atlas_mem.h")


def declared_functions():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*|size_t|long long)\s+(atlas_\w+)\s*\(", src, re.M)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "atlas_mem_forward" in names and "atlas_mem_backward" in names
    assert len(names) >= 9


def test_library_exports_every_declared_symbol(native_lib):
    for name in declared_functions():
        assert hasattr(native_lib, name), name
    assert native_lib.atlas_mem_abi_version() == 2
    assert native_lib.atlas_mem_error_string(0) == b"ok"


def test_struct_layouts_match_header(native_lib):
    from atlas_rnn_b200 import _lib
    prog = r'''
#include <stdio.h>
#include <stddef.h>
#include "atlas_mem.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu %zu\n", sizeof(AtlasMemShape), sizeof(AtlasMemFwd), sizeof(AtlasMemBwd),
         offsetof(AtlasMemShape, chunk), offsetof(AtlasMemFwd, buf_out), offsetof(AtlasMemBwd, dbuf_in));
  printf("%zu %zu\n", offsetof(AtlasMemFwd, status), offsetof(AtlasMemBwd, status));
  return 0;
}
'''
    with tempfile.TemporaryDirectory() as td:
        c = os.path.join(td, "t.c")
        open(c, "w").write(prog)
        exe = os.path.join(td, "t")
        subprocess.run(["gcc", "-I", os.path.dirname(HEADER), c, "-o", exe], check=True)
        got = [int(x) for x in subprocess.run([exe], capture_output=True, text=True).stdout.split()]
    exp = [ctypes.sizeof(_lib.Shape), ctypes.sizeof(_lib.Fwd), ctypes.sizeof(_lib.Bwd),
           _lib.Shape.chunk.offset, _lib.Fwd.buf_out.offset, _lib.Bwd.dbuf_in.offset,
           _lib.Fwd.status.offset, _lib.Bwd.status.offset]
    assert got == exp


def test_null_arguments_rejected(native_lib):
    assert native_lib.atlas_mem_workspace_size(None, None, None, None) == 1
    assert native_lib.atlas_mem_read_status(None, None) == 1
    assert native_lib.atlas_mem_selftest_wait_timeout(None, 10, None) == 1
    assert native_lib.atlas_mem_forward(None, None, None, 0, None, 0, None) == 1


def test_no_cpu_fallback():
    from atlas_rnn_b200 import memory_recurrence
    x = torch.randn(1, 4, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        memory_recurrence(x, x, x, torch.rand(1, 4), torch.rand(1, 4), S_ref=torch.zeros(1, 8, 8),
                          S0=torch.zeros(1, 8, 8))


def test_scan_has_no_cpu_path():
    """The AssocScan drop-in runs only on the GPU kernels (no silent CPU fallback)."""
    import torch
    from atlas_rnn_b200 import AssocScan
    with pytest.raises(RuntimeError):
        AssocScan()(torch.ones(1, 2), torch.ones(1, 2, 3))
