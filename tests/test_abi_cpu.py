"""The C-ABI library loads and exports every function ``include/*.h``
declares; ctypes signatures in ``halo_b200._lib`` cover the same set.
No compute calls (no GPU needed)."""
from __future__ import annotations

import ctypes
import glob
import os
import re


ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*[A-Za-z_][\w \*]*?\b(halo_\w+)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return names


def test_header_declares_entry_points():
    names = _declared_functions()
    assert {"halo_chunked_decode", "halo_decode_workspace_bytes", "halo_lse_merge",
            "halo_last_error_string", "halo_device_error", "halo_version"} <= names


def test_library_exports_all_declared_symbols():
    from halo_b200 import _lib as L
    lib = L.lib()
    missing = [n for n in sorted(_declared_functions()) if not hasattr(lib, n)]
    assert not missing, f"library misses {missing}"
    # the Python binding declares a signature for every exported entry point
    assert set(L.SIGNATURES) == _declared_functions()
    assert lib.halo_version() >= 100


def test_invalid_arguments_are_reported_without_gpu():
    """Argument validation happens on the host before any CUDA call."""
    from halo_b200 import _lib as L
    lib = L.lib()
    prob = L.DecodeProblem()
    prob.B, prob.H, prob.H_kv, prob.D, prob.Dv, prob.dtype = 1, 6, 4, 128, 128, L.DTYPE_BF16
    rc = lib.halo_decode_workspace_bytes(ctypes.byref(prob), None, 0)
    assert rc == L.HALO_ERR_INVALID_ARG
    assert b"not divisible" in lib.halo_last_error_string()
    prob.H, prob.D, prob.Dv = 8, 40, 40
    assert lib.halo_decode_workspace_bytes(ctypes.byref(prob), None, 0) == L.HALO_ERR_UNSUPPORTED
    prob.D = prob.Dv = 128
    prob.q = 0x2000
    c = L.KVChunk()
    c.k = c.v = 0x1000
    c.k_stride_t = c.v_stride_t = 3          # 6 bytes: not 16-byte aligned
    c.len = 8
    arr = (L.KVChunk * 1)(c)
    assert lib.halo_decode_workspace_bytes(ctypes.byref(prob), arr, 1) == L.HALO_ERR_MISALIGNED
    c.k_stride_t = c.v_stride_t = 128
    c.k_stride_h = c.v_stride_h = 128 * 8
    c.k_stride_b = c.v_stride_b = 128 * 8 * 4
    arr = (L.KVChunk * 1)(c)
    assert lib.halo_decode_workspace_bytes(ctypes.byref(prob), arr, 1) > 0
