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


def _valid_problem(L):
    prob = L.DecodeProblem()
    prob.B, prob.H, prob.H_kv, prob.D, prob.Dv, prob.dtype = 1, 8, 2, 128, 128, L.DTYPE_BF16
    prob.q = 0x2000
    prob.scale = 0.088
    c = L.KVChunk()
    c.k = c.v = 0x100000
    c.k_stride_t = c.v_stride_t = 128
    c.k_stride_h = c.v_stride_h = 128 * 64
    c.k_stride_b = c.v_stride_b = 128 * 64 * 2
    c.len = 64
    return prob, (L.KVChunk * 1)(c)


def test_exchange_arguments_are_checked_before_any_launch():
    """halo_sharded_decode rejects a bad world / rank / buffer table before
    it launches the split-KV kernel; on a host without a GPU any launch
    would report HALO_ERR_CUDA instead."""
    from halo_b200 import _lib as L
    lib = L.lib()
    assert lib.halo_exchange_bytes(2, 64, 128) == 2 * 2 * 64 * 130 * 8 + 16
    for world, rows, dv in ((0, 64, 128), (9, 64, 128), (2, 0, 128), (2, 64, 257)):
        assert lib.halo_exchange_bytes(world, rows, dv) == L.HALO_ERR_INVALID_ARG
    prob, arr = _valid_problem(L)
    bufs2 = (ctypes.c_void_p * 2)(0x4000, 0x8000)
    null2 = (ctypes.c_void_p * 2)(0x4000, None)
    out = 0x10000
    cases = [
        (0, 0, bufs2, L.DTYPE_F32, out),      # world 0
        (2, 2, bufs2, L.DTYPE_F32, out),      # rank outside the world
        (9, 0, bufs2, L.DTYPE_F32, out),      # more ranks than the exchange holds
        (2, 1, null2, L.DTYPE_F32, out),      # a peer buffer missing
        (2, 0, bufs2, 7, out),                # unknown output dtype
        (2, 0, bufs2, L.DTYPE_F32, None),     # no output
    ]
    for world, rank, bufs, odt, o in cases:
        rc = lib.halo_sharded_decode(ctypes.byref(prob), arr, 1, 0x30000, 1 << 20, world, rank,
                                     bufs, odt, o, 1024, 128, None, None)
        assert rc == L.HALO_ERR_INVALID_ARG, (world, rank, odt)
        rc = lib.halo_sharded_merge(1, 8, 128, 4, 0x100, None, 0x200, 1, 4, 128, 512, world,
                                    rank, bufs, odt, o, 1024, 128, None, None)
        assert rc == L.HALO_ERR_INVALID_ARG, (world, rank, odt)
    rc = lib.halo_sharded_merge(1, 8, 300, 4, 0x100, None, 0x200, 1, 4, 300, 1200, 2, 0, bufs2,
                                L.DTYPE_F32, out, 2400, 300, None, None)
    assert rc == L.HALO_ERR_INVALID_ARG


def test_scorer_arguments_are_checked_before_any_launch():
    from halo_b200 import _lib as L
    lib = L.lib()
    # page mean: bad page size, negative first page, unknown dtype
    for page, begin, dt in ((0, 0, L.DTYPE_BF16), (16, -1, L.DTYPE_BF16), (16, 0, 9)):
        rc = lib.halo_page_mean(0x1000, 0, 0, 0, 1, 2, 64, dt, page, begin, 4, 0x2000, 0, 0, 0,
                                None)
        assert rc == L.HALO_ERR_INVALID_ARG
    # no pages: nothing to do, no launch
    assert lib.halo_page_mean(0x1000, 0, 0, 0, 1, 2, 64, L.DTYPE_BF16, 16, 0, 0, 0x2000, 0, 0,
                              0, None) == L.HALO_OK

    def press(H, H_kv, P, k, n_sink=1, topk=0x5000):
        return lib.halo_page_press_topk(0x1000, 0, 0, 0, 1, H, 1, H_kv, 64, L.DTYPE_BF16, 0x2000,
                                        0, 0, 0, P, 1.0, 0.5, 2.0, 64, n_sink, 0x3000, k, None,
                                        topk, None)
    assert press(6, 4, 10, 2) == L.HALO_ERR_INVALID_ARG          # H not a multiple of H_kv
    assert press(8, 2, 10, 11) == L.HALO_ERR_INVALID_ARG         # k > P
    assert press(8, 2, 10, 2, n_sink=-1) == L.HALO_ERR_INVALID_ARG
    assert press(8, 2, 10, 2, topk=None) == L.HALO_ERR_INVALID_ARG
    assert press(8, 2, 8193, 2) == L.HALO_ERR_UNSUPPORTED        # top-k holds 8192 pages
    assert press(8, 2, 0, 0) == L.HALO_OK
    rc = lib.halo_page_score_topk(0x1000, 0, 0, 0, 1, 8, 1, 2, 64, L.DTYPE_BF16, 0x2000, 0x3000,
                                  0, 0, 0, 16385, 0x4000, None, 4, None, 0x5000, None)
    assert rc == L.HALO_ERR_UNSUPPORTED                          # top-k holds 16384 pages


def test_kivi_arguments_are_checked_before_any_launch():
    from halo_b200 import _lib as L
    lib = L.lib()

    def quant(dtype=L.DTYPE_F16, bits=2, group=32, T=64, D=128):
        return lib.halo_kivi_quantize(0x1000, 0, 0, 0, 1, 2, T, D, dtype, bits, group, 0x2000, 0,
                                      0, 0, 0x3000, 0x4000, 0, 0, 0, None)
    assert quant(dtype=L.DTYPE_F32) == L.HALO_ERR_UNSUPPORTED    # fp16 / bf16 only
    assert quant(bits=3) == L.HALO_ERR_UNSUPPORTED
    assert quant(group=48) == L.HALO_ERR_INVALID_ARG             # must divide D
    assert quant(bits=2, group=8, D=64) == L.HALO_ERR_UNSUPPORTED   # 2-bit groups: x16
    assert quant(T=0) == L.HALO_OK                               # nothing to do

    prob = L.DecodeProblem()
    prob.B, prob.H, prob.H_kv, prob.D, prob.Dv, prob.dtype = 1, 8, 2, 128, 128, L.DTYPE_F16
    prob.q = 0x2000
    kt = L.KiviTensor(0x10000, 0x20000, 0x30000, 64 * 32, 64 * 32, 64 * 4, 64 * 4, 64)
    mg = L.MergeArgs()
    mg.mode, mg.out_dtype, mg.out = L.MERGE_FINALIZE, L.DTYPE_F32, 0x40000

    def decode(p=prob, k=kt, rows=64, bits=2, causal=0, merge=mg):
        return lib.halo_kivi_decode(ctypes.byref(p), ctypes.byref(k), ctypes.byref(kt), rows, bits,
                                    0, causal, 0x50000, 1 << 20, ctypes.byref(merge), None)
    assert decode(bits=3) == L.HALO_ERR_UNSUPPORTED
    assert decode(rows=65) == L.HALO_ERR_INVALID_ARG             # t_cap 64 does not cover 65
    bad = L.KiviTensor(0x10008, 0x20000, 0x30000, 64 * 32, 64 * 32, 64 * 4, 64 * 4, 64)
    assert decode(k=bad) == L.HALO_ERR_MISALIGNED
    assert decode(causal=1) == L.HALO_ERR_INVALID_ARG            # causal needs q_pos
    acc = L.MergeArgs()
    acc.mode = L.MERGE_ACCUMULATE                                # without m, l, o
    assert decode(merge=acc) == L.HALO_ERR_INVALID_ARG
    p96 = L.DecodeProblem()
    p96.B, p96.H, p96.H_kv, p96.D, p96.Dv, p96.dtype = 1, 8, 2, 96, 96, L.DTYPE_F16
    assert decode(p=p96) == L.HALO_ERR_UNSUPPORTED               # head_dim 64 / 128 only


def test_merge_arguments_are_checked_before_any_launch():
    from halo_b200 import _lib as L
    lib = L.lib()
    mg = L.MergeArgs()
    mg.mode, mg.out_dtype, mg.out = L.MERGE_FINALIZE, L.DTYPE_F32, 0x40000

    def merge(B=1, H=8, Dv=128, P=4, m=0x100, o=0x200, args=mg):
        return lib.halo_lse_merge(B, H, Dv, P, m, None, o, 1, P, Dv, P * Dv,
                                  ctypes.byref(args), None)
    assert merge(B=0) == L.HALO_ERR_INVALID_ARG
    assert merge(m=None) == L.HALO_ERR_INVALID_ARG
    assert merge(Dv=300) == L.HALO_ERR_UNSUPPORTED
    assert merge(Dv=130) == L.HALO_ERR_UNSUPPORTED               # 5 columns a lane: no kernel
    bad = L.MergeArgs()
    bad.mode = 7
    assert merge(args=bad) == L.HALO_ERR_INVALID_ARG
    prior = L.MergeArgs()
    prior.mode, prior.out_dtype, prior.out, prior.m = L.MERGE_FINALIZE, L.DTYPE_F32, 0x40000, 0x8
    assert merge(args=prior) == L.HALO_ERR_INVALID_ARG           # m without l and o
