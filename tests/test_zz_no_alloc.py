"""halo_chunked_decode_noalloc: the decode entry point for callers that cannot
allocate device memory (their framework owns every allocation, their plugin
host forbids cudaMalloc on the hot path, or they call through a bare C ABI).
It must give the same answer as halo_chunked_decode with a caller workspace,
call after call, while its scratch lives in one fixed array inside the
library.  This file is collected last on purpose."""
from __future__ import annotations

import ctypes
import math

import pytest
import torch


def _problem(L, q, H_kv, q_pos, scale):
    p = L.DecodeProblem()
    p.B, p.H, p.D = q.shape
    p.H_kv, p.Dv = H_kv, q.shape[-1]
    p.dtype = L.halo_dtype(q.dtype)
    p.q = q.data_ptr()
    p.q_stride_b, p.q_stride_h = q.stride(0), q.stride(1)
    p.q_pos = q_pos.data_ptr() if q_pos is not None else None
    p.scale = scale
    return p


def _chunks(L, k, v, chunk, causal):
    T = k.shape[2]
    arr = []
    for a in range(0, T, chunk):
        c = L.KVChunk()
        kk, vv = k[:, :, a:], v[:, :, a:]
        c.k, c.v = kk.data_ptr(), vv.data_ptr()
        c.k_stride_b, c.k_stride_h, c.k_stride_t = k.stride(0), k.stride(1), k.stride(2)
        c.v_stride_b, c.v_stride_h, c.v_stride_t = v.stride(0), v.stride(1), v.stride(2)
        c.start, c.len, c.causal = a, min(chunk, T - a), int(causal)
        arr.append(c)
    return (L.KVChunk * len(arr))(*arr), len(arr)


def _merge(L, out, lse):
    mg = L.MergeArgs()
    mg.mode = L.MERGE_FINALIZE
    mg.out_dtype = L.halo_dtype(out.dtype)
    mg.out = out.data_ptr()
    mg.out_stride_b, mg.out_stride_h = out.stride(0), out.stride(1)
    mg.lse = lse.data_ptr()
    return mg


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_twice(cuda_device):
    from halo_b200 import _lib as L
    lib = L.lib()
    dev = cuda_device
    B, H, H_kv, D, T, chunk = 2, 16, 4, 128, 3000, 512
    stream = torch.cuda.current_stream(dev).cuda_stream
    g = torch.Generator(device=dev).manual_seed(11)
    k = torch.randn(B, H_kv, T, D, device=dev, generator=g).bfloat16()
    v = torch.randn(B, H_kv, T, D, device=dev, generator=g).bfloat16()
    arr, n = _chunks(L, k, v, chunk, causal=True)
    for call in range(2):   # two calls in a row: the shared scratch is reused
        q = torch.randn(B, H, D, device=dev, generator=g).bfloat16()
        q_pos = torch.tensor([T - 1, 900 + 700 * call], device=dev)
        prob = _problem(L, q, H_kv, q_pos, 1.0 / math.sqrt(D))
        need = lib.halo_decode_workspace_bytes(ctypes.byref(prob), arr, n)
        assert need > 0
        ws = torch.zeros(need, dtype=torch.uint8, device=dev)   # control block zeroed
        out_ref = torch.empty(B, H, D, dtype=torch.float32, device=dev)
        lse_ref = torch.empty(B, H, dtype=torch.float32, device=dev)
        L.check(lib.halo_chunked_decode(ctypes.byref(prob), arr, n, ws.data_ptr(), need,
                                        ctypes.byref(_merge(L, out_ref, lse_ref)), stream),
                "halo_chunked_decode")
        out = torch.full((B, H, D), float("nan"), dtype=torch.float32, device=dev)
        lse = torch.full((B, H), float("nan"), dtype=torch.float32, device=dev)
        L.check(lib.halo_chunked_decode_noalloc(ctypes.byref(prob), arr, n,
                                                ctypes.byref(_merge(L, out, lse)), stream),
                "halo_chunked_decode_noalloc")
        torch.cuda.synchronize(dev)
        assert (out - out_ref).abs().max().item() <= 2e-3
        assert (lse - lse_ref).abs().max().item() <= 1e-4
    assert L.device_error() == 0


@pytest.mark.gpu
def test_noalloc_dynamic_schedule_twice_matches_oracle(cuda_device):
    """A context long enough for the dynamically scheduled split-KV kernel
    (B1, 64 q-heads / 8 KV heads, head_dim 128, 32768 rows: 512 tiles per
    KV head against 8 x 37 needed), whose CTAs take row pieces from counters
    kept in the first 4 KB of the scratch.  Two calls in a row must both
    match the workspace entry point and the float64 oracle: the second call
    only works if the counters the first one used were cleared."""
    from halo_b200 import _lib as L
    from oracle import attention as OA
    lib = L.lib()
    dev = cuda_device
    B, H, H_kv, D, T, chunk = 1, 64, 8, 128, 32768, 4096
    stream = torch.cuda.current_stream(dev).cuda_stream
    g = torch.Generator().manual_seed(12)
    k = torch.randn(B, H_kv, T, D, generator=g).bfloat16()
    v = torch.randn(B, H_kv, T, D, generator=g).bfloat16()
    kd, vd = k.to(dev), v.to(dev)
    arr, n = _chunks(L, kd, vd, chunk, causal=False)
    G = H // H_kv
    for call in range(2):
        q = torch.randn(B, H, D, generator=g).bfloat16()
        qd = q.to(dev)
        prob = _problem(L, qd, H_kv, None, 1.0 / math.sqrt(D))
        need = lib.halo_decode_workspace_bytes(ctypes.byref(prob), arr, n)
        assert 0 < need <= 8 << 20
        ws = torch.zeros(need, dtype=torch.uint8, device=dev)
        out_ref = torch.empty(B, H, D, dtype=torch.float32, device=dev)
        lse_ref = torch.empty(B, H, dtype=torch.float32, device=dev)
        L.check(lib.halo_chunked_decode(ctypes.byref(prob), arr, n, ws.data_ptr(), need,
                                        ctypes.byref(_merge(L, out_ref, lse_ref)), stream),
                "halo_chunked_decode")
        out = torch.full((B, H, D), float("nan"), dtype=torch.float32, device=dev)
        lse = torch.full((B, H), float("nan"), dtype=torch.float32, device=dev)
        L.check(lib.halo_chunked_decode_noalloc(ctypes.byref(prob), arr, n,
                                                ctypes.byref(_merge(L, out, lse)), stream),
                "halo_chunked_decode_noalloc")
        torch.cuda.synchronize(dev)
        assert (out - out_ref).abs().max().item() <= 2e-3
        assert (lse - lse_ref).abs().max().item() <= 1e-4
        for hk in range(H_kv):
            hs = slice(hk * G, (hk + 1) * G)
            ro, rl = OA.full_attention_f64(q[:, hs], k[:, hk:hk + 1], v[:, hk:hk + 1])
            assert (out[:, hs].cpu().double() - ro[:, :, 0]).abs().max().item() <= 2e-3
            assert (lse[:, hs].cpu().double() - rl[:, :, 0]).abs().max().item() <= 1e-4
    assert L.device_error() == 0


def test_noalloc_rejects_problems_beyond_its_scratch():
    """A problem whose partials exceed the fixed 8 MiB scratch is refused
    before anything is enqueued (no GPU work, no allocation)."""
    from halo_b200 import _lib as L
    lib = L.lib()
    p = L.DecodeProblem()
    p.B, p.H, p.H_kv, p.D, p.Dv, p.dtype = 64, 64, 8, 128, 128, L.DTYPE_BF16
    p.q, p.q_stride_b, p.q_stride_h, p.scale = 0x10000, 64 * 128, 128, 0.088
    c = L.KVChunk()
    c.k = c.v = 0x20000
    c.k_stride_t = c.v_stride_t = 128
    c.k_stride_h = c.v_stride_h = 128 * 4096
    c.k_stride_b = c.v_stride_b = 128 * 4096 * 8
    c.len = 4096
    arr = (L.KVChunk * 1)(c)
    mg = L.MergeArgs()
    mg.mode, mg.out_dtype, mg.out = L.MERGE_FINALIZE, L.DTYPE_BF16, 0x30000
    rc = lib.halo_chunked_decode_noalloc(ctypes.byref(p), arr, 1, ctypes.byref(mg), None)
    assert rc == L.HALO_ERR_WORKSPACE
    assert b"8388608" in lib.halo_last_error_string()
