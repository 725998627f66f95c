"""Failure detection on the GPU without a fault.

The cross-GPU exchange merge (``halo_sharded_merge``) is given a world of two
whose second rank never runs: the rows it should store into this rank's
exchange buffer never arrive.  The kernel's polls are bounded (2 s of
``%globaltimer``); on expiry it records ``HALO_ERR_TIMEOUT`` in the device
error word, writes no output and returns.  The host reads the status, and the
context stays usable for the next call.  Collected near the end (it holds
the GPU for the length of the wait); the no-alloc test comes after it."""
from __future__ import annotations

import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_exchange_wait_for_absent_peer_times_out_with_status(cuda_device):
    from halo_b200 import _lib as L
    lib = L.lib()
    L.device_error()                                   # start from a clear word
    B, H, Dv, P = 1, 4, 128, 3
    g = torch.Generator().manual_seed(5)
    m = torch.randn(B, H, P, generator=g).to(cuda_device)
    l = (torch.rand(B, H, P, generator=g) + 0.5).to(cuda_device)
    o = torch.randn(B, H, P, Dv, generator=g).to(cuda_device)
    nbytes = lib.halo_exchange_bytes(2, B * H, Dv)
    assert nbytes > 0
    own = torch.zeros(nbytes, dtype=torch.uint8, device=cuda_device)
    peer = torch.zeros(nbytes, dtype=torch.uint8, device=cuda_device)   # nobody runs rank 1
    bufs = (ctypes.c_void_p * 2)(own.data_ptr(), peer.data_ptr())
    out = torch.full((B, H, Dv), 7.0, device=cuda_device)
    lse = torch.full((B, H), 7.0, device=cuda_device)
    torch.cuda.synchronize()
    t0 = time.monotonic()
    rc = lib.halo_sharded_merge(B, H, Dv, P, m.data_ptr(), l.data_ptr(), o.data_ptr(), 1, P, Dv,
                                P * Dv, 2, 0, bufs, L.DTYPE_F32, out.data_ptr(), out.stride(0),
                                out.stride(1), lse.data_ptr(), L.stream_handle(cuda_device))
    L.check(rc, "halo_sharded_merge")
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    assert L.device_error() == L.HALO_ERR_TIMEOUT
    assert 1.5 < waited < 60.0
    assert bool((out == 7.0).all()) and bool((lse == 7.0).all())     # nothing written

    # the context is still usable: a one-rank merge right after is exact
    one = torch.zeros(lib.halo_exchange_bytes(1, B * H, Dv), dtype=torch.uint8,
                      device=cuda_device)
    rc = lib.halo_sharded_merge(B, H, Dv, P, m.data_ptr(), l.data_ptr(), o.data_ptr(), 1, P, Dv,
                                P * Dv, 1, 0, (ctypes.c_void_p * 1)(one.data_ptr()), L.DTYPE_F32,
                                out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(),
                                L.stream_handle(cuda_device))
    L.check(rc, "halo_sharded_merge")
    torch.cuda.synchronize()
    assert L.device_error() == 0
    md, ld, od = m.double().cpu(), l.double().cpu(), o.double().cpu()
    M = md.amax(-1, keepdim=True)
    w = torch.exp(md - M)
    Lw = (w * ld).sum(-1)
    ref = (w.unsqueeze(-1) * od).sum(-2) / Lw.unsqueeze(-1)
    assert (out.double().cpu() - ref).abs().max().item() <= 1e-5
    assert (lse.double().cpu() - (M.squeeze(-1) + torch.log(Lw))).abs().max().item() <= 1e-5
