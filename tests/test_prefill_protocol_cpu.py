"""The prefill kernel's barrier protocol, checked on CPU models
(``tests/prefill_protocol.py``).

* The kernel (one polling MMA issuer for both query tiles, one score buffer
  per tile, the producer arriving for tiles a query tile sits out) never
  stalls, whatever the chunk layout: long runs of K/V tiles that the earlier
  query tile sits out, segments only the later tile sees first, one or two
  query tiles, 2- and 4-stage rings.
* The alternative of one blocking issuer per query tile does stall once a
  tile sits out two K/V tiles in a row, which is why the kernel polls.
* The host therefore accepts every chunk order: nothing is refused before
  launch (``HALO_ERR_SPLIT`` is never returned)."""
from __future__ import annotations

import ctypes
import random

import pytest

import prefill_protocol as P


def _random_layout(rng, max_run=None):
    while True:
        segs = []
        for _ in range(rng.randint(1, 5)):
            n_u = rng.randint(1, 4)
            segs.append((n_u, rng.randint(0, n_u)))
        if max_run is None or P.max_sit_out_run(segs) <= max_run:
            return segs


def _stalls(segs, ST, seeds, **kw):
    for seed in range(seeds):
        try:
            P.simulate(segs, ST, seed=seed, **kw)
        except P.Stall:
            return True
    return False


@pytest.mark.parametrize("segs", [[(3, 2), (1, 0), (3, 3)], [(4, 1)], [(2, 2), (4, 0)]])
def test_blocking_per_tile_issuers_stall_on_two_sat_out_tiles_in_a_row(segs):
    assert P.max_sit_out_run(segs) >= 2
    assert _stalls(segs, ST=2, seeds=20)


@pytest.mark.parametrize("ST", [2, 4])
@pytest.mark.parametrize("has_b", [True, False])
def test_kernel_protocol_never_stalls(ST, has_b):
    rng = random.Random(17 + ST + has_b)
    layouts = [[(3, 2), (1, 0), (3, 3)], [(4, 1)], [(2, 2), (4, 0)], [(2, 0), (3, 3)],
               [(1, 0), (1, 0), (1, 0), (2, 2)], [(4, 0)]]
    layouts += [_random_layout(rng) for _ in range(60)]
    for segs in layouts:
        for seed in range(6):
            P.simulate_kernel(segs, ST, seed=seed, has_b=has_b)


def test_kernel_protocol_long_walks():
    """Walks longer than the ring many times over, with sit-out runs at the
    start, the middle and the end."""
    for segs in ([(40, 40)], [(30, 0), (10, 10)], [(10, 10), (12, 3), (8, 8)],
                 [(5, 1)] * 8):
        for ST in (2, 4):
            for seed in range(3):
                P.simulate_kernel(segs, ST, seed=seed)


def test_host_accepts_chunk_orders_the_earlier_kernel_refused():
    """Two query tiles (positions 1000..1255) over causal segments where the
    first tile sits out the last two short pages: accepted now (on a machine
    without a GPU the call gets as far as the CUDA driver; with one it would
    launch on fake pointers, so it is only made without)."""
    import torch
    from halo_b200 import _lib as L
    if torch.cuda.is_available():
        pytest.skip("would launch on fake pointers")
    lib = L.lib()
    D, H, H_kv = 128, 4, 2
    prob = L.PrefillProblem()
    prob.B, prob.H, prob.H_kv, prob.T_q, prob.D = 1, H, H_kv, 256, D
    prob.dtype = L.DTYPE_BF16
    prob.q = 0x10000
    prob.q_stride_b, prob.q_stride_h, prob.q_stride_t = H * 256 * D, 256 * D, D
    prob.q_pos0 = 1000
    prob.scale = 0.088

    def chunk(base, start, n):
        c = L.KVChunk()
        c.k, c.v = base, base + 0x800000
        c.k_stride_t = c.v_stride_t = D
        c.k_stride_h = c.v_stride_h = n * D
        c.k_stride_b = c.v_stride_b = H_kv * n * D
        c.start, c.len, c.causal = start, n, 1
        return c
    po = L.PrefillOut()
    po.mode, po.out_dtype, po.out = L.MERGE_FINALIZE, L.DTYPE_F32, 0x20000
    po.out_stride_b, po.out_stride_h, po.out_stride_t = H * 256 * D, 256 * D, D
    pages = (L.KVChunk * 3)(chunk(0x1000000, 0, 1000), chunk(0x3000000, 1128, 64),
                            chunk(0x5000000, 1192, 64))
    rc = lib.halo_prefill_attention(ctypes.byref(prob), pages, 3, ctypes.byref(po), None)
    assert rc != L.HALO_ERR_SPLIT
    assert rc == L.HALO_ERR_CUDA       # stops at the driver: no GPU here


def test_prefill_workspace_bytes():
    """Workspace size of the fp16 V staging: 256 bytes of flags plus one
    fp16 copy per coalesced segment (rounded up to 256 bytes), none for
    fp16 inputs; a too small or misaligned workspace is refused before any
    CUDA call."""
    from halo_b200 import _lib as L
    lib = L.lib()
    B, H, H_kv, D = 2, 8, 2, 128
    prob = L.PrefillProblem()
    prob.B, prob.H, prob.H_kv, prob.T_q, prob.D = B, H, H_kv, 100, D
    prob.dtype = L.DTYPE_BF16
    prob.q = 0x10000
    prob.q_stride_b, prob.q_stride_h, prob.q_stride_t = H * 100 * D, 100 * D, D
    prob.scale = 0.088

    def chunk(base, start, n, cap):
        c = L.KVChunk()
        c.k, c.v = base, base + 0x8000000
        c.k_stride_t = c.v_stride_t = D
        c.k_stride_h = c.v_stride_h = cap * D
        c.k_stride_b = c.v_stride_b = H_kv * cap * D
        c.start, c.len, c.causal = start, n, 1
        return c
    # two chunks contiguous in memory and position (one segment) + one apart
    a = chunk(0x1000000, 0, 300, 1000)
    b = chunk(0x1000000 + 300 * D * 2, 300, 200, 1000)
    c = chunk(0x9000000, 500, 37, 37)
    arr = (L.KVChunk * 3)(a, b, c)
    seg = lambda rows: (B * H_kv * rows * D * 2 + 255) // 256 * 256
    assert lib.halo_prefill_workspace_bytes(ctypes.byref(prob), arr, 3) == 256 + seg(500) + seg(37)
    prob.dtype = L.DTYPE_F16
    assert lib.halo_prefill_workspace_bytes(ctypes.byref(prob), arr, 3) == 0
    prob.dtype = L.DTYPE_BF16
    po = L.PrefillOut()
    po.mode, po.out_dtype, po.out = L.MERGE_FINALIZE, L.DTYPE_F32, 0x20000
    po.out_stride_b, po.out_stride_h, po.out_stride_t = H * 100 * D, 100 * D, D
    need = lib.halo_prefill_workspace_bytes(ctypes.byref(prob), arr, 3)
    rc = lib.halo_prefill_attention_ws(ctypes.byref(prob), arr, 3, ctypes.byref(po), 0x100000,
                                       need - 256, None)
    assert rc == L.HALO_ERR_WORKSPACE
    rc = lib.halo_prefill_attention_ws(ctypes.byref(prob), arr, 3, ctypes.byref(po), 0x100010,
                                       need, None)
    assert rc == L.HALO_ERR_MISALIGNED
