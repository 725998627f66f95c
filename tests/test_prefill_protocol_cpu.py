"""The prefill kernel's barrier protocol, checked on a CPU model
(``tests/prefill_protocol.py``), and the host-side chunk-order guard that
follows from it (``pf_order_ok`` in ``halo_b200/csrc/prefill.cu``).

* With the kernel's issuer, a query tile that sits out two or more K/V tiles
  in a row can stall the CTA (the model finds deadlocks), while layouts whose
  sit-out runs are at most one tile long never stall.
* ``halo_prefill_attention`` refuses exactly the layouts with longer runs
  (``HALO_ERR_SPLIT``, before any launch).
* An issuer that polls its next QK and P V and skips sat-out tiles without
  waiting never stalls, whatever the layout (the planned kernel fix)."""
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
def test_kernel_issuer_stalls_on_two_sat_out_tiles_in_a_row(segs):
    assert P.max_sit_out_run(segs) >= 2
    assert _stalls(segs, ST=2, seeds=20)


def test_kernel_issuer_never_stalls_with_runs_of_one():
    rng = random.Random(3)
    for _ in range(60):
        segs = _random_layout(rng, max_run=1)
        for ST in (2, 4):
            assert not _stalls(segs, ST, seeds=6), segs


@pytest.mark.parametrize("NB,SPT", [(2, 2), (1, 1)])
def test_polling_issuer_never_stalls(NB, SPT):
    rng = random.Random(11 + NB)
    for _ in range(40):
        segs = _random_layout(rng)
        for ST in (2, 4):
            assert not _stalls(segs, ST, seeds=4, NB=NB, SPT=SPT, issuer="polling"), segs


def _segment_chunk(L, kind, base, k, Q, D=128, H_kv=2):
    """A causal or full segment whose tiles two query tiles at positions
    Q..Q+255 (A: Q..Q+127, B: Q+128..Q+255) see as (B's tiles, A's tiles)."""
    if kind == "full":
        start, n, causal, seen = 0, 128 * k, 0, (k, k)
    elif kind == "tail":       # A sees all but the last tile
        start, n, causal, seen = Q + 192 - 128 * (k - 1), 128 * k, 1, (k, k - 1)
    else:                      # "bonly": one short page only B sees
        start, n, causal, seen = Q + 160, 64, 1, (1, 0)
    c = L.KVChunk()
    c.k, c.v = base, base + 0x4000000
    c.k_stride_t = c.v_stride_t = D
    c.k_stride_h = c.v_stride_h = n * D
    c.k_stride_b = c.v_stride_b = H_kv * n * D
    c.start, c.len, c.causal = start, n, causal
    return c, seen


def test_host_guard_refuses_exactly_the_long_runs():
    import torch
    from halo_b200 import _lib as L
    lib = L.lib()
    D, H, H_kv, Q = 128, 4, 2, 5000
    prob = L.PrefillProblem()
    prob.B, prob.H, prob.H_kv, prob.T_q, prob.D = 1, H, H_kv, 256, D
    prob.dtype = L.DTYPE_BF16
    prob.q = 0x10000
    prob.q_stride_b, prob.q_stride_h, prob.q_stride_t = H * 256 * D, 256 * D, D
    prob.q_pos0 = Q
    prob.scale = 0.088
    po = L.PrefillOut()
    po.mode, po.out_dtype, po.out = L.MERGE_FINALIZE, L.DTYPE_F32, 0x20000
    po.out_stride_b, po.out_stride_h, po.out_stride_t = H * 256 * D, 256 * D, D
    rng = random.Random(5)
    refused = accepted = 0
    for _ in range(200):
        chunks, segs = [], []
        for i in range(rng.randint(1, 6)):
            kind = rng.choice(["full", "tail", "bonly"])
            c, seen = _segment_chunk(L, kind, 0x100000000 + i * 0x10000000,
                                     rng.randint(2, 3), Q)
            chunks.append(c)
            segs.append(seen)
        long_run = P.max_sit_out_run(segs) > 1
        if not long_run and torch.cuda.is_available():
            continue               # would launch on fake pointers
        arr = (L.KVChunk * len(chunks))(*chunks)
        rc = lib.halo_prefill_attention(ctypes.byref(prob), arr, len(chunks), ctypes.byref(po),
                                        None)
        assert (rc == L.HALO_ERR_SPLIT) == long_run, (segs, rc)
        refused += long_run
        accepted += not long_run
    assert refused > 10
