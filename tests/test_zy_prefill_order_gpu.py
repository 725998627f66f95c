"""Chunk layouts in which a CTA's earlier query tile sits out several K/V
tiles in a row that the later tile sees -- paged caches (32-row causal
pages in separate allocations), pages out of position order, and a page
list that starts with pages only the later tile sees -- run in ONE call of
the prefill kernel (its single MMA issuer polls, so no order stalls it) and
match the oracle.  Also: bf16 V holding values fp16 cannot represent
(|v| >= 65536) takes the two-MMA bf16 route and stays exact to tolerance."""
from __future__ import annotations

import random

import pytest
import torch

import inputs as I  # noqa: F401  (puts tests/golden on the path for the oracle)
from oracle import attention as OA

pytestmark = pytest.mark.gpu


def _pages(k, v, page, order, dev):
    """One allocation per page with a spare row, so no two pages coalesce."""
    B, H_kv, T, D = k.shape
    pages, keep = [], []
    for a in order:
        kb = torch.empty(B, H_kv, page + 1, D, dtype=k.dtype, device=dev)
        vb = torch.empty(B, H_kv, page + 1, D, dtype=v.dtype, device=dev)
        kb[..., :page, :].copy_(k[..., a:a + page, :])
        vb[..., :page, :].copy_(v[..., a:a + page, :])
        keep += [kb, vb]
        pages.append((kb[..., :page, :], vb[..., :page, :], a, True))
    return pages, keep


@pytest.mark.parametrize("layout", ["in_order", "shuffled", "late_pages_first", "mixed"])
def test_prefill_paged_layouts_in_one_call(cuda_device, layout):
    from halo_b200 import _lib as L
    from halo_b200 import ops
    g = torch.Generator().manual_seed(55)
    B, H, H_kv, D, T_q, T, page = 1, 4, 2, 128, 256, 1024, 32
    q = torch.randn(B, H, T_q, D, generator=g).bfloat16()
    k = torch.randn(B, H_kv, T, D, generator=g).bfloat16()
    v = torch.randn(B, H_kv, T, D, generator=g).bfloat16()
    starts = list(range(0, T, page))
    if layout == "shuffled":
        random.Random(3).shuffle(starts)
    elif layout == "late_pages_first":        # pages only the later query tile sees lead
        starts = starts[-4:] + starts[:-4]
    keep_alive = []
    if layout == "mixed":                     # one big contiguous segment + pages
        kd, vd = k.to(cuda_device), v.to(cuda_device)
        chunks = [(kd[..., :T - 8 * page, :], vd[..., :T - 8 * page, :], 0, True)]
        pages, keep_alive = _pages(k, v, page, starts[-8:][::-1], cuda_device)
        chunks += pages
    else:
        chunks, keep_alive = _pages(k, v, page, starts, cuda_device)
    assert len(chunks) <= ops.PREFILL_MAX_CHUNKS
    L.device_error()
    n0 = L.launch_count()
    out, lse = ops.prefill_attention(q.to(cuda_device), chunks, query_pos_offset=T - T_q,
                                     out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert L.launch_count() - n0 == 2        # fp16 copy of V + one kp3_kernel launch
    assert L.device_error() == 0
    ro, rl = OA.full_attention_f64(q, k, v, q_pos=T - T_q)
    assert (out.cpu().double() - ro).abs().max().item() <= 2e-3
    fin = torch.isfinite(rl)
    assert (lse.cpu().double()[fin] - rl[fin]).abs().max().item() <= 1e-4


@pytest.mark.parametrize("big", [7.0e4, 1.0e6])
def test_prefill_bf16_values_beyond_fp16_take_the_bf16_route(cuda_device, big):
    """A few V entries of magnitude >= 65536 (bf16 can hold them, fp16
    cannot): the pre-pass flags the call and the kernel runs P V in bf16
    (P as high part + residual).  Errors scale with max|v|: within
    2e-3 + 1e-5 max|v| of the float64 oracle, finite everywhere."""
    from halo_b200 import _lib as L
    from halo_b200 import ops
    g = torch.Generator().manual_seed(66)
    B, H, H_kv, D, T_q, T = 1, 4, 2, 128, 200, 900
    q = torch.randn(B, H, T_q, D, generator=g).bfloat16()
    k = torch.randn(B, H_kv, T, D, generator=g).bfloat16()
    v = torch.randn(B, H_kv, T, D, generator=g)
    v[0, 1, 123, 7] = big
    v[0, 0, 800, 100] = -big
    v = v.bfloat16()
    kd, vd = k.to(cuda_device), v.to(cuda_device)
    L.device_error()
    out, lse = ops.prefill_attention(q.to(cuda_device), [(kd, vd, 0, True)],
                                     query_pos_offset=T - T_q, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert L.device_error() == 0
    assert torch.isfinite(out).all()
    ro, rl = OA.full_attention_f64(q, k, v, q_pos=T - T_q)
    vmax = v.float().abs().max().item()
    assert (out.cpu().double() - ro).abs().max().item() <= 2e-3 + 1e-5 * vmax
    assert (lse.cpu().double() - rl).abs().max().item() <= 1e-4
