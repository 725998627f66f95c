"""Chunk orders the prefill kernel refuses in one call (``HALO_ERR_SPLIT``)
run correctly through the wrapper, which splits them into one call per chunk
with a running state.  The layout is a paged cache: 32-row causal pages in
separate allocations, so near the query positions the earlier query tile of
a pair cannot see several pages in a row that the later tile sees."""
from __future__ import annotations

import pytest
import torch

import inputs as I  # noqa: F401  (puts tests/golden on the path for the oracle)
from oracle import attention as OA

pytestmark = pytest.mark.gpu


def test_prefill_paged_causal_pages_split_into_safe_calls(cuda_device):
    from halo_b200 import _lib as L
    from halo_b200 import ops
    g = torch.Generator().manual_seed(55)
    B, H, H_kv, D, T_q, T, page = 1, 4, 2, 128, 256, 1024, 32
    q = torch.randn(B, H, T_q, D, generator=g).bfloat16()
    k = torch.randn(B, H_kv, T, D, generator=g).bfloat16()
    v = torch.randn(B, H_kv, T, D, generator=g).bfloat16()
    pages, keep = [], []
    for a in range(0, T, page):
        # one allocation per page with a spare row, so no two pages coalesce
        kb = torch.empty(B, H_kv, page + 1, D, dtype=k.dtype, device=cuda_device)
        vb = torch.empty(B, H_kv, page + 1, D, dtype=v.dtype, device=cuda_device)
        kb[..., :page, :].copy_(k[..., a:a + page, :])
        vb[..., :page, :].copy_(v[..., a:a + page, :])
        keep += [kb, vb]
        pages.append((kb[..., :page, :], vb[..., :page, :], a, True))
    L.device_error()
    out, lse = ops.prefill_attention(q.to(cuda_device), pages, query_pos_offset=T - T_q,
                                     out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert L.device_error() == 0
    ro, rl = OA.full_attention_f64(q, k, v, q_pos=T - T_q)
    assert (out.cpu().double() - ro).abs().max().item() <= 2e-3
    fin = torch.isfinite(rl)
    assert (lse.cpu().double()[fin] - rl[fin]).abs().max().item() <= 1e-4
