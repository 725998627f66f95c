"""GPU parity of the scorer-driven tiered decode step (halo_b200.tiered):
selected cold chunks equal the oracle's Quest top-k (modulo score ties),
the output equals the oracle's attention over hot + selected chunks, and the
delta refetch copies exactly the chunks that were not resident."""
from __future__ import annotations

import pytest
import torch

from oracle import attention as OA
from oracle import scorer as OS

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _layer(B=2, H_kv=2, D=64, C=64, P=16, seed=0, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(B, H_kv, P * C, D, generator=g)
    for h in range(H_kv):
        k[:, h, :, torch.randperm(D, generator=g)[:4]] *= 10
    v = torch.randn(B, H_kv, P * C, D, generator=g)
    return k.to(dtype), v.to(dtype)


def _oracle_select(q, k, C, hot, k_sel):
    H_kv = k.shape[1]
    kmin, kmax = OS.page_summaries(k.float().numpy(), C)
    qg = OS.gqa_mean_query(q.float().numpy()[:, :, None, :], H_kv, dtype="bf16")
    top, per_page = OS.select_topk(OS.score_pages(qg, kmin, kmax), k_sel, exclude=hot)
    return top, per_page


def _same_selection(got, want, per_page):
    if sorted(got) == sorted(want):
        return
    kth = min(per_page[i] for i in want)
    for i in set(got) ^ set(want):
        assert abs(per_page[i] - kth) / max(abs(kth), 1e-30) < 1e-6


def test_tiered_step_matches_oracle_and_refetches_the_delta():
    from halo_b200.tiered import TieredLayer
    B, H, H_kv, D, C, P, k_sel = 2, 8, 2, 64, 64, 16, 4
    hot = [0, 13, 14, 15]
    k, v = _layer(B, H_kv, D, C, P)
    lay = TieredLayer(k.to(DEV), v.to(DEV), chunk_size=C, hot_chunks=hot, n_slots=k_sel)
    assert lay.k_cold.is_pinned() and lay.v_cold.is_pinned()
    assert lay.cold == [c for c in range(P) if c not in hot]
    g = torch.Generator().manual_seed(5)
    prev = set()
    for step in range(4):
        q = torch.randn(B, H, D, generator=g).bfloat16()
        n_before = lay.stats["refetched_chunks"]
        out, lse, chosen = lay.step(q.to(DEV), k_sel=k_sel)
        want, per_page = _oracle_select(q, k, C, hot, k_sel)
        _same_selection(chosen, [int(i) for i in want], per_page)
        assert not set(chosen) & set(hot)
        assert lay.stats["refetched_chunks"] - n_before == len(set(chosen) - prev)
        prev = set(chosen)
        keep = torch.zeros(P * C, dtype=torch.bool)
        for c in hot + chosen:
            keep[c * C:(c + 1) * C] = True
        ro, rl = OA.full_attention_f64(q.unsqueeze(2), k, v, keep=keep)
        # bf16 output: the fp32 result within 2e-3, plus one bf16 rounding
        err = (out.float().cpu().double() - ro[:, :, 0]).abs().max().item()
        assert err <= 2e-3 + 2 ** -8 * ro.abs().max().item()
        assert (lse.cpu().double() - rl[:, :, 0]).abs().max().item() <= 1e-4
    from halo_b200 import _lib as L
    assert L.device_error() == 0


def test_tiered_step_reuses_resident_chunks():
    """The same query twice: the second step copies nothing."""
    from halo_b200.tiered import TieredLayer
    k, v = _layer(seed=3)
    lay = TieredLayer(k.to(DEV), v.to(DEV), chunk_size=64, hot_chunks=[0, 15], n_slots=6)
    q = torch.randn(2, 8, 64, generator=torch.Generator().manual_seed(1)).bfloat16().to(DEV)
    o1, l1, c1 = lay.step(q, k_sel=4)
    n1 = lay.stats["refetched_chunks"]
    o2, l2, c2 = lay.step(q, k_sel=4)
    assert c1 == c2 and lay.stats["refetched_chunks"] == n1 == 4
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


def test_nvme_tier_round_trip_through_hbm(tmp_path):
    """A block written in HBM goes to the NVMe tier through the pinned bounce
    buffer and comes back to HBM with one positioned read and one DMA."""
    from halo_b200.memory_tier import TieredStorage
    st = TieredStorage(tiers=["gpu", "dram", "nvme"], num_layers=2, num_kv_heads=4,
                       head_dim=128, block_size=64, dtype=torch.bfloat16,
                       device=torch.device(DEV), max_blocks=8, nvme_path=str(tmp_path / "nvme"))
    g = torch.Generator().manual_seed(5)
    k = torch.randn(4, 64, 128, generator=g).bfloat16().to(DEV)
    v = torch.randn(4, 64, 128, generator=g).bfloat16().to(DEV)
    st.write_new_block(layer=1, block=5, keys=k, values=v, tier="gpu")
    st.move_block(layer=1, block=5, src="gpu", dst="nvme")
    rk, rv = st.refetch_block(layer=1, block=5, device=torch.device(DEV))
    torch.cuda.synchronize()
    assert rk.is_cuda and torch.equal(rk, k) and torch.equal(rv, v)
    st.close()
