"""Host control flow of the drop-in classes against the reference's own
results (``tests/golden/host.json``, made by ``make_golden.py`` from
halo/scorer.py:36-88, refetcher.py:24-114, demoter.py:20-80,
kv_cache.py:69-219 and memory_tier.py:105-258 of lzbaclz/HALO): hotness
scores and hot sets, refetch predictions, and a multi-layer, multi-step
``update_hotness`` trace (telemetry and the block tier directory after
every call).  CPU only: these classes do bookkeeping, not attention."""
from __future__ import annotations

import json
import os
import sys

import pytest
import torch

import inputs as I

sys.path.insert(0, I.HERE)
from make_golden import gen_host  # noqa: E402

from halo_b200.demoter import HALODemoter
from halo_b200.kv_cache import HALOCache
from halo_b200.memory_tier import MemoryTier, TieredStorage
from halo_b200.policy import HALOConfig
from halo_b200.refetcher import HALORefetcher
from halo_b200.scorer import HALOScorer

MODS = (HALOConfig, HALOScorer, HALODemoter, HALORefetcher, HALOCache, MemoryTier, TieredStorage)


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(I.HERE, "host.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def ours():
    return gen_host(MODS)


def test_hotness_scores_and_hot_sets_match_reference(golden, ours):
    assert len(ours["snapshots"]) == len(golden["snapshots"]) == len(I.HOST_SCORE_CASES)
    for case, g, o in zip(I.HOST_SCORE_CASES, golden["snapshots"], ours["snapshots"]):
        assert torch.allclose(torch.tensor(o["score"]), torch.tensor(g["score"]),
                              rtol=0, atol=1e-6), case
        for key in ("hot", "hot_half", "hot_all", "predicted"):
            assert o[key] == g[key], (case, key)
    assert ours["jaccard"] == golden["jaccard"]


@pytest.mark.parametrize("trace", ["trace_quarter", "trace_identity"])
def test_update_hotness_trace_matches_reference(golden, ours, trace):
    """Demotions, refetch hits/misses and the tier of every block after each
    call equal the reference's (hot_ratio 0.25, and 1.0: nothing moves)."""
    assert len(ours[trace]) == len(golden[trace])
    for i, (g, o) in enumerate(zip(golden[trace], ours[trace])):
        assert o["hot"] == g["hot"], (trace, i)
        assert o["directory"] == g["directory"], (trace, i)
        assert o["telemetry"] == g["telemetry"], (trace, i)


def test_identity_ratio_never_demotes(ours):
    last = ours["trace_identity"][-1]["telemetry"]
    assert last["demoted_blocks"] == 0 and last["refetch_misses"] == 0


def test_reset_clears_bookkeeping():
    cfg = HALOConfig(**I.HOST_CONFIG)
    st = TieredStorage(tiers=[MemoryTier.GPU, MemoryTier.DRAM], num_layers=1, num_kv_heads=2,
                       head_dim=8, block_size=cfg.block_size, dtype=torch.float32,
                       device=torch.device("cpu"), max_blocks=16)
    cache = HALOCache(config=cfg, storage=st, scorer=HALOScorer(cfg),
                      demoter=HALODemoter(cfg, storage=st), refetcher=HALORefetcher(cfg, storage=st))
    for step in range(3):
        cache.update_hotness(0, I.host_trace_attention(step, 0, 64))
        cache.step()
    assert cache.demoted_blocks_total > 0 and cache.step_index == 3
    cache.reset()
    assert cache.step_index == 0 and cache.demoted_blocks_total == 0
    assert cache.refetched_blocks_total == 0
    assert json.dumps(cache.telemetry())          # JSON-serialisable
