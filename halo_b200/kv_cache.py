"""``HALOCache``: a ``transformers`` ``DynamicCache`` that carries HALO's
tiering handles (the interface of ``halo/kv_cache.py`` in lzbaclz/HALO,
:69-219).

Attention sees exactly what ``DynamicCache.update`` returns; the tiers
change only through :meth:`update_hotness`, which works on index tensors:
the positions that left the hot set (``torch.isin``) become the blocks to
demote one tier down, then the refetcher's prediction for the next step is
scheduled.  That order -- demote what cooled, then refetch what is
predicted -- is the policy's, and the telemetry counts follow from it.
"""
from __future__ import annotations

try:
    from transformers.cache_utils import DynamicCache as _BaseCache
except Exception:  # pragma: no cover - transformers is part of the runtime image
    class _BaseCache:  # type: ignore[no-redef]
        """Per-layer append-only K/V lists, concatenated on read (used only
        when transformers is not importable)."""

        def __init__(self) -> None:
            self._parts: list = []

        def update(self, key_states, value_states, layer_idx, *args, **kwargs):
            import torch
            while len(self._parts) <= layer_idx:
                self._parts.append(([], []))
            ks, vs = self._parts[layer_idx]
            ks.append(key_states)
            vs.append(value_states)
            if len(ks) > 1:       # keep one tensor per layer
                ks[:] = [torch.cat(ks, dim=-2)]
                vs[:] = [torch.cat(vs, dim=-2)]
            return ks[0], vs[0]

        def get_seq_length(self, layer_idx: int = 0) -> int:
            if layer_idx >= len(self._parts) or not self._parts[layer_idx][0]:
                return 0
            return int(self._parts[layer_idx][0][0].shape[-2])


def _tier_below(tiers, name: str) -> str:
    """The next slower tier after ``name`` in ``tiers`` (itself if last or
    absent)."""
    order = [str(getattr(t, "value", t)) for t in tiers]
    if name not in order:
        return name
    return order[min(order.index(name) + 1, len(order) - 1)]


class HALOCache(_BaseCache):
    """KV cache with HALO's scorer, demoter and refetcher attached."""

    def __init__(self, *, config, storage, scorer, demoter, refetcher) -> None:
        super().__init__()
        self.cfg = config
        self.storage = storage
        self.scorer = scorer
        self.demoter = demoter
        self.refetcher = refetcher
        self._step = 0
        self._last_hot_indices: dict = {}    # layer -> hot positions (int64, sorted)
        self._last_score: dict = {}          # layer -> hotness score (K,)
        self.demoted_blocks_total = 0
        self.refetched_blocks_total = 0

    def reset(self) -> None:
        """Empty the cache and the HALO bookkeeping (one call per generate)."""
        _BaseCache.__init__(self)
        self._step = 0
        self._last_hot_indices = {}
        self._last_score = {}
        self.demoted_blocks_total = 0
        self.refetched_blocks_total = 0

    def step(self) -> None:
        self._step += 1

    @property
    def step_index(self) -> int:
        return self._step

    def update_hotness(self, layer_idx: int, attn_weights) -> None:
        """Score this step's head-mean attention ``(K,)``; demote the blocks
        of positions that left the hot set, then schedule the refetch of the
        predicted next hot set."""
        import torch
        score = self.scorer.score(attn_weights, step=self._step)
        hot = self.scorer.topk_hot(score)
        prev = self._last_hot_indices.get(layer_idx)
        if prev is not None:
            cooled = prev[~torch.isin(prev, hot)]
            if cooled.numel():
                blocks = torch.unique(torch.div(cooled, self.cfg.block_size,
                                                 rounding_mode="floor")).tolist()
                self.demoter.demote(layer=layer_idx, block_indices=blocks, src="gpu",
                                    dst=_tier_below(self.cfg.tiers, "gpu"))
                self.demoted_blocks_total += len(blocks)
        misses = self.refetcher.misses
        self.refetcher.schedule(layer=layer_idx,
                                predicted_indices=self.refetcher.predict_hot(
                                    layer=layer_idx, last_hot_indices=hot, last_score=score))
        self.refetched_blocks_total += self.refetcher.misses - misses
        self._last_hot_indices[layer_idx] = hot
        self._last_score[layer_idx] = score

    def telemetry(self) -> dict:
        """JSON-able counters (the reference's keys)."""
        rf = self.refetcher
        n = rf.hits + rf.misses
        return {"step": self._step, "demoted_blocks": self.demoted_blocks_total,
                "refetched_blocks": self.refetched_blocks_total, "refetch_hits": rf.hits,
                "refetch_misses": rf.misses, "refetch_hit_rate": rf.hits / n if n else 0.0}


__all__ = ["HALOCache"]
