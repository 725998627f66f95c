"""``HALOCache``: a ``transformers`` ``DynamicCache`` with HALO's tiering
handles (``halo/kv_cache.py`` in lzbaclz/HALO, :69-219).

It returns exactly what ``DynamicCache.update`` returns, so attention sees
the same keys and values; HALO state changes only through
:meth:`update_hotness` (demote what cooled, prefetch what is predicted hot).
"""
from __future__ import annotations

try:
    from transformers.cache_utils import DynamicCache as _BaseCache
    _HAS_TRANSFORMERS = True
except Exception:  # pragma: no cover
    _HAS_TRANSFORMERS = False

    class _BaseCache:  # type: ignore[no-redef]
        """Minimal per-layer concatenating cache when transformers is absent."""

        def __init__(self) -> None:
            self.key_cache: list = []
            self.value_cache: list = []

        def update(self, key_states, value_states, layer_idx, *args, **kwargs):
            import torch
            while len(self.key_cache) <= layer_idx:
                self.key_cache.append(None)
                self.value_cache.append(None)
            if self.key_cache[layer_idx] is None:
                self.key_cache[layer_idx], self.value_cache[layer_idx] = key_states, value_states
            else:
                self.key_cache[layer_idx] = torch.cat([self.key_cache[layer_idx], key_states], -2)
                self.value_cache[layer_idx] = torch.cat([self.value_cache[layer_idx], value_states], -2)
            return self.key_cache[layer_idx], self.value_cache[layer_idx]

        def get_seq_length(self, layer_idx: int = 0) -> int:
            if layer_idx >= len(self.key_cache) or self.key_cache[layer_idx] is None:
                return 0
            return self.key_cache[layer_idx].shape[-2]


class HALOCache(_BaseCache):
    """KV cache carrying HALO's scorer, demoter and refetcher."""

    def __init__(self, *, config, storage, scorer, demoter, refetcher) -> None:
        super().__init__()
        self.cfg = config
        self.storage = storage
        self.scorer = scorer
        self.demoter = demoter
        self.refetcher = refetcher
        self._step = 0
        self._last_hot_indices: dict = {}
        self._last_score: dict = {}
        self.demoted_blocks_total = 0
        self.refetched_blocks_total = 0

    def reset(self) -> None:
        """Forget all cached layers and HALO bookkeeping (one per ``generate``)."""
        try:
            _BaseCache.__init__(self)
        except Exception:  # pragma: no cover
            for name in ("key_cache", "value_cache"):
                if isinstance(getattr(self, name, None), list):
                    getattr(self, name).clear()
        self._step = 0
        self._last_hot_indices.clear()
        self._last_score.clear()
        self.demoted_blocks_total = 0
        self.refetched_blocks_total = 0

    def step(self) -> None:
        self._step += 1

    @property
    def step_index(self) -> int:
        return self._step

    def update_hotness(self, layer_idx: int, attn_weights) -> None:
        """Score the head-mean attention ``(K,)``, demote blocks that left the
        hot set, prefetch the predicted next hot set."""
        score = self.scorer.score(attn_weights, step=self._step)
        hot = self.scorer.topk_hot(score)
        prev = self._last_hot_indices.get(layer_idx)
        if prev is not None:
            cooled = sorted(set(prev.tolist()) - set(hot.tolist()))
            if cooled:
                blocks = sorted({c // self.cfg.block_size for c in cooled})
                self.demoter.demote(layer=layer_idx, block_indices=blocks, src="gpu",
                                    dst=self._next_tier_after("gpu"))
                self.demoted_blocks_total += len(blocks)
        predicted = self.refetcher.predict_hot(layer=layer_idx, last_hot_indices=hot,
                                               last_score=score)
        before = self.refetcher.misses
        self.refetcher.schedule(layer=layer_idx, predicted_indices=predicted)
        self.refetched_blocks_total += self.refetcher.misses - before
        self._last_hot_indices[layer_idx] = hot
        self._last_score[layer_idx] = score

    def telemetry(self) -> dict:
        tot = self.refetcher.hits + self.refetcher.misses
        return {
            "step": self._step,
            "demoted_blocks": self.demoted_blocks_total,
            "refetched_blocks": self.refetched_blocks_total,
            "refetch_hits": self.refetcher.hits,
            "refetch_misses": self.refetcher.misses,
            "refetch_hit_rate": (self.refetcher.hits / tot) if tot else 0.0,
        }

    def _next_tier_after(self, current: str) -> str:
        names = list(self.cfg.tiers)
        if current not in names:
            return current
        return names[min(names.index(current) + 1, len(names) - 1)]


__all__ = ["HALOCache"]
