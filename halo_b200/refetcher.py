"""Predictive refetcher: brings the blocks predicted hot back to the GPU
tier (the read path of ``halo/refetcher.py`` in lzbaclz/HALO, :24-114).

Prediction: the ``k`` best-scoring positions, ``k`` = the hot-set size
``max(int(hot_ratio * K), 1)`` widened by ``lookahead`` (every position at
``hot_ratio >= 1``), in position order.  Scheduling works on the set of
blocks those positions fall in: blocks already on the GPU tier count as
hits; the others, unless a refetch of theirs is still recorded in flight,
count as misses and move up -- grouped by source tier, each group as one
batched move (runs of consecutive blocks copy as one slab, see
``TieredStorage.move_blocks``) on the mover's side stream.  A block stays
recorded in flight until :meth:`wait`; the counts and the tier directory
after every call match the reference's per-block walk.
"""
from __future__ import annotations

from halo_b200.memory_tier import TierMover


class HALORefetcher:
    """Batched, asynchronous refetch of predicted-hot blocks."""

    def __init__(self, config, *, storage) -> None:
        self.cfg = config
        self.storage = storage
        self.hits = 0
        self.misses = 0
        self._inflight: set = set()          # (layer, block) refetches not yet waited for
        self._mover = None if storage is None else TierMover(
            storage, asynchronous=bool(config.async_refetch))

    def predict_hot(self, *, layer: int, last_hot_indices, last_score):
        """Positions expected hot next step (sorted ``int64`` tensor)."""
        import torch
        n = int(last_score.shape[-1])
        if self.cfg.hot_ratio >= 1.0:
            return torch.arange(n, dtype=torch.long, device=last_score.device)
        width = min(n, max(1, int(self.cfg.hot_ratio * n)) + int(self.cfg.lookahead))
        picked = torch.topk(last_score, k=width).indices
        return torch.sort(picked).values

    def schedule(self, *, layer: int, predicted_indices) -> None:
        """Refetch the predicted blocks that are not on the GPU tier."""
        import torch
        pos = torch.as_tensor(predicted_indices, dtype=torch.long).reshape(-1)
        if pos.numel() == 0:
            return
        blocks = torch.unique(torch.div(pos, self.cfg.block_size, rounding_mode="floor")).tolist()
        tiers = self.storage.locate_blocks(layer=layer, blocks=blocks)
        by_source: dict = {}
        for blk, tier in zip(blocks, tiers):
            if tier == "gpu":
                self.hits += 1
            elif (layer, blk) not in self._inflight:
                by_source.setdefault(tier, []).append(blk)
        for tier, group in by_source.items():
            self.misses += len(group)
            self._inflight.update((layer, b) for b in group)
            self._mover.move(layer, group, tier, "gpu")

    def wait(self) -> None:
        """Make the current stream wait for every refetch issued so far;
        the in-flight record is cleared."""
        if self._mover is not None:
            self._mover.fence()
        self._inflight.clear()

    @property
    def hit_rate(self) -> float:
        n = self.hits + self.misses
        return self.hits / n if n else 0.0

    def __repr__(self) -> str:  # pragma: no cover
        return (f"<HALORefetcher hits={self.hits} misses={self.misses} "
                f"in_flight={len(self._inflight)}>")


__all__ = ["HALORefetcher"]
